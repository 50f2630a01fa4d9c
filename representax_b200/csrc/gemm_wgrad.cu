// Weight-gradient (A MN-major, B MN-major) variants of the tcgen05 GEMM.
#include "gemm_kernel.cuh"

namespace rx {
namespace gemm {

LaunchFn pick_wgrad(int epi, int out) {
  if (epi != 0) return nullptr;
  switch (out) {
    case OUT_BF16: return launch<256, 4, true, true, 0, OUT_BF16>;
    case OUT_F32: return launch<256, 4, true, true, 0, OUT_F32>;
    case OUT_F32_ACC: return launch<256, 4, true, true, 0, OUT_F32_ACC>;
    case OUT_F32_ATOMIC: return launch<256, 4, true, true, 0, OUT_F32_ATOMIC>;
    default: return nullptr;
  }
}

LaunchFn pick_wgrad_pair(int epi, int out) {
  if (epi != 0) return nullptr;
  switch (out) {
    case OUT_BF16: return launch_pair<true, true, 0, OUT_BF16>;
    case OUT_F32: return launch_pair<true, true, 0, OUT_F32>;
    case OUT_F32_ACC: return launch_pair<true, true, 0, OUT_F32_ACC>;
    case OUT_F32_ATOMIC: return launch_pair<true, true, 0, OUT_F32_ATOMIC>;
    default: return nullptr;
  }
}

}  // namespace gemm
}  // namespace rx
