// Input-gradient (A K-major, B MN-major) variants of the tcgen05 GEMM.
#include "gemm_kernel.cuh"

namespace rx {
namespace gemm {

LaunchFn pick_dgrad(int epi, int out) {
  if (epi == EPI_RESID && out == OUT_BF16) return launch<256, 4, false, true, EPI_RESID, OUT_BF16>;
  if (epi != 0 && epi != EPI_DGELU) return nullptr;
  const bool dgelu = epi == EPI_DGELU;
  switch (out) {
    case OUT_BF16:
      return dgelu ? launch<256, 4, false, true, EPI_DGELU, OUT_BF16>
                   : launch<256, 4, false, true, 0, OUT_BF16>;
    case OUT_F32:
      return dgelu ? launch<256, 4, false, true, EPI_DGELU, OUT_F32>
                   : launch<256, 4, false, true, 0, OUT_F32>;
    case OUT_F32_ACC:
      return dgelu ? nullptr : launch<256, 4, false, true, 0, OUT_F32_ACC>;
    default:
      return nullptr;
  }
}

LaunchFn pick_dgrad_pair(int epi, int out) {
  if (epi == EPI_RESID && out == OUT_BF16) return launch_pair<false, true, EPI_RESID, OUT_BF16>;
  if (epi == (EPI_DGELU | EPI_COLSUM) && out == OUT_BF16) return launch_pair<false, true, EPI_DGELU | EPI_COLSUM, OUT_BF16>;
  if (epi != 0 && epi != EPI_DGELU) return nullptr;
  const bool dgelu = epi == EPI_DGELU;
  switch (out) {
    case OUT_BF16:
      return dgelu ? launch_pair<false, true, EPI_DGELU, OUT_BF16> : launch_pair<false, true, 0, OUT_BF16>;
    case OUT_F32:
      return dgelu ? launch_pair<false, true, EPI_DGELU, OUT_F32> : launch_pair<false, true, 0, OUT_F32>;
    case OUT_F32_ACC:
      return dgelu ? nullptr : launch_pair<false, true, 0, OUT_F32_ACC>;
    default:
      return nullptr;
  }
}

}  // namespace gemm
}  // namespace rx
