// Forward (A K-major, B K-major) variants of the tcgen05 GEMM.
#include "gemm_kernel.cuh"

namespace rx {
namespace gemm {

template <int OUT>
static LaunchFn pick_epi(int epi) {
  constexpr int BN = 256, ST = 4;
  switch (epi) {
    case 0: return launch<BN, ST, false, false, 0, OUT>;
    case EPI_BIAS: return launch<BN, ST, false, false, EPI_BIAS, OUT>;
    case EPI_BIAS | EPI_GELU: return launch<BN, ST, false, false, EPI_BIAS | EPI_GELU, OUT>;
    case EPI_BIAS | EPI_RESID: return launch<BN, ST, false, false, EPI_BIAS | EPI_RESID, OUT>;
    case EPI_RESID: return launch<BN, ST, false, false, EPI_RESID, OUT>;
    case EPI_BIAS | EPI_DROP | EPI_RESID:
      if constexpr (OUT == OUT_BF16) return launch<BN, ST, false, false, EPI_BIAS | EPI_DROP | EPI_RESID, OUT>;
      return nullptr;
    default: return nullptr;
  }
}

LaunchFn pick_forward(int epi, int out) {
  if (out == OUT_BF16) return pick_epi<OUT_BF16>(epi);
  if (out == OUT_F32) return pick_epi<OUT_F32>(epi);
  if (out == OUT_F32_ACC && epi == 0) return launch<256, 4, false, false, 0, OUT_F32_ACC>;
  return nullptr;
}

template <int OUT>
static LaunchFn pick_epi_pair(int epi) {
  switch (epi) {
    case 0: return launch_pair<false, false, 0, OUT>;
    case EPI_BIAS: return launch_pair<false, false, EPI_BIAS, OUT>;
    case EPI_BIAS | EPI_GELU: return launch_pair<false, false, EPI_BIAS | EPI_GELU, OUT>;
    case EPI_BIAS | EPI_RESID: return launch_pair<false, false, EPI_BIAS | EPI_RESID, OUT>;
    case EPI_RESID: return launch_pair<false, false, EPI_RESID, OUT>;
    case EPI_BIAS | EPI_DROP | EPI_RESID:
      if constexpr (OUT == OUT_BF16) return launch_pair<false, false, EPI_BIAS | EPI_DROP | EPI_RESID, OUT>;
      return nullptr;
    default: return nullptr;
  }
}

LaunchFn pick_forward_pair(int epi, int out) {
  if (out == OUT_BF16) return pick_epi_pair<OUT_BF16>(epi);
  if (out == OUT_F32) return pick_epi_pair<OUT_F32>(epi);
  if (out == OUT_F32_ACC && epi == 0) return launch_pair<false, false, 0, OUT_F32_ACC>;
  return nullptr;
}

}  // namespace gemm
}  // namespace rx
