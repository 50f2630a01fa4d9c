// FP8 linear layers on tcgen05 (kind::f8f6f4), with per-tensor dynamic
// scaling:
//
//   amax      one pass per tensor, |x| max reduced with an integer atomic max
//             on the float bits (valid for non-negative floats);
//   quantize  scale = max(amax / FP8_MAX, FLT_MIN); q = sat(x / scale) in E4M3
//             or E5M2, optionally written transposed (32x32 shared-memory
//             tiles) so that every GEMM operand is K-major;
//   GEMM      the persistent tcgen05 GEMM of gemm_kernel.cuh with 8-bit
//             operands (128 values per 128-byte K row, K = 32 per MMA) and the
//             two operand scales multiplied into the fp32 accumulator in the
//             epilogue (read from device memory: no host synchronisation).
//
// A linear layer y = x W^T runs forward as E4M3 x E4M3; its input gradient
// dy W as E5M2 x E4M3 (W transposed); its weight gradient dy^T x as
// E5M2 x E4M3 (both transposed), accumulating into fp32.
//
// Reference parity: `_scaled_quantize` / `_fp8_linear_dot` and its custom VJP
// (src/representax/precision.py:127-221): the same per-tensor amax scaling,
// formats and fp32 accumulation.
#include <cuda_fp8.h>

#include <algorithm>
#include <cfloat>

#include "gemm_kernel.cuh"

namespace rx {
namespace gemm {

template <int KIND, int OUT>
static LaunchFn pick_fp8_epi(int epi) {
  constexpr int BN = 256, ST = 4;
  switch (epi) {
    case 0: return launch<BN, ST, false, false, 0, OUT, KIND>;
    case EPI_BIAS: return launch<BN, ST, false, false, EPI_BIAS, OUT, KIND>;
    case EPI_RESID: return launch<BN, ST, false, false, EPI_RESID, OUT, KIND>;
    case EPI_BIAS | EPI_RESID: return launch<BN, ST, false, false, EPI_BIAS | EPI_RESID, OUT, KIND>;
    default: return nullptr;
  }
}

template <int KIND>
static LaunchFn pick_fp8_out(int epi, int out) {
  if (out == OUT_BF16) return pick_fp8_epi<KIND, OUT_BF16>(epi);
  if (out == OUT_F32_ATOMIC && epi == 0) return launch<256, 4, false, false, 0, OUT_F32_ATOMIC, KIND>;
  return nullptr;
}

static LaunchFn pick_fp8(int a_fmt, int b_fmt, int epi, int out) {
  switch (fp8_kind(a_fmt, b_fmt)) {
    case fp8_kind(0, 0): return pick_fp8_out<fp8_kind(0, 0)>(epi, out);
    case fp8_kind(1, 0): return pick_fp8_out<fp8_kind(1, 0)>(epi, out);
    case fp8_kind(0, 1): return pick_fp8_out<fp8_kind(0, 1)>(epi, out);
    default: return nullptr;
  }
}

}  // namespace gemm

namespace fp8 {

__global__ void amax_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int64_t cols, int64_t ld,
                            unsigned int* __restrict__ amax_bits) {
  float m = 0.f;
  const int64_t n = rows * cols;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    m = fmaxf(m, fabsf(__bfloat162float(x[r * ld + c])));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(amax_bits, __float_as_uint(m));
}

// scale = max(amax / fmt_max, FLT_MIN) into scale_out (fp32).
__global__ void scale_kernel(const unsigned int* __restrict__ amax_bits, float fmt_max, float* scale_out) {
  scale_out[0] = fmaxf(__uint_as_float(amax_bits[0]) / fmt_max, FLT_MIN);
}

template <bool E5M2>
__device__ __forceinline__ uint8_t to_fp8(float v) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, E5M2 ? __NV_E5M2 : __NV_E4M3));
}

// Tiles of 32 x 32 through shared memory; TRANS writes out[c, r].
template <bool E5M2, bool TRANS>
__global__ void quantize_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int64_t cols, int64_t ldx,
                                const float* __restrict__ scale, uint8_t* __restrict__ out, int64_t ldo) {
  __shared__ uint8_t tile[32][33];
  const float sc = scale[0];
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32, c0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int j = ty; j < 32; j += 8) {
    const int64_t r = r0 + j, c = c0 + tx;
    uint8_t q = 0;
    if (r < rows && c < cols) q = to_fp8<E5M2>(__bfloat162float(x[r * ldx + c]) / sc);
    if constexpr (TRANS) {
      tile[j][tx] = q;
    } else if (r < rows && c < cols) {
      out[r * ldo + c] = q;
    }
  }
  if constexpr (TRANS) {
    __syncthreads();
    for (int j = ty; j < 32; j += 8) {
      const int64_t c = c0 + j, r = r0 + tx;  // output row = input column
      if (c < cols && r < rows) out[c * ldo + r] = tile[tx][j];
    }
  }
}

}  // namespace fp8

// amax of a bf16 matrix into scale[0] = max(amax / FMT_MAX, FLT_MIN).
void fp8_scale(const at::Tensor& x, at::Tensor& scale, at::Tensor& amax_scratch, bool e5m2) {
  check_bf16(x, "x");
  check_f32(scale, "scale");
  RX_CHECK(x.dim() == 2 && x.stride(1) == 1, "x must be a row-major matrix");
  RX_CHECK(amax_scratch.scalar_type() == at::kInt && amax_scratch.numel() >= 1, "amax scratch must be int32");
  const int device = x.get_device();
  c10::cuda::CUDAGuard guard(device);
  auto st = at::cuda::getCurrentCUDAStream(device).stream();
  RX_CUDA_CHECK(cudaMemsetAsync(amax_scratch.data_ptr(), 0, sizeof(unsigned int), st));
  const int64_t n = x.size(0) * x.size(1);
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4 * num_sms(device))));
  if (n > 0)
    fp8::amax_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.size(0),
                                             x.size(1), x.stride(0),
                                             reinterpret_cast<unsigned int*>(amax_scratch.data_ptr()));
  fp8::scale_kernel<<<1, 1, 0, st>>>(reinterpret_cast<const unsigned int*>(amax_scratch.data_ptr()),
                                     e5m2 ? 57344.f : 448.f, scale.data_ptr<float>());
  RX_CUDA_CHECK(cudaGetLastError());
}

// out (uint8, [R, C] or transposed [C, R]) = fp8(x / scale).
void fp8_quantize(const at::Tensor& x, const at::Tensor& scale, at::Tensor& out, bool e5m2, bool transpose) {
  check_bf16(x, "x");
  check_f32(scale, "scale");
  RX_CHECK(out.scalar_type() == at::kByte && out.is_cuda() && out.dim() == 2 && out.stride(1) == 1,
           "out must be a uint8 matrix");
  const int64_t R = x.size(0), Cc = x.size(1);
  RX_CHECK(transpose ? (out.size(0) == Cc && out.size(1) == R) : (out.size(0) == R && out.size(1) == Cc),
           "out shape does not match");
  if (R == 0 || Cc == 0) return;
  const int device = x.get_device();
  c10::cuda::CUDAGuard guard(device);
  auto st = at::cuda::getCurrentCUDAStream(device).stream();
  dim3 grid(static_cast<unsigned>((Cc + 31) / 32), static_cast<unsigned>((R + 31) / 32));
  dim3 block(32, 8);
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto op = out.data_ptr<uint8_t>();
#define RX_Q(E, T) fp8::quantize_kernel<E, T><<<grid, block, 0, st>>>(xp, R, Cc, x.stride(0), scale.data_ptr<float>(), \
                                                                      op, out.stride(0))
  if (e5m2) {
    if (transpose) RX_Q(true, true); else RX_Q(true, false);
  } else {
    if (transpose) RX_Q(false, true); else RX_Q(false, false);
  }
#undef RX_Q
  RX_CUDA_CHECK(cudaGetLastError());
}

// C[M, N] = epilogue(alpha * scales[0] * scales[1] * A . B^T) with 8-bit A [M, K]
// and B [N, K] (both K-major); formats 0 = E4M3, 1 = E5M2.
void gemm_fp8(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, int64_t a_fmt, int64_t b_fmt,
              int64_t epi, int64_t out_mode, double alpha, const at::Tensor& scales,
              const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
              const at::Tensor& status) {
  using namespace gemm;
  RX_CHECK(A.scalar_type() == at::kByte && B.scalar_type() == at::kByte, "fp8 operands are uint8 tensors");
  RX_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1 &&
               C.stride(1) == 1, "row-major matrices required");
  const int64_t M = C.size(0), N = C.size(1), K = A.size(1);
  RX_CHECK(A.size(0) == M && B.size(0) == N && B.size(1) == K, "fp8 gemm shapes do not match");
  RX_CHECK(K > 0, "empty fp8 gemm");  // row strides (multiples of 16 bytes) are checked by the tensor maps
  check_f32(scales, "scales");
  RX_CHECK(scales.numel() >= 2, "scales must hold the two operand scales");
  Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.C = C.data_ptr();
  p.ldc = C.stride(0);
  p.alpha = static_cast<float>(alpha);
  p.scales = scales.data_ptr<float>();
  p.status = status_ptr(status);
  p.timeout_ns = kWaitBudgetNs;
  if (out_mode == OUT_BF16) {
    check_bf16(C, "C");
    RX_CHECK(C.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0, "C alignment");
  } else {
    check_f32(C, "C");
    RX_CHECK(C.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0, "C alignment");
  }
  if (epi & EPI_BIAS) {
    RX_CHECK(bias.has_value() && bias->numel() == N && bias->is_contiguous(), "bias must be [N]");
    check_bf16(*bias, "bias");
    p.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  if (epi & EPI_RESID) {
    RX_CHECK(residual.has_value() && residual->size(0) == M && residual->size(1) == N && residual->stride(1) == 1 &&
                 residual->stride(0) % 8 == 0, "bad residual");
    check_bf16(*residual, "residual");
    p.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    p.ld_res = residual->stride(0);
  }
  constexpr int BN = 256;
  p.m_tiles = static_cast<int>((M + BM - 1) / BM);
  p.n_tiles = static_cast<int>((N + BN - 1) / BN);
  p.kb_total = static_cast<int>((K + 127) / 128);
  const int device = C.get_device();
  const int sms = num_sms(device);
  const int tiles = p.m_tiles * p.n_tiles;
  int splits = 1;
  if (out_mode == OUT_F32_ATOMIC && tiles < sms) splits = std::max(1, std::min(p.kb_total / 2, (sms + tiles - 1) / tiles));
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  p.splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;
  p.num_units = tiles * p.splits;
  LaunchFn fn = pick_fp8(static_cast<int>(a_fmt), static_cast<int>(b_fmt), static_cast<int>(epi),
                         static_cast<int>(out_mode));
  RX_CHECK(fn != nullptr, "unsupported fp8 gemm variant a=", a_fmt, " b=", b_fmt, " epi=", epi, " out=", out_mode);
  CUtensorMap ta = make_tmap_2d_u8(A.data_ptr(), M, K, A.stride(0), BM);
  CUtensorMap tb = make_tmap_2d_u8(B.data_ptr(), N, K, B.stride(0), BN);
  c10::cuda::CUDAGuard guard(device);
  fn(ta, tb, p, std::min(p.num_units, sms), at::cuda::getCurrentCUDAStream(device).stream(), device);
}

}  // namespace rx
