// Sequence pooling over packed token rows (mean / first token / last token),
// optional L2 normalisation, their backward passes, and small reductions
// (bias-gradient column sums, fp32 -> bf16 casts).
//
// Reference parity: `mean_pool` + `l2_normalize`
// (src/representax/models/components.py:238-258), last-valid-token pooling
// (src/representax/models/qwen3_vl/model.py:87-93) and CLS pooling
// (src/representax/models/sentence.py:47-132).
#include "common.h"
#include "sm100.cuh"

namespace rx {
namespace pool {

enum Mode : int { MEAN = 0, FIRST = 1, LAST = 2 };
constexpr int kThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float total = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) total += scratch[w];
  return total;
}

// out[b] = normalize(pool(h[cu[b] : cu[b+1]])), norm[b] = ||pool||.
// H <= 4 * kThreads * 2 handled by the per-thread column loop.
template <int MODE>
__global__ void __launch_bounds__(kThreads)
    pool_fwd_kernel(const __nv_bfloat16* __restrict__ h, const int* __restrict__ cu,
                    float* __restrict__ out, float* __restrict__ norm, int H, bool normalize) {
  __shared__ float scratch[32];
  const int b = blockIdx.x;
  const int s = cu[b], e = cu[b + 1];
  const int len = e - s;
  constexpr int kMaxPairs = 8;  // up to 4096 columns
  float acc[kMaxPairs][2];
#pragma unroll
  for (int i = 0; i < kMaxPairs; ++i) acc[i][0] = acc[i][1] = 0.f;
  const int pairs = H / 2;
  int t0 = s, t1 = e;
  if (MODE == FIRST) t1 = min(e, s + 1);
  if (MODE == LAST) t0 = max(s, e - 1);
  for (int t = t0; t < t1; ++t) {
    const __nv_bfloat162* row = reinterpret_cast<const __nv_bfloat162*>(h + static_cast<int64_t>(t) * H);
#pragma unroll
    for (int i = 0; i < kMaxPairs; ++i) {
      const int c = threadIdx.x + i * kThreads;
      if (c < pairs) {
        const float2 f = __bfloat1622float2(row[c]);
        acc[i][0] += f.x;
        acc[i][1] += f.y;
      }
    }
  }
  const float inv_len = (MODE == MEAN) ? 1.f / fmaxf(static_cast<float>(len), 1.f) : 1.f;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPairs; ++i) {
    acc[i][0] *= inv_len;
    acc[i][1] *= inv_len;
    sq += acc[i][0] * acc[i][0] + acc[i][1] * acc[i][1];
  }
  const float n = sqrtf(block_sum(sq, scratch));
  const float inv = normalize ? 1.f / fmaxf(n, 1e-12f) : 1.f;
#pragma unroll
  for (int i = 0; i < kMaxPairs; ++i) {
    const int c = threadIdx.x + i * kThreads;
    if (c < pairs) {
      reinterpret_cast<float2*>(out + static_cast<int64_t>(b) * H)[c] =
          make_float2(acc[i][0] * inv, acc[i][1] * inv);
    }
  }
  if (threadIdx.x == 0) norm[b] = n;
}

// Given d(out): dpool = (dout - out * <out, dout>) / max(norm, eps) when
// normalised, then dh[t] = dpool * weight(t) for the pooled tokens and 0 for
// the others.
template <int MODE>
__global__ void __launch_bounds__(kThreads)
    pool_bwd_kernel(const float* __restrict__ dout, const float* __restrict__ out,
                    const float* __restrict__ norm, const int* __restrict__ cu,
                    __nv_bfloat16* __restrict__ dh, int H, bool normalize) {
  __shared__ float scratch[32];
  const int b = blockIdx.x;
  const int s = cu[b], e = cu[b + 1];
  const int len = e - s;
  constexpr int kMaxPairs = 8;
  const int pairs = H / 2;
  float g[kMaxPairs][2];
  float dot = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPairs; ++i) {
    const int c = threadIdx.x + i * kThreads;
    g[i][0] = g[i][1] = 0.f;
    if (c < pairs) {
      const float2 d = reinterpret_cast<const float2*>(dout + static_cast<int64_t>(b) * H)[c];
      const float2 o = reinterpret_cast<const float2*>(out + static_cast<int64_t>(b) * H)[c];
      g[i][0] = d.x;
      g[i][1] = d.y;
      dot += d.x * o.x + d.y * o.y;
    }
  }
  if (normalize) {
    dot = block_sum(dot, scratch);
    const float inv = 1.f / fmaxf(norm[b], 1e-12f);
#pragma unroll
    for (int i = 0; i < kMaxPairs; ++i) {
      const int c = threadIdx.x + i * kThreads;
      if (c < pairs) {
        const float2 o = reinterpret_cast<const float2*>(out + static_cast<int64_t>(b) * H)[c];
        g[i][0] = (g[i][0] - o.x * dot) * inv;
        g[i][1] = (g[i][1] - o.y * dot) * inv;
      }
    }
  }
  const float w = (MODE == MEAN) ? 1.f / fmaxf(static_cast<float>(len), 1.f) : 1.f;
  for (int t = s; t < e; ++t) {
    bool take = true;
    if (MODE == FIRST) take = (t == s);
    if (MODE == LAST) take = (t == e - 1);
    __nv_bfloat162* row = reinterpret_cast<__nv_bfloat162*>(dh + static_cast<int64_t>(t) * H);
#pragma unroll
    for (int i = 0; i < kMaxPairs; ++i) {
      const int c = threadIdx.x + i * kThreads;
      if (c < pairs) row[c] = take ? __floats2bfloat162_rn(g[i][0] * w, g[i][1] * w)
                                   : __floats2bfloat162_rn(0.f, 0.f);
    }
  }
}

// out[col] += sum_rows x[row, col]  (bf16 input, fp32 accumulator).
// Each thread owns one 16-byte column chunk (8 columns) and walks a strided
// set of rows with vector loads, so a warp reads whole row segments; the CTA
// then reduces its row groups in shared memory and adds one atomic per column.
constexpr int kColsumThreads = 256;
__global__ void __launch_bounds__(kColsumThreads)
    colsum_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld, int rows, int cols,
                  float* __restrict__ out) {
  extern __shared__ float part[];  // [groups][cols]
  const int chunks = cols >> 3;
  const int groups = kColsumThreads / chunks;  // row groups per CTA (>= 1)
  const int tid = threadIdx.x;
  const int c = tid % chunks;
  const int grp = tid / chunks;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (grp < groups) {
    // Four rows in flight per thread: with one group per CTA (2048 columns)
    // a single outstanding load per thread leaves HBM mostly idle.
    const int stride = gridDim.x * groups;
    for (int r = blockIdx.x * groups + grp; r < rows; r += 4 * stride) {
      uint4 w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int rr = r + u * stride;
        w[u] = rr < rows ? reinterpret_cast<const uint4*>(x + static_cast<int64_t>(rr) * ld)[c]
                         : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w[u]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          acc[2 * j] += f.x;
          acc[2 * j + 1] += f.y;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) part[grp * cols + c * 8 + j] = acc[j];
  }
  __syncthreads();
  for (int col = tid; col < cols; col += kColsumThreads) {
    float s = 0.f;
    for (int g = 0; g < groups; ++g) s += part[g * cols + col];
    atomicAdd(out + col, s);
  }
}

__global__ void cast_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst,
                                 int64_t n) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i + 3 < n) {
    const float4 v = *reinterpret_cast<const float4*>(src + i);
    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&lo);
    w.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(dst + i) = w;
  } else {
    for (int64_t j = i; j < n; ++j) dst[j] = __float2bfloat16_rn(src[j]);
  }
}

}  // namespace pool

void pool_forward(const at::Tensor& h, const at::Tensor& cu_seqlens, at::Tensor& out,
                  at::Tensor& norm, int64_t mode, bool normalize) {
  check_bf16(h, "h");
  check_f32(out, "out");
  const int64_t H = h.size(1);
  RX_CHECK(H % 2 == 0 && H <= 4096, "pool width must be even and <= 4096");
  RX_CHECK(h.is_contiguous() && out.is_contiguous(), "pool tensors must be contiguous");
  const int batch = static_cast<int>(cu_seqlens.numel() - 1);
  if (batch <= 0) return;
  c10::cuda::CUDAGuard guard(h.get_device());
  auto st = at::cuda::getCurrentCUDAStream().stream();
  auto* hp = reinterpret_cast<const __nv_bfloat16*>(h.data_ptr());
  const int* cu = cu_seqlens.data_ptr<int>();
  switch (mode) {
    case pool::MEAN: pool::pool_fwd_kernel<pool::MEAN><<<batch, pool::kThreads, 0, st>>>(hp, cu, out.data_ptr<float>(), norm.data_ptr<float>(), H, normalize); break;
    case pool::FIRST: pool::pool_fwd_kernel<pool::FIRST><<<batch, pool::kThreads, 0, st>>>(hp, cu, out.data_ptr<float>(), norm.data_ptr<float>(), H, normalize); break;
    case pool::LAST: pool::pool_fwd_kernel<pool::LAST><<<batch, pool::kThreads, 0, st>>>(hp, cu, out.data_ptr<float>(), norm.data_ptr<float>(), H, normalize); break;
    default: RX_CHECK(false, "unknown pooling mode");
  }
  RX_CUDA_CHECK(cudaGetLastError());
}

void pool_backward(const at::Tensor& dout, const at::Tensor& out, const at::Tensor& norm,
                   const at::Tensor& cu_seqlens, at::Tensor& dh, int64_t mode, bool normalize) {
  check_f32(dout, "dout");
  check_bf16(dh, "dh");
  const int64_t H = dh.size(1);
  RX_CHECK(dout.is_contiguous() && out.is_contiguous() && dh.is_contiguous(), "pool tensors must be contiguous");
  const int batch = static_cast<int>(cu_seqlens.numel() - 1);
  if (batch <= 0) return;
  c10::cuda::CUDAGuard guard(dh.get_device());
  auto st = at::cuda::getCurrentCUDAStream().stream();
  auto* dhp = reinterpret_cast<__nv_bfloat16*>(dh.data_ptr());
  const int* cu = cu_seqlens.data_ptr<int>();
  switch (mode) {
    case pool::MEAN: pool::pool_bwd_kernel<pool::MEAN><<<batch, pool::kThreads, 0, st>>>(dout.data_ptr<float>(), out.data_ptr<float>(), norm.data_ptr<float>(), cu, dhp, H, normalize); break;
    case pool::FIRST: pool::pool_bwd_kernel<pool::FIRST><<<batch, pool::kThreads, 0, st>>>(dout.data_ptr<float>(), out.data_ptr<float>(), norm.data_ptr<float>(), cu, dhp, H, normalize); break;
    case pool::LAST: pool::pool_bwd_kernel<pool::LAST><<<batch, pool::kThreads, 0, st>>>(dout.data_ptr<float>(), out.data_ptr<float>(), norm.data_ptr<float>(), cu, dhp, H, normalize); break;
    default: RX_CHECK(false, "unknown pooling mode");
  }
  RX_CUDA_CHECK(cudaGetLastError());
}

void colsum_accumulate(const at::Tensor& x, at::Tensor& out) {
  check_bf16(x, "x");
  check_f32(out, "out");
  RX_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.size(1) % 8 == 0 && x.stride(0) % 8 == 0 &&
               reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
           "colsum needs a 16-byte aligned [rows, cols % 8 == 0] matrix");
  RX_CHECK(out.numel() == x.size(1) && out.is_contiguous(), "colsum output must be [cols]");
  const int rows = static_cast<int>(x.size(0)), cols = static_cast<int>(x.size(1));
  if (rows == 0) return;
  constexpr int kMaxCols = pool::kColsumThreads * 8;
  if (cols > kMaxCols) {  // wide matrices: independent column blocks
    for (int c0 = 0; c0 < cols; c0 += kMaxCols) {
      const int c1 = std::min(cols, c0 + kMaxCols);
      at::Tensor xs = x.narrow(1, c0, c1 - c0);
      at::Tensor os = out.narrow(0, c0, c1 - c0);
      colsum_accumulate(xs, os);
    }
    return;
  }
  c10::cuda::CUDAGuard guard(x.get_device());
  const int groups = pool::kColsumThreads / (cols / 8);
  const size_t smem = static_cast<size_t>(groups) * cols * sizeof(float);
  const int sms = num_sms(x.get_device());
  const int grid = std::max(1, std::min((rows + groups - 1) / groups, 2 * sms));
  auto kern = pool::colsum_kernel;
  if (smem > 48 * 1024)
    RX_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  kern<<<grid, pool::kColsumThreads, smem, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), rows, cols, out.data_ptr<float>());
  RX_CUDA_CHECK(cudaGetLastError());
}

void cast_bf16(const at::Tensor& src, at::Tensor& dst) {
  check_f32(src, "src");
  check_bf16(dst, "dst");
  RX_CHECK(src.is_contiguous() && dst.is_contiguous() && src.numel() == dst.numel(), "cast shape mismatch");
  const int64_t n = src.numel();
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(src.get_device());
  const int64_t blocks = (n / 4 + 1 + 255) / 256;
  pool::cast_bf16_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      src.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()), n);
  RX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace rx
