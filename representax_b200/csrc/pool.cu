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

// The pooled rows are processed in slices of kSliceRows consecutive packed
// rows (a slice may span sequences), one CTA per slice, 16-byte accesses:
// the thread for column chunk c (8 columns) of row group g walks rows
// g, g + G, ... of the slice. Sequence boundaries come from a binary search of
// cu_seqlens held in shared memory.
constexpr int kSliceRows = 32;
constexpr int kMaxBatch = 4096;  // cu_seqlens entries a slice kernel can hold

__device__ __forceinline__ int seq_of(const int* s_cu, int batch, int row) {
  int lo = 0, hi = batch;  // s_cu[lo] <= row < s_cu[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (s_cu[mid] <= row) lo = mid; else hi = mid;
  }
  return lo;
}

__device__ __forceinline__ void load_cu(const int* cu, int batch, int* s_cu) {
  for (int i = threadIdx.x; i <= batch; i += blockDim.x) s_cu[i] = cu[i];
  __syncthreads();
}

// MEAN, phase 1: acc[b] += sum of the slice's rows of sequence b (fp32
// atomics, one per column per sequence run per thread). Rows are loaded four
// at a time before they are accumulated, so each thread keeps four 16-byte
// loads in flight.
__device__ __forceinline__ void sum_rows(const __nv_bfloat16* __restrict__ h, const int* s_cu, int batch,
                                         float* __restrict__ acc, int H, int c, int first, int end, int step) {
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  int run = -1;
  for (int r = first; r < end; r += 4 * step) {
    uint4 w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int rr = r + u * step;
      w[u] = rr < end ? reinterpret_cast<const uint4*>(h + static_cast<int64_t>(rr) * H)[c] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int rr = r + u * step;
      if (rr >= end) break;
      const int b = seq_of(s_cu, batch, rr);
      if (b != run) {
        if (run >= 0) {
          float* dst = acc + static_cast<int64_t>(run) * H + c * 8;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            atomicAdd(dst + j, a[j]);
            a[j] = 0.f;
          }
        }
        run = b;
      }
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&w[u]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(p2[j]);
        a[2 * j] += f.x;
        a[2 * j + 1] += f.y;
      }
    }
  }
  if (run >= 0) {
    float* dst = acc + static_cast<int64_t>(run) * H + c * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) atomicAdd(dst + j, a[j]);
  }
}

__global__ void __launch_bounds__(kThreads)
    pool_sum_kernel(const __nv_bfloat16* __restrict__ h, const int* __restrict__ cu, int batch, int total,
                    float* __restrict__ acc, int H) {
  extern __shared__ int s_cu[];
  load_cu(cu, batch, s_cu);
  const int chunks = H >> 3;
  const int r0 = blockIdx.x * kSliceRows, r1 = min(total, r0 + kSliceRows);
  if (chunks <= kThreads) {  // `groups` row groups of one thread per column chunk
    const int groups = kThreads / chunks;
    const int g = threadIdx.x / chunks;
    if (g < groups) sum_rows(h, s_cu, batch, acc, H, threadIdx.x % chunks, r0 + g, r1, groups);
  } else {
    for (int c = threadIdx.x; c < chunks; c += kThreads) sum_rows(h, s_cu, batch, acc, H, c, r0, r1, 1);
  }
}

// Phase 2 (every mode): one CTA per sequence. MEAN divides the accumulated
// sum by the length; FIRST / LAST read their one row from h. Then the L2
// norm and the optional normalisation; out and norm are written.
template <int MODE>
__global__ void __launch_bounds__(kThreads)
    pool_finish_kernel(const __nv_bfloat16* __restrict__ h, const int* __restrict__ cu,
                       float* __restrict__ out, float* __restrict__ norm, int H, bool normalize) {
  __shared__ float scratch[32];
  const int b = blockIdx.x;
  const int s = cu[b], e = cu[b + 1];
  const int len = e - s;
  float* row = out + static_cast<int64_t>(b) * H;
  const int row_src = MODE == FIRST ? s : e - 1;
  const float inv_len = 1.f / fmaxf(static_cast<float>(len), 1.f);
  float sq = 0.f;
  for (int c = threadIdx.x; c < H; c += kThreads) {
    float v;
    if (MODE == MEAN) {
      v = row[c] * inv_len;
    } else {
      v = len > 0 ? __bfloat162float(h[static_cast<int64_t>(row_src) * H + c]) : 0.f;
    }
    row[c] = v;
    sq += v * v;
  }
  const float n = sqrtf(block_sum(sq, scratch));
  if (normalize) {
    const float inv = 1.f / fmaxf(n, 1e-12f);
    for (int c = threadIdx.x; c < H; c += kThreads) row[c] *= inv;
  }
  if (threadIdx.x == 0) norm[b] = n;
}

// Backward, phase 1: g[b] = (dout - out <out, dout>) / max(norm, eps) when
// normalised, times 1 / len for MEAN (the weight of every pooled token).
template <int MODE>
__global__ void __launch_bounds__(kThreads)
    pool_grad_kernel(const float* __restrict__ dout, const float* __restrict__ out,
                     const float* __restrict__ norm, const int* __restrict__ cu, float* __restrict__ g,
                     int H, bool normalize) {
  __shared__ float scratch[32];
  const int b = blockIdx.x;
  const int len = cu[b + 1] - cu[b];
  const float* d = dout + static_cast<int64_t>(b) * H;
  const float* o = out + static_cast<int64_t>(b) * H;
  float dot = 0.f;
  if (normalize)
    for (int c = threadIdx.x; c < H; c += kThreads) dot += d[c] * o[c];
  dot = normalize ? block_sum(dot, scratch) : 0.f;
  const float inv = normalize ? 1.f / fmaxf(norm[b], 1e-12f) : 1.f;
  const float w = MODE == MEAN ? 1.f / fmaxf(static_cast<float>(len), 1.f) : 1.f;
  for (int c = threadIdx.x; c < H; c += kThreads) g[static_cast<int64_t>(b) * H + c] = (d[c] - o[c] * dot) * inv * w;
}

// Backward, phase 2: every row of a slice gets g[its sequence] (MEAN) or
// g / 0 (FIRST / LAST: only the pooled row is non-zero), as bf16.
template <int MODE>
__global__ void __launch_bounds__(kThreads)
    pool_rows_kernel(const float* __restrict__ g, const int* __restrict__ cu, int batch, int total,
                     __nv_bfloat16* __restrict__ dh, int H) {
  extern __shared__ int s_cu[];
  load_cu(cu, batch, s_cu);
  const int chunks = H >> 3;
  const int r0 = blockIdx.x * kSliceRows, r1 = min(total, r0 + kSliceRows);
  const int items = (r1 - r0) * chunks;
  for (int i = threadIdx.x; i < items; i += kThreads) {
    const int r = r0 + i / chunks, c = i % chunks;
    const int b = seq_of(s_cu, batch, r);
    bool take = true;
    if (MODE == FIRST) take = r == s_cu[b];
    if (MODE == LAST) take = r == s_cu[b + 1] - 1;
    uint4 w = make_uint4(0u, 0u, 0u, 0u);
    if (take) {
      const float4* src = reinterpret_cast<const float4*>(g + static_cast<int64_t>(b) * H + c * 8);
      const float4 lo = src[0], hi = src[1];
      __nv_bfloat162 q[4] = {__floats2bfloat162_rn(lo.x, lo.y), __floats2bfloat162_rn(lo.z, lo.w),
                             __floats2bfloat162_rn(hi.x, hi.y), __floats2bfloat162_rn(hi.z, hi.w)};
      w = *reinterpret_cast<uint4*>(q);
    }
    reinterpret_cast<uint4*>(dh + static_cast<int64_t>(r) * H)[c] = w;
  }
}

// out[col] += sum_rows x[row, col]  (bf16 input, fp32 accumulator).
// One CTA per slice of `slice` rows; thread (g, c) owns the 16-byte
// column chunk c (8 columns) for rows g, g + G, ... of the slice (G row groups
// when the row has at most 256 chunks, else one group of `chunks` threads),
// keeping four loads in flight; row groups meet in shared memory and each
// column gets one atomic per CTA.
__global__ void __launch_bounds__(1024)
    colsum_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld, int rows, int cols, int slice,
                  float* __restrict__ out) {
  extern __shared__ float part[];  // [groups][cols]
  const int chunks = cols >> 3;
  const int groups = blockDim.x / chunks;  // >= 1
  const int c = threadIdx.x % chunks, g = threadIdx.x / chunks;
  const int r0 = blockIdx.x * slice, r1 = min(rows, r0 + slice);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (g < groups) {
    for (int r = r0 + g; r < r1; r += 4 * groups) {
      uint4 w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int rr = r + u * groups;
        w[u] = rr < r1 ? reinterpret_cast<const uint4*>(x + static_cast<int64_t>(rr) * ld)[c]
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
  }
  if (groups == 1) {
    if (g == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) atomicAdd(out + c * 8 + j, acc[j]);
    }
    return;
  }
  if (g < groups) {
#pragma unroll
    for (int j = 0; j < 8; ++j) part[g * cols + c * 8 + j] = acc[j];
  }
  __syncthreads();
  for (int col = threadIdx.x; col < cols; col += blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < groups; ++q) s += part[q * cols + col];
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
  RX_CHECK(H % 8 == 0 && H <= 4096, "pool width must be a multiple of 8 and <= 4096");
  RX_CHECK(h.is_contiguous() && out.is_contiguous(), "pool tensors must be contiguous");
  RX_CHECK(reinterpret_cast<uintptr_t>(h.data_ptr()) % 16 == 0, "h must be 16-byte aligned");
  const int batch = static_cast<int>(cu_seqlens.numel() - 1);
  if (batch <= 0) return;
  RX_CHECK(batch <= pool::kMaxBatch, "at most ", pool::kMaxBatch, " sequences per pooling call");
  c10::cuda::CUDAGuard guard(h.get_device());
  auto st = at::cuda::getCurrentCUDAStream().stream();
  auto* hp = reinterpret_cast<const __nv_bfloat16*>(h.data_ptr());
  const int* cu = cu_seqlens.data_ptr<int>();
  const int total = static_cast<int>(h.size(0));
  float* o = out.data_ptr<float>();
  switch (mode) {
    case pool::MEAN: {
      RX_CUDA_CHECK(cudaMemsetAsync(o, 0, sizeof(float) * batch * H, st));
      if (total > 0) {
        const int slices = (total + pool::kSliceRows - 1) / pool::kSliceRows;
        pool::pool_sum_kernel<<<slices, pool::kThreads, sizeof(int) * (batch + 1), st>>>(hp, cu, batch, total, o,
                                                                                         static_cast<int>(H));
      }
      pool::pool_finish_kernel<pool::MEAN><<<batch, pool::kThreads, 0, st>>>(hp, cu, o, norm.data_ptr<float>(), H, normalize);
      break;
    }
    case pool::FIRST: pool::pool_finish_kernel<pool::FIRST><<<batch, pool::kThreads, 0, st>>>(hp, cu, o, norm.data_ptr<float>(), H, normalize); break;
    case pool::LAST: pool::pool_finish_kernel<pool::LAST><<<batch, pool::kThreads, 0, st>>>(hp, cu, o, norm.data_ptr<float>(), H, normalize); break;
    default: RX_CHECK(false, "unknown pooling mode");
  }
  RX_CUDA_CHECK(cudaGetLastError());
}

void pool_backward(const at::Tensor& dout, const at::Tensor& out, const at::Tensor& norm,
                   const at::Tensor& cu_seqlens, at::Tensor& dh, int64_t mode, bool normalize) {
  check_f32(dout, "dout");
  check_bf16(dh, "dh");
  const int64_t H = dh.size(1);
  RX_CHECK(H % 8 == 0 && H <= 4096, "pool width must be a multiple of 8 and <= 4096");
  RX_CHECK(dout.is_contiguous() && out.is_contiguous() && dh.is_contiguous(), "pool tensors must be contiguous");
  RX_CHECK(reinterpret_cast<uintptr_t>(dh.data_ptr()) % 16 == 0, "dh must be 16-byte aligned");
  const int batch = static_cast<int>(cu_seqlens.numel() - 1);
  if (batch <= 0) return;
  RX_CHECK(batch <= pool::kMaxBatch, "at most ", pool::kMaxBatch, " sequences per pooling call");
  c10::cuda::CUDAGuard guard(dh.get_device());
  auto st = at::cuda::getCurrentCUDAStream().stream();
  auto* dhp = reinterpret_cast<__nv_bfloat16*>(dh.data_ptr());
  const int* cu = cu_seqlens.data_ptr<int>();
  const int total = static_cast<int>(dh.size(0));
  at::Tensor g = at::empty({batch, H}, dout.options());
  const int slices = (total + pool::kSliceRows - 1) / pool::kSliceRows;
  const size_t smem = sizeof(int) * (batch + 1);
#define RX_POOL_BWD(M)                                                                                           \
  pool::pool_grad_kernel<M><<<batch, pool::kThreads, 0, st>>>(dout.data_ptr<float>(), out.data_ptr<float>(),   \
                                                              norm.data_ptr<float>(), cu, g.data_ptr<float>(),  \
                                                              static_cast<int>(H), normalize);                  \
  if (total > 0)                                                                                                 \
    pool::pool_rows_kernel<M><<<slices, pool::kThreads, smem, st>>>(g.data_ptr<float>(), cu, batch, total, dhp,  \
                                                                    static_cast<int>(H))
  switch (mode) {
    case pool::MEAN: RX_POOL_BWD(pool::MEAN); break;
    case pool::FIRST: RX_POOL_BWD(pool::FIRST); break;
    case pool::LAST: RX_POOL_BWD(pool::LAST); break;
    default: RX_CHECK(false, "unknown pooling mode");
  }
#undef RX_POOL_BWD
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
  constexpr int kMaxCols = 1024 * 8;
  if (cols > kMaxCols) {  // very wide matrices: independent column blocks
    for (int c0 = 0; c0 < cols; c0 += kMaxCols) {
      const int c1 = std::min(cols, c0 + kMaxCols);
      at::Tensor xs = x.narrow(1, c0, c1 - c0);
      at::Tensor os = out.narrow(0, c0, c1 - c0);
      colsum_accumulate(xs, os);
    }
    return;
  }
  c10::cuda::CUDAGuard guard(x.get_device());
  const int chunks = cols / 8;
  // up to 256 threads of row groups for narrow rows, else one thread per chunk
  const int threads = chunks <= 256 ? (256 / chunks) * chunks : (chunks + 31) / 32 * 32;
  const int groups = threads / chunks;
  const size_t smem = groups > 1 ? static_cast<size_t>(groups) * cols * sizeof(float) : 0;
  // enough CTAs to fill every SM (up to 8 resident each) so that ~64 KB of
  // loads are in flight per SM; each CTA sums a slice of at least 4 rows per group
  int sms = 148;
  RX_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, x.get_device()));
  const int per_sm = std::max(1, std::min(8, 2048 / threads));
  const int slice = std::max(4 * groups, (rows + sms * per_sm - 1) / (sms * per_sm));
  const int grid = (rows + slice - 1) / slice;
  auto kern = pool::colsum_kernel;
  if (smem > 48 * 1024)
    RX_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  kern<<<grid, threads, smem, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), rows, cols, slice,
      out.data_ptr<float>());
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
