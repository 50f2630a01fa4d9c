// Sequence pooling over packed token rows (mean / first token / last token),
// optional L2 normalisation, their backward passes, and small reductions
// (bias-gradient column sums, fp32 -> bf16 casts).
//
// Reference parity: `mean_pool` + `l2_normalize`
// (src/representax/models/components.py:238-258), last-valid-token pooling
// (src/representax/models/qwen3_vl/model.py:87-93) and CLS pooling
// (src/representax/models/sentence.py:47-132).
#include <algorithm>

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

// Every sequence is cut into `splits` contiguous row ranges, one CTA each
// (grid splits x batch): no searches and no atomics. Thread (g, c) owns the
// 16-byte column chunk c (8 columns) of rows g, g + G, ... of its range with
// four loads in flight; the G row groups meet in shared memory.
__device__ __forceinline__ void row_range(const int* cu, int b, int s, int splits, int& r0, int& r1, int& len) {
  const int start = cu[b], end = cu[b + 1];
  len = end - start;
  r0 = start + static_cast<int>(static_cast<int64_t>(len) * s / splits);
  r1 = start + static_cast<int>(static_cast<int64_t>(len) * (s + 1) / splits);
}

// MEAN, phase 1: part[b, s, :] = sum of the rows of range s of sequence b.
__global__ void __launch_bounds__(1024)
    pool_partial_kernel(const __nv_bfloat16* __restrict__ h, const int* __restrict__ cu, float* __restrict__ part,
                        int H, int splits) {
  extern __shared__ float red[];  // [G][H]
  const int s = blockIdx.x, b = blockIdx.y;
  int r0, r1, len;
  row_range(cu, b, s, splits, r0, r1, len);
  const int chunks = H >> 3, G = blockDim.x / chunks;
  const int c = threadIdx.x % chunks, g = threadIdx.x / chunks;  // g == G: padding threads of the last warp
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int r = g < G ? r0 + g : r1; r < r1; r += 4 * G) {
    uint4 w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int rr = r + u * G;
      w[u] = rr < r1 ? reinterpret_cast<const uint4*>(h + static_cast<int64_t>(rr) * H)[c] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&w[u]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(p2[j]);
        a[2 * j] += f.x;
        a[2 * j + 1] += f.y;
      }
    }
  }
  float* dst = part + (static_cast<int64_t>(b) * splits + s) * H;
  if (G == 1) {
    if (g > 0) return;
    reinterpret_cast<float4*>(dst)[2 * c] = make_float4(a[0], a[1], a[2], a[3]);
    reinterpret_cast<float4*>(dst)[2 * c + 1] = make_float4(a[4], a[5], a[6], a[7]);
    return;
  }
  if (g < G) {
#pragma unroll
    for (int j = 0; j < 8; ++j) red[g * H + c * 8 + j] = a[j];
  }
  __syncthreads();
  for (int col = threadIdx.x; col < H; col += blockDim.x) {
    float t = 0.f;
    for (int q = 0; q < G; ++q) t += red[q * H + col];
    dst[col] = t;
  }
}

// Phase 2 (every mode): one CTA per sequence. MEAN adds the partial sums in
// order and divides by the length; FIRST / LAST read their one row from h.
// Then the L2 norm and the optional normalisation; out and norm are written.
template <int MODE>
__global__ void __launch_bounds__(kThreads)
    pool_finish_kernel(const __nv_bfloat16* __restrict__ h, const int* __restrict__ cu, const float* __restrict__ part,
                       int splits, float* __restrict__ out, float* __restrict__ norm, int H, bool normalize) {
  __shared__ float scratch[32];
  const int b = blockIdx.x;
  const int s = cu[b], e = cu[b + 1];
  const int len = e - s;
  float* row = out + static_cast<int64_t>(b) * H;
  const int row_src = MODE == FIRST ? s : e - 1;
  const float inv_len = 1.f / fmaxf(static_cast<float>(len), 1.f);
  float sq = 0.f;
  for (int c = threadIdx.x; c < H; c += kThreads) {
    float v = 0.f;
    if (MODE == MEAN) {
      const float* pp = part + static_cast<int64_t>(b) * splits * H + c;
      for (int q = 0; q < splits; ++q) v += pp[static_cast<int64_t>(q) * H];
      v *= inv_len;
    } else if (len > 0) {
      v = __bfloat162float(h[static_cast<int64_t>(row_src) * H + c]);
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

// Backward, one launch: CTA (s, b) recomputes its sequence's pooled gradient
// g = (dout - out <out, dout>) / max(norm, eps) (when normalised) times
// 1 / len for MEAN, then writes g (MEAN) or g / 0 (FIRST / LAST: only the
// pooled row is non-zero) as bf16 into every row of its range.
template <int MODE>
__global__ void __launch_bounds__(1024)
    pool_backward_kernel(const float* __restrict__ dout, const float* __restrict__ out,
                         const float* __restrict__ norm, const int* __restrict__ cu, __nv_bfloat16* __restrict__ dh,
                         int H, int splits, bool normalize) {
  __shared__ float scratch[32];
  const int s = blockIdx.x, b = blockIdx.y;
  int r0, r1, len;
  row_range(cu, b, s, splits, r0, r1, len);
  const int chunks = H >> 3, G = blockDim.x / chunks;
  const int c = threadIdx.x % chunks, g = threadIdx.x / chunks;
  const float* d = dout + static_cast<int64_t>(b) * H + c * 8;
  const float* o = out + static_cast<int64_t>(b) * H + c * 8;
  float dv[8], ov[8];
  const float4 d0 = reinterpret_cast<const float4*>(d)[0], d1 = reinterpret_cast<const float4*>(d)[1];
  const float4 o0 = reinterpret_cast<const float4*>(o)[0], o1 = reinterpret_cast<const float4*>(o)[1];
  dv[0] = d0.x; dv[1] = d0.y; dv[2] = d0.z; dv[3] = d0.w; dv[4] = d1.x; dv[5] = d1.y; dv[6] = d1.z; dv[7] = d1.w;
  ov[0] = o0.x; ov[1] = o0.y; ov[2] = o0.z; ov[3] = o0.w; ov[4] = o1.x; ov[5] = o1.y; ov[6] = o1.z; ov[7] = o1.w;
  float dot = 0.f;
  if (normalize) {
    if (g == 0) {
#pragma unroll
      for (int j = 0; j < 8; ++j) dot += dv[j] * ov[j];
    }
    dot = block_sum(dot, scratch);
  }
  const float inv = normalize ? 1.f / fmaxf(norm[b], 1e-12f) : 1.f;
  const float w = MODE == MEAN ? 1.f / fmaxf(static_cast<float>(len), 1.f) : 1.f;
  uint4 val;
  __nv_bfloat162* v2 = reinterpret_cast<__nv_bfloat162*>(&val);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    v2[j] = __floats2bfloat162_rn((dv[2 * j] - ov[2 * j] * dot) * inv * w, (dv[2 * j + 1] - ov[2 * j + 1] * dot) * inv * w);
  const int pooled = MODE == FIRST ? cu[b] : cu[b + 1] - 1;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  for (int r = g < G ? r0 + g : r1; r < r1; r += G) {
    const bool take = MODE == MEAN || r == pooled;
    reinterpret_cast<uint4*>(dh + static_cast<int64_t>(r) * H)[c] = take ? val : zero;
  }
}

// out[col] += sum_rows x[row, col]  (bf16 input, fp32 accumulator).
// One CTA per slice of `slice` rows; thread (g, c) owns the 16-byte
// column chunk c (8 columns) for rows g, g + G, ... of the slice (G row
// groups of `chunks` threads), keeping eight loads in flight; row groups meet
// in shared memory and each column gets one atomic per CTA.
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
    for (int r = r0 + g; r < r1; r += 8 * groups) {
      // unconditional loads (rows past the slice re-read its last row and are
      // masked below) so that all eight are issued before the first is used
      uint4 w[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int rr = min(r + u * groups, r1 - 1);
        w[u] = ldg_v4_issue(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(rr) * ld) + c);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) hold_v4(w[u]);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (r + u * groups >= r1) w[u] = make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
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

// Row groups per CTA of the pooling kernels: up to 512 threads of 8-column chunks.
static int pool_groups(int64_t H) { return std::max<int64_t>(1, 512 / (H / 8)); }
// Row ranges per sequence: enough CTAs for about four per SM.
static int pool_splits(int batch, int device) {
  return std::max(1, std::min(16, (4 * num_sms(device) + batch - 1) / batch));
}

void pool_forward(const at::Tensor& h, const at::Tensor& cu_seqlens, at::Tensor& out,
                  at::Tensor& norm, int64_t mode, bool normalize) {
  check_bf16(h, "h");
  check_f32(out, "out");
  const int64_t H = h.size(1);
  RX_CHECK(H % 8 == 0 && H <= 8192, "pool width must be a multiple of 8 and <= 8192");
  RX_CHECK(h.is_contiguous() && out.is_contiguous(), "pool tensors must be contiguous");
  RX_CHECK(reinterpret_cast<uintptr_t>(h.data_ptr()) % 16 == 0, "h must be 16-byte aligned");
  const int batch = static_cast<int>(cu_seqlens.numel() - 1);
  if (batch <= 0) return;
  const int device = h.get_device();
  c10::cuda::CUDAGuard guard(device);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  auto* hp = reinterpret_cast<const __nv_bfloat16*>(h.data_ptr());
  const int* cu = cu_seqlens.data_ptr<int>();
  float* o = out.data_ptr<float>();
  switch (mode) {
    case pool::MEAN: {
      const int splits = pool_splits(batch, device), G = pool_groups(H);
      const int threads = (G * static_cast<int>(H / 8) + 31) / 32 * 32;
      at::Tensor part = at::empty({batch, splits, H}, out.options());
      const size_t smem = G > 1 ? sizeof(float) * G * H : 0;
      if (smem > 48 * 1024)
        RX_CUDA_CHECK(cudaFuncSetAttribute(pool::pool_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem)));
      pool::pool_partial_kernel<<<dim3(splits, batch), threads, smem, st>>>(hp, cu, part.data_ptr<float>(),
                                                                           static_cast<int>(H), splits);
      pool::pool_finish_kernel<pool::MEAN><<<batch, pool::kThreads, 0, st>>>(
          hp, cu, part.data_ptr<float>(), splits, o, norm.data_ptr<float>(), H, normalize);
      break;
    }
    case pool::FIRST:
      pool::pool_finish_kernel<pool::FIRST><<<batch, pool::kThreads, 0, st>>>(hp, cu, nullptr, 0, o,
                                                                              norm.data_ptr<float>(), H, normalize);
      break;
    case pool::LAST:
      pool::pool_finish_kernel<pool::LAST><<<batch, pool::kThreads, 0, st>>>(hp, cu, nullptr, 0, o,
                                                                             norm.data_ptr<float>(), H, normalize);
      break;
    default: RX_CHECK(false, "unknown pooling mode");
  }
  RX_CUDA_CHECK(cudaGetLastError());
}

void pool_backward(const at::Tensor& dout, const at::Tensor& out, const at::Tensor& norm,
                   const at::Tensor& cu_seqlens, at::Tensor& dh, int64_t mode, bool normalize) {
  check_f32(dout, "dout");
  check_bf16(dh, "dh");
  const int64_t H = dh.size(1);
  RX_CHECK(H % 8 == 0 && H <= 8192, "pool width must be a multiple of 8 and <= 8192");
  RX_CHECK(dout.is_contiguous() && out.is_contiguous() && dh.is_contiguous(), "pool tensors must be contiguous");
  RX_CHECK(reinterpret_cast<uintptr_t>(dh.data_ptr()) % 16 == 0 &&
               reinterpret_cast<uintptr_t>(dout.data_ptr()) % 16 == 0 &&
               reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
           "pool tensors must be 16-byte aligned");
  const int batch = static_cast<int>(cu_seqlens.numel() - 1);
  if (batch <= 0) return;
  const int device = dh.get_device();
  c10::cuda::CUDAGuard guard(device);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  auto* dhp = reinterpret_cast<__nv_bfloat16*>(dh.data_ptr());
  const int* cu = cu_seqlens.data_ptr<int>();
  const int splits = pool_splits(batch, device), G = pool_groups(H);
  const dim3 grid(splits, batch);
  const int threads = (G * static_cast<int>(H / 8) + 31) / 32 * 32;  // whole warps for block_sum
#define RX_POOL_BWD(M)                                                                                            \
  pool::pool_backward_kernel<M><<<grid, threads, 0, st>>>(dout.data_ptr<float>(), out.data_ptr<float>(),         \
                                                          norm.data_ptr<float>(), cu, dhp, static_cast<int>(H), \
                                                          splits, normalize)
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
  // one CTA per SM of up to 1024 threads (row groups of one thread per chunk,
  // each keeping eight 16-byte loads in flight); the groups meet in shared
  // memory, so every column takes one atomic per CTA
  const int groups = std::max(1, 1024 / chunks);
  const int threads = groups * chunks;
  const size_t smem = groups > 1 ? static_cast<size_t>(groups) * cols * sizeof(float) : 0;
  const int sms = num_sms(x.get_device());
  const int slice = std::max(8 * groups, (rows + sms - 1) / sms);
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
