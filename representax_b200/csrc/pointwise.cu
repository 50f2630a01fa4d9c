// Memory-bound per-token kernels of the decoder / vision families:
//
//  * rotary position embedding (rotate-half form) on packed [T, heads * D]
//    rows, with multi-axis positions (M-RoPE: every frequency reads the
//    position of its axis from a per-frequency table, which expresses both
//    the interleaved Qwen3-VL layout and the sectioned Qwen2.5-Omni one),
//    optionally fused with the per-head RMSNorm of Qwen3 q/k projections;
//    backward = inverse rotation (+ RMSNorm backward, weight gradient
//    reduced per CTA and added with one fp32 atomic per element per CTA);
//  * gated activations y = act(z[:, :I]) * z[:, I:] (GeGLU with erf or tanh
//    GELU, SwiGLU) and plain activations y = act(z), forward and backward.
//
// One warp owns one (token, head) row for RoPE: lane l holds elements
// l + 32k, so each rotate-half pair (i, i + D/2) lives in one thread and the
// rotation needs no shuffles; RMSNorm statistics use a warp reduction.
// GLU/activation kernels move 16-byte vectors (8 bf16) per thread.
//
// Reference parity: RoPE / M-RoPE (src/representax/models/modernvbert/model.py:82-112,
// src/representax/models/qwen3_vl/text.py:30-61), q/k RMSNorm
// (src/representax/models/qwen3_vl/text.py:184-185), GeGLU / SwiGLU
// (src/representax/models/modernvbert/model.py:264-269,
// src/representax/models/qwen3_vl/text.py:201-202).
#include "common.h"
#include "philox.cuh"

#include <algorithm>

namespace rx {
namespace pw {

constexpr int kRopeWarps = 8;

template <int D, bool NORM>
__global__ void __launch_bounds__(kRopeWarps * 32)
    rope_fwd_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, __nv_bfloat16* y, int64_t ldy,
                    const int* __restrict__ pos, int axes, const int* __restrict__ axis_of,
                    const float* __restrict__ inv_freq, const float* __restrict__ norm_w, float eps,
                    int total, int heads) {
  constexpr int E = D / 32;  // elements per lane
  const int lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(total) * heads;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kRopeWarps + (threadIdx.x >> 5); row < rows;
       row += static_cast<int64_t>(gridDim.x) * kRopeWarps) {
    const int64_t tok = row / heads;
    const int h = static_cast<int>(row % heads);
    const __nv_bfloat16* src = x + tok * ldx + h * D;
    float v[E];
#pragma unroll
    for (int k = 0; k < E; ++k) v[k] = __bfloat162float(src[lane + 32 * k]);
    if constexpr (NORM) {
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < E; ++k) ss += v[k] * v[k];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float rstd = rsqrtf(ss / D + eps);
#pragma unroll
      for (int k = 0; k < E; ++k) v[k] = v[k] * rstd * norm_w[lane + 32 * k];
    }
    __nv_bfloat16* dst = y + tok * ldy + h * D;
#pragma unroll
    for (int k = 0; k < E / 2; ++k) {
      const int f = lane + 32 * k;  // frequency index; elements f and f + D/2
      const int axis = axes > 1 ? axis_of[f] : 0;
      const float angle = static_cast<float>(pos[static_cast<int64_t>(axis) * total + tok]) * inv_freq[f];
      float sn, cs;
      sincosf(angle, &sn, &cs);
      const float a = v[k], b = v[k + E / 2];
      dst[f] = __float2bfloat16(a * cs - b * sn);
      dst[f + D / 2] = __float2bfloat16(b * cs + a * sn);
    }
  }
}

template <int D, bool NORM>
__global__ void __launch_bounds__(kRopeWarps * 32)
    rope_bwd_kernel(const __nv_bfloat16* __restrict__ dy, int64_t lddy, __nv_bfloat16* dx, int64_t lddx,
                    const __nv_bfloat16* __restrict__ x, int64_t ldx, const int* __restrict__ pos, int axes,
                    const int* __restrict__ axis_of, const float* __restrict__ inv_freq,
                    const float* __restrict__ norm_w, float eps, float* __restrict__ dw, int total,
                    int heads) {
  constexpr int E = D / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t rows = static_cast<int64_t>(total) * heads;
  float dw_part[E];
#pragma unroll
  for (int k = 0; k < E; ++k) dw_part[k] = 0.f;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * kRopeWarps + warp; row < rows;
       row += static_cast<int64_t>(gridDim.x) * kRopeWarps) {
    const int64_t tok = row / heads;
    const int h = static_cast<int>(row % heads);
    const __nv_bfloat16* g_src = dy + tok * lddy + h * D;
    float g[E];
#pragma unroll
    for (int k = 0; k < E; ++k) g[k] = __bfloat162float(g_src[lane + 32 * k]);
    // Inverse rotation: the gradient with respect to the pre-rotation vector.
#pragma unroll
    for (int k = 0; k < E / 2; ++k) {
      const int f = lane + 32 * k;
      const int axis = axes > 1 ? axis_of[f] : 0;
      const float angle = static_cast<float>(pos[static_cast<int64_t>(axis) * total + tok]) * inv_freq[f];
      float sn, cs;
      sincosf(angle, &sn, &cs);
      const float a = g[k], b = g[k + E / 2];
      g[k] = a * cs + b * sn;
      g[k + E / 2] = b * cs - a * sn;
    }
    if constexpr (NORM) {
      const __nv_bfloat16* xs = x + tok * ldx + h * D;
      float xv[E], ss = 0.f;
#pragma unroll
      for (int k = 0; k < E; ++k) {
        xv[k] = __bfloat162float(xs[lane + 32 * k]);
        ss += xv[k] * xv[k];
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float rstd = rsqrtf(ss / D + eps);
      float dot = 0.f;
#pragma unroll
      for (int k = 0; k < E; ++k) {
        const float xhat = xv[k] * rstd;
        dw_part[k] += g[k] * xhat;
        g[k] *= norm_w[lane + 32 * k];
        dot += g[k] * xhat;
        xv[k] = xhat;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
      dot /= D;
#pragma unroll
      for (int k = 0; k < E; ++k) g[k] = rstd * (g[k] - xv[k] * dot);
    }
    __nv_bfloat16* out = dx + tok * lddx + h * D;
#pragma unroll
    for (int k = 0; k < E; ++k) out[lane + 32 * k] = __float2bfloat16(g[k]);
  }
  if constexpr (NORM) {
    __shared__ float part[kRopeWarps][D];
#pragma unroll
    for (int k = 0; k < E; ++k) part[warp][lane + 32 * k] = dw_part[k];
    __syncthreads();
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kRopeWarps; ++w) s += part[w][i];
      atomicAdd(dw + i, s);
    }
  }
}

// ------------------------------------------------------------ activations
enum Act { GELU_ERF = 0, GELU_TANH = 1, SILU = 2, QUICK_GELU = 3 };

__device__ __forceinline__ float act_f(float x, int act) {
  switch (act) {
    case GELU_ERF: return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
    case GELU_TANH: {
      const float u = 0.79788456080286536f * (x + 0.044715f * x * x * x);
      return 0.5f * x * (1.f + tanhf(u));
    }
    case SILU: return x / (1.f + expf(-x));
    default: return x / (1.f + expf(-1.702f * x));
  }
}

__device__ __forceinline__ float act_grad(float x, int act) {
  switch (act) {
    case GELU_ERF: {
      const float cdf = 0.5f * (1.f + erff(x * 0.70710678118654752f));
      const float pdf = 0.39894228040143268f * expf(-0.5f * x * x);
      return cdf + x * pdf;
    }
    case GELU_TANH: {
      const float u = 0.79788456080286536f * (x + 0.044715f * x * x * x);
      const float t = tanhf(u);
      return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * 0.79788456080286536f * (1.f + 3.f * 0.044715f * x * x);
    }
    case SILU: {
      const float s = 1.f / (1.f + expf(-x));
      return s * (1.f + x * (1.f - s));
    }
    default: {
      const float s = 1.f / (1.f + expf(-1.702f * x));
      return s * (1.f + 1.702f * x * (1.f - s));
    }
  }
}

struct alignas(16) Vec8 {
  __nv_bfloat162 h[4];
};

__device__ __forceinline__ void unpack8(const Vec8& v, float (&f)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(v.h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ Vec8 pack8(const float (&f)[8]) {
  Vec8 v;
#pragma unroll
  for (int i = 0; i < 4; ++i) v.h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

// GATED: y[t, c] = act(z[t, c]) * z[t, I + c]; else y = act(z).
template <bool GATED>
__global__ void act_fwd_kernel(const __nv_bfloat16* __restrict__ z, int64_t ldz, __nv_bfloat16* __restrict__ y,
                               int64_t ldy, int total, int width, int act) {
  const int vecs = width / 8;
  const int64_t n = static_cast<int64_t>(total) * vecs;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / vecs;
    const int c = static_cast<int>(i % vecs) * 8;
    float a[8], out[8];
    unpack8(*reinterpret_cast<const Vec8*>(z + t * ldz + c), a);
    if constexpr (GATED) {
      float b[8];
      unpack8(*reinterpret_cast<const Vec8*>(z + t * ldz + width + c), b);
#pragma unroll
      for (int e = 0; e < 8; ++e) out[e] = act_f(a[e], act) * b[e];
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) out[e] = act_f(a[e], act);
    }
    *reinterpret_cast<Vec8*>(y + t * ldy + c) = pack8(out);
  }
}

template <bool GATED>
__global__ void act_bwd_kernel(const __nv_bfloat16* __restrict__ dy, int64_t lddy,
                               const __nv_bfloat16* __restrict__ z, int64_t ldz, __nv_bfloat16* __restrict__ dz,
                               int64_t lddz, int total, int width, int act) {
  const int vecs = width / 8;
  const int64_t n = static_cast<int64_t>(total) * vecs;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / vecs;
    const int c = static_cast<int>(i % vecs) * 8;
    float g[8], a[8], da[8];
    unpack8(*reinterpret_cast<const Vec8*>(dy + t * lddy + c), g);
    unpack8(*reinterpret_cast<const Vec8*>(z + t * ldz + c), a);
    if constexpr (GATED) {
      float b[8], db[8];
      unpack8(*reinterpret_cast<const Vec8*>(z + t * ldz + width + c), b);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        da[e] = g[e] * b[e] * act_grad(a[e], act);
        db[e] = g[e] * act_f(a[e], act);
      }
      *reinterpret_cast<Vec8*>(dz + t * lddz + width + c) = pack8(db);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) da[e] = g[e] * act_grad(a[e], act);
    }
    *reinterpret_cast<Vec8*>(dz + t * lddz + c) = pack8(da);
  }
}

// y = x * keep(m, n) / (1 - p) over a [rows, cols] bf16 matrix (cols % 4 == 0);
// one Philox block per 4 consecutive columns, the same mask as the GEMM
// epilogue's EPI_DROP at the same site. x and y may alias.
__global__ void dropout_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, __nv_bfloat16* y, int64_t ldy,
                               int64_t rows, int64_t cols, DropoutSite site) {
  const int64_t quads = cols / 4;
  const int64_t n = rows * quads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / quads, q = i % quads;
    const Keep8 k8 = keep8_of(site);
    const uint32_t keep = keep16(site, k8.t8, static_cast<uint32_t>(r), static_cast<uint32_t>(q >> 2)) >> (4 * (q & 3));
    const uint2 in = *reinterpret_cast<const uint2*>(x + r * ldx + 4 * q);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&in);
    const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    float v[4] = {a.x, a.y, b.x, b.y};
#pragma unroll
    for (int w = 0; w < 4; ++w) v[w] = ((keep >> w) & 1u) ? v[w] * k8.scale : 0.f;
    uint2 out;
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&out);
    o[0] = __floats2bfloat162_rn(v[0], v[1]);
    o[1] = __floats2bfloat162_rn(v[2], v[3]);
    *reinterpret_cast<uint2*>(y + r * ldy + 4 * q) = out;
  }
}

// Dropout of a [rows, cols] matrix that also adds the column sums of the
// result into colsum (fp32 [cols]): a block owns 256 columns (4 per thread)
// and a range of rows, and adds its partial sums with one atomic per column.
// y = dropout(x) with the column sums of the (rounded) result added into
// `colsum` (a bias gradient). One CTA per slice of rows: thread (g, u) owns
// the 16-column unit u (one Philox block per row) of rows g, g + G, ... of the
// slice, with eight rows' loads in flight; the G row groups meet in shared
// memory, so each column takes one atomic per CTA.
__global__ void __launch_bounds__(512)
    dropout_colsum_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, __nv_bfloat16* y, int64_t ldy,
                          int64_t rows, int64_t cols, DropoutSite site, float* __restrict__ colsum,
                          int64_t rows_per_block) {
  extern __shared__ float part[];  // [groups][cols]
  const int units = static_cast<int>(cols / 16);
  const int groups = blockDim.x / units;
  const int u = threadIdx.x % units, g = threadIdx.x / units;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  const int64_t r1 = r0 + rows_per_block < rows ? r0 + rows_per_block : rows;
  const Keep8 k8 = keep8_of(site);
  float acc[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) acc[j] = 0.f;
  if (g < groups) {
    for (int64_t r = r0 + g; r < r1; r += 8 * groups) {
      uint4 in[8][2];
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int64_t rr = r + t * groups < r1 ? r + t * groups : r1 - 1;  // past the slice: re-read, not used
        const uint4* src = reinterpret_cast<const uint4*>(x + rr * ldx + 16 * u);
        in[t][0] = __ldg(src);
        in[t][1] = __ldg(src + 1);
      }
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int64_t rr = r + t * groups;
        if (rr >= r1) break;
        const uint32_t keep = keep16(site, k8.t8, static_cast<uint32_t>(rr), static_cast<uint32_t>(u));
        uint4 out[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const __nv_bfloat162* i2 = reinterpret_cast<const __nv_bfloat162*>(&in[t][h]);
          __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&out[h]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = 8 * h + 2 * j;
            const float2 f = __bfloat1622float2(i2[j]);
            o2[j] = __floats2bfloat162_rn(((keep >> c) & 1u) ? f.x * k8.scale : 0.f,
                                          ((keep >> (c + 1)) & 1u) ? f.y * k8.scale : 0.f);
            const float2 back = __bfloat1622float2(o2[j]);
            acc[c] += back.x;
            acc[c + 1] += back.y;
          }
        }
        uint4* dst = reinterpret_cast<uint4*>(y + rr * ldy + 16 * u);
        dst[0] = out[0];
        dst[1] = out[1];
      }
    }
  }
  if (groups == 1) {
    if (g == 0) {
#pragma unroll
      for (int j = 0; j < 16; ++j) atomicAdd(colsum + 16 * u + j, acc[j]);
    }
    return;
  }
  if (g < groups) {
#pragma unroll
    for (int j = 0; j < 16; ++j) part[g * cols + 16 * u + j] = acc[j];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    float t = 0.f;
    for (int k = 0; k < groups; ++k) t += part[k * cols + c];
    atomicAdd(colsum + c, t);
  }
}

}  // namespace pw

namespace {
void check_rows(const at::Tensor& t, int64_t width, const char* name) {
  check_bf16(t, name);
  RX_CHECK(t.dim() == 2 && t.stride(1) == 1 && t.size(1) == width, name, " must be a [T, ", width, "] row view");
}
void check_vec_rows(const at::Tensor& t, const char* name) {
  RX_CHECK(t.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name,
           " rows must be 16-byte aligned");
}
int grid_for(int64_t work, int per_block, int device) {
  const int64_t blocks = (work + per_block - 1) / per_block;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, 8ll * num_sms(device))));
}
}  // namespace

// y = rope(norm?(x)); x and y may be the same tensor.
void rope_forward(const at::Tensor& x, at::Tensor& y, const at::Tensor& pos, const c10::optional<at::Tensor>& axis_of,
                  const at::Tensor& inv_freq, int64_t heads, const c10::optional<at::Tensor>& norm_w, double eps) {
  const int64_t T = x.size(0);
  RX_CHECK(heads > 0 && x.size(1) % heads == 0, "bad heads");
  const int64_t D = x.size(1) / heads;
  RX_CHECK(D == 64 || D == 128, "RoPE head_dim must be 64 or 128");
  check_rows(x, heads * D, "x");
  check_rows(y, heads * D, "y");
  RX_CHECK(y.size(0) == T, "y rows");
  RX_CHECK(pos.scalar_type() == at::kInt && pos.is_cuda() && pos.is_contiguous() && pos.dim() == 2 &&
               pos.size(1) == T, "pos must be int32 [axes, T]");
  const int axes = static_cast<int>(pos.size(0));
  const int* axis_ptr = nullptr;
  if (axes > 1) {
    RX_CHECK(axis_of.has_value() && axis_of->scalar_type() == at::kInt && axis_of->numel() == D / 2,
             "multi-axis RoPE needs an int32 [D/2] axis table");
    axis_ptr = axis_of->data_ptr<int>();
  }
  check_f32(inv_freq, "inv_freq");
  RX_CHECK(inv_freq.numel() == D / 2, "inv_freq must have D/2 entries");
  const float* w = nullptr;
  if (norm_w.has_value()) {
    check_f32(*norm_w, "norm_w");
    RX_CHECK(norm_w->numel() == D, "norm weight must have D entries");
    w = norm_w->data_ptr<float>();
  }
  if (T == 0) return;
  const int device = x.get_device();
  c10::cuda::CUDAGuard guard(device);
  auto st = at::cuda::getCurrentCUDAStream(device).stream();
  const int grid = grid_for(T * heads, pw::kRopeWarps, device);
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  const float e = static_cast<float>(eps);
  const int t = static_cast<int>(T), hh = static_cast<int>(heads);
#define RX_ROPE_FWD(DD, NN)                                                                              \
  pw::rope_fwd_kernel<DD, NN><<<grid, pw::kRopeWarps * 32, 0, st>>>(xp, x.stride(0), yp, y.stride(0),   \
                                                                     pos.data_ptr<int>(), axes, axis_ptr, \
                                                                     inv_freq.data_ptr<float>(), w, e, t, hh)
  if (D == 64) {
    if (w) RX_ROPE_FWD(64, true); else RX_ROPE_FWD(64, false);
  } else {
    if (w) RX_ROPE_FWD(128, true); else RX_ROPE_FWD(128, false);
  }
#undef RX_ROPE_FWD
  RX_CUDA_CHECK(cudaGetLastError());
}

// dx = d(norm?(x) -> rope)/dx applied to dy; dy and dx may alias. With a
// norm, `x` is the pre-norm input and `dw` (fp32 [D]) accumulates the
// weight gradient.
void rope_backward(const at::Tensor& dy, at::Tensor& dx, const c10::optional<at::Tensor>& x, const at::Tensor& pos,
                   const c10::optional<at::Tensor>& axis_of, const at::Tensor& inv_freq, int64_t heads,
                   const c10::optional<at::Tensor>& norm_w, double eps, const c10::optional<at::Tensor>& dw) {
  const int64_t T = dy.size(0);
  const int64_t D = dy.size(1) / heads;
  RX_CHECK(D == 64 || D == 128, "RoPE head_dim must be 64 or 128");
  check_rows(dy, heads * D, "dy");
  check_rows(dx, heads * D, "dx");
  RX_CHECK(pos.scalar_type() == at::kInt && pos.is_contiguous() && pos.dim() == 2 && pos.size(1) == T,
           "pos must be int32 [axes, T]");
  const int axes = static_cast<int>(pos.size(0));
  const int* axis_ptr = axes > 1 ? axis_of.value().data_ptr<int>() : nullptr;
  check_f32(inv_freq, "inv_freq");
  const float* w = nullptr;
  float* dwp = nullptr;
  const __nv_bfloat16* xp = nullptr;
  int64_t ldx = 0;
  if (norm_w.has_value()) {
    RX_CHECK(x.has_value() && dw.has_value(), "the norm backward needs x and dw");
    check_rows(*x, heads * D, "x");
    check_f32(*norm_w, "norm_w");
    check_f32(*dw, "dw");
    RX_CHECK(dw->numel() == D, "dw must have D entries");
    w = norm_w->data_ptr<float>();
    dwp = dw->data_ptr<float>();
    xp = reinterpret_cast<const __nv_bfloat16*>(x->data_ptr());
    ldx = x->stride(0);
  }
  if (T == 0) return;
  const int device = dy.get_device();
  c10::cuda::CUDAGuard guard(device);
  auto st = at::cuda::getCurrentCUDAStream(device).stream();
  const int grid = grid_for(T * heads, pw::kRopeWarps * 4, device);
  auto gp = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  auto op = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr());
  const float e = static_cast<float>(eps);
  const int t = static_cast<int>(T), hh = static_cast<int>(heads);
#define RX_ROPE_BWD(DD, NN)                                                                                     \
  pw::rope_bwd_kernel<DD, NN><<<grid, pw::kRopeWarps * 32, 0, st>>>(gp, dy.stride(0), op, dx.stride(0), xp, ldx, \
                                                                     pos.data_ptr<int>(), axes, axis_ptr,        \
                                                                     inv_freq.data_ptr<float>(), w, e, dwp, t, hh)
  if (D == 64) {
    if (w) RX_ROPE_BWD(64, true); else RX_ROPE_BWD(64, false);
  } else {
    if (w) RX_ROPE_BWD(128, true); else RX_ROPE_BWD(128, false);
  }
#undef RX_ROPE_BWD
  RX_CUDA_CHECK(cudaGetLastError());
}

// gated: z [T, 2I] -> y [T, I]; plain: z [T, I] -> y [T, I].
void activation_forward(const at::Tensor& z, at::Tensor& y, int64_t act, bool gated) {
  const int64_t T = z.size(0);
  const int64_t width = y.size(1);
  check_rows(z, gated ? 2 * width : width, "z");
  check_rows(y, width, "y");
  RX_CHECK(width % 8 == 0, "activation width must be a multiple of 8");
  check_vec_rows(z, "z");
  check_vec_rows(y, "y");
  RX_CHECK(act >= 0 && act <= 3, "unknown activation code");
  if (T == 0) return;
  const int device = z.get_device();
  c10::cuda::CUDAGuard guard(device);
  auto st = at::cuda::getCurrentCUDAStream(device).stream();
  const int grid = grid_for(T * width / 8, 256, device);
  auto zp = reinterpret_cast<const __nv_bfloat16*>(z.data_ptr());
  auto yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  if (gated)
    pw::act_fwd_kernel<true><<<grid, 256, 0, st>>>(zp, z.stride(0), yp, y.stride(0), static_cast<int>(T),
                                                    static_cast<int>(width), static_cast<int>(act));
  else
    pw::act_fwd_kernel<false><<<grid, 256, 0, st>>>(zp, z.stride(0), yp, y.stride(0), static_cast<int>(T),
                                                     static_cast<int>(width), static_cast<int>(act));
  RX_CUDA_CHECK(cudaGetLastError());
}

void activation_backward(const at::Tensor& dy, const at::Tensor& z, at::Tensor& dz, int64_t act, bool gated) {
  const int64_t T = dy.size(0);
  const int64_t width = dy.size(1);
  check_rows(dy, width, "dy");
  check_rows(z, gated ? 2 * width : width, "z");
  check_rows(dz, gated ? 2 * width : width, "dz");
  RX_CHECK(width % 8 == 0, "activation width must be a multiple of 8");
  check_vec_rows(dy, "dy");
  check_vec_rows(z, "z");
  check_vec_rows(dz, "dz");
  if (T == 0) return;
  const int device = dy.get_device();
  c10::cuda::CUDAGuard guard(device);
  auto st = at::cuda::getCurrentCUDAStream(device).stream();
  const int grid = grid_for(T * width / 8, 256, device);
  auto gp = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr());
  auto zp = reinterpret_cast<const __nv_bfloat16*>(z.data_ptr());
  auto dp = reinterpret_cast<__nv_bfloat16*>(dz.data_ptr());
  if (gated)
    pw::act_bwd_kernel<true><<<grid, 256, 0, st>>>(gp, dy.stride(0), zp, z.stride(0), dp, dz.stride(0),
                                                    static_cast<int>(T), static_cast<int>(width),
                                                    static_cast<int>(act));
  else
    pw::act_bwd_kernel<false><<<grid, 256, 0, st>>>(gp, dy.stride(0), zp, z.stride(0), dp, dz.stride(0),
                                                     static_cast<int>(T), static_cast<int>(width),
                                                     static_cast<int>(act));
  RX_CUDA_CHECK(cudaGetLastError());
}

void colsum_accumulate(const at::Tensor& x, at::Tensor& out);

void dropout_apply(const at::Tensor& x, at::Tensor& y, int64_t seed, int64_t stream, double p,
                   const c10::optional<at::Tensor>& colsum) {
  check_bf16(x, "x");
  check_bf16(y, "y");
  RX_CHECK(x.dim() == 2 && y.sizes() == x.sizes() && x.stride(1) == 1 && y.stride(1) == 1, "dropout needs matrices");
  RX_CHECK(x.size(1) % 4 == 0 && x.stride(0) % 4 == 0 && y.stride(0) % 4 == 0 &&
               reinterpret_cast<uintptr_t>(x.data_ptr()) % 8 == 0 && reinterpret_cast<uintptr_t>(y.data_ptr()) % 8 == 0,
           "dropout rows must be 8-byte aligned with width % 4 == 0");
  RX_CHECK(p > 0.0 && p < 1.0, "dropout probability must be in (0, 1)");
  const int64_t rows = x.size(0), cols = x.size(1);
  if (rows == 0) return;
  const int device = x.get_device();
  c10::cuda::CUDAGuard guard(device);
  if (colsum.has_value()) {
    check_f32(*colsum, "colsum");
    RX_CHECK(colsum->numel() == cols && colsum->is_contiguous(), "colsum must be fp32 [cols]");
    const int64_t units = cols / 16;
    const bool vec_ok = cols % 16 == 0 && x.stride(0) % 8 == 0 && y.stride(0) % 8 == 0 &&
                        reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                        reinterpret_cast<uintptr_t>(y.data_ptr()) % 16 == 0;
    if (units > 512 || !vec_ok) {  // wide or unaligned rows: plain dropout kernel, then a column-sum pass
      const int grid = grid_for(rows * cols / 4, 256, device);
      pw::dropout_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream(device).stream()>>>(
          reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
          reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), y.stride(0), rows, cols, make_dropout_site(seed, stream, p));
      RX_CUDA_CHECK(cudaGetLastError());
      at::Tensor sums = *colsum;
      colsum_accumulate(y, sums);
      return;
    }
    const int groups = static_cast<int>(std::max<int64_t>(1, 512 / units));
    const int threads = static_cast<int>(groups * units);
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(4ll * num_sms(device), (rows + 8 * groups - 1) /
                                                                                          (8 * groups)));
    const int64_t rows_per_block = (rows + blocks - 1) / blocks;
    const dim3 grid2(static_cast<unsigned>((rows + rows_per_block - 1) / rows_per_block));
    const size_t smem = groups > 1 ? static_cast<size_t>(groups) * cols * sizeof(float) : 0;
    if (smem > 48 * 1024)
      RX_CUDA_CHECK(cudaFuncSetAttribute(pw::dropout_colsum_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)));
    pw::dropout_colsum_kernel<<<grid2, threads, smem, at::cuda::getCurrentCUDAStream(device).stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0),
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), y.stride(0), rows, cols, make_dropout_site(seed, stream, p),
        colsum->data_ptr<float>(), rows_per_block);
    RX_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const int grid = grid_for(rows * cols / 4, 256, device);
  pw::dropout_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream(device).stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()),
      y.stride(0), rows, cols, make_dropout_site(seed, stream, p));
  RX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace rx
