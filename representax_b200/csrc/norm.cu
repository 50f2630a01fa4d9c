// Row-normalisation kernels for sm_100a: LayerNorm / RMSNorm forward and
// backward, the fused BERT embedding (three gathers + sum + LayerNorm), and
// its scatter-add backward.
//
// One warp owns one row; each lane holds H/256 (rounded up) 16-byte vectors
// of the row in registers, so the statistics are exact two-pass (mean, then
// centred variance) in fp32 without re-reading global memory. Parameter
// gradients (gamma, beta, and optionally the bias of the linear layer that
// produced the row) are reduced per CTA in registers/shared memory and added
// to fp32 accumulators with one atomic per column per CTA.
//
// Reference parity: LayerNorm / RMSNorm with fp32 statistics
// (src/representax/models/components.py:97-150) and BERT embeddings with
// padding-row gradient suppression (src/representax/models/bert/model.py:74-146).
#include <algorithm>

#include "common.h"
#include "sm100.cuh"

namespace rx {
namespace norm {

constexpr int kWarps = 8;

__device__ __forceinline__ void unpack8(const uint4& w, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 t = __bfloat1622float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 w;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
  return w;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------- forward
// RMS = true: y = x * rsqrt(mean(x^2) + eps) * gamma (no centring, no beta).
// When `word` is non-null the row is built as word[id] + pos[pid] + type[tid]
// (BERT embeddings) instead of being read from `x`.
template <int MAXV, bool RMS>
__global__ void __launch_bounds__(kWarps * 32)
    norm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ ids,
                    const int* __restrict__ pos_ids, const int* __restrict__ type_ids,
                    const __nv_bfloat16* __restrict__ word, const __nv_bfloat16* __restrict__ pos,
                    const __nv_bfloat16* __restrict__ type, const __nv_bfloat16* __restrict__ gamma,
                    const __nv_bfloat16* __restrict__ beta, __nv_bfloat16* __restrict__ y,
                    float* __restrict__ mean_out, float* __restrict__ rstd_out, int rows, int H,
                    float eps, __nv_bfloat16* __restrict__ sum_out) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nv = H >> 3;
  float v[MAXV][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = lane + 32 * i;
    if (c < nv) {
      if (word != nullptr) {
        float a[8], b[8], t[8];
        unpack8(reinterpret_cast<const uint4*>(word + static_cast<int64_t>(ids[row]) * H)[c], a);
        unpack8(reinterpret_cast<const uint4*>(pos + static_cast<int64_t>(pos_ids[row]) * H)[c], b);
        unpack8(reinterpret_cast<const uint4*>(type + static_cast<int64_t>(type_ids ? type_ids[row] : 0) * H)[c], t);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = a[j] + b[j] + t[j];
        if (sum_out != nullptr)
          reinterpret_cast<uint4*>(sum_out + static_cast<int64_t>(row) * H)[c] = pack8(v[i]);
      } else {
        unpack8(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * H)[c], v[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) s += RMS ? v[i][j] * v[i][j] : v[i][j];
    }
  }
  s = warp_sum(s);
  float mean = 0.f, rstd;
  if (RMS) {
    rstd = rsqrtf(s / H + eps);
  } else {
    mean = s / H;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      if (lane + 32 * i < nv) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float d = v[i][j] - mean;
          q += d * d;
        }
      }
    }
    q = warp_sum(q);
    rstd = rsqrtf(q / H + eps);
  }
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int c = lane + 32 * i;
    if (c < nv) {
      float g[8], b[8], o[8];
      unpack8(reinterpret_cast<const uint4*>(gamma)[c], g);
      if (!RMS && beta != nullptr) {
        unpack8(reinterpret_cast<const uint4*>(beta)[c], b);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) b[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (v[i][j] - mean) * rstd * g[j] + b[j];
      reinterpret_cast<uint4*>(y + static_cast<int64_t>(row) * H)[c] = pack8(o);
    }
  }
  if (lane == 0) {
    if (mean_out) mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// ---------------------------------------------------------------- backward
// dx = rstd * (dy*g - mean(dy*g) - xhat * mean(dy*g*xhat))     (LayerNorm)
// dx = rstd * (dy*g - xhat * mean(dy*g*xhat))                  (RMSNorm)
// dgamma += sum dy*xhat, dbeta += sum dy, dbias_prev += sum dx.
// When `word_grad` is non-null, x is rebuilt from the embedding tables and dx
// is scattered into the fp32 table gradients instead of being stored.
// Parameter-gradient partials (dgamma, dbeta, dbias_prev) live in shared
// memory, one [3][H] region per warp; each lane only touches the columns it
// owns, so no atomics are needed until the final per-CTA reduction. Keeping
// them out of registers lets three 8-warp CTAs share an SM.
template <int MAXV, bool RMS>
__global__ void __launch_bounds__(kWarps * 32, (MAXV <= 4 ? 3 : 1))
    norm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                    const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                    const __nv_bfloat16* __restrict__ gamma, __nv_bfloat16* __restrict__ dx,
                    float* __restrict__ dgamma, float* __restrict__ dbeta,
                    float* __restrict__ dbias_prev, int rows, int H,
                    // embedding mode
                    const int* __restrict__ ids, const int* __restrict__ pos_ids,
                    const int* __restrict__ type_ids, const __nv_bfloat16* __restrict__ word,
                    const __nv_bfloat16* __restrict__ pos, const __nv_bfloat16* __restrict__ type,
                    float* __restrict__ word_grad, float* __restrict__ pos_grad,
                    float* __restrict__ type_grad, int pad_id) {
  extern __shared__ float red[];  // [kWarps][3][H] partial sums
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nv = H >> 3;
  float* pg = red + static_cast<size_t>(warp) * 3 * H;
  float* pb = pg + H;
  float* pd = pb + H;
  for (int i = lane; i < 3 * H; i += 32) pg[i] = 0.f;
  __syncwarp();

  for (int row = blockIdx.x * kWarps + warp; row < rows; row += gridDim.x * kWarps) {
    const float mean = RMS ? 0.f : mean_in[row];
    const float rstd = rstd_in[row];
    float xv[MAXV][8];
    uint4 dpk[MAXV];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c = lane + 32 * i;
      if (c < nv) {
        if (word != nullptr) {
          float a[8], b[8], t[8];
          unpack8(reinterpret_cast<const uint4*>(word + static_cast<int64_t>(ids[row]) * H)[c], a);
          unpack8(reinterpret_cast<const uint4*>(pos + static_cast<int64_t>(pos_ids[row]) * H)[c], b);
          unpack8(reinterpret_cast<const uint4*>(type + static_cast<int64_t>(type_ids ? type_ids[row] : 0) * H)[c], t);
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[i][j] = a[j] + b[j] + t[j];
        } else {
          unpack8(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * H)[c], xv[i]);
        }
        dpk[i] = reinterpret_cast<const uint4*>(dy + static_cast<int64_t>(row) * H)[c];
        float d[8], g[8];
        unpack8(dpk[i], d);
        unpack8(reinterpret_cast<const uint4*>(gamma)[c], g);
        float4* gp = reinterpret_cast<float4*>(pg + c * 8);
        float4* bp = reinterpret_cast<float4*>(pb + c * 8);
        float4 g0 = gp[0], g1 = gp[1], b0 = bp[0], b1 = bp[1];
        float xh[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[j] = (xv[i][j] - mean) * rstd;
          const float dyg = d[j] * g[j];
          s1 += dyg;
          s2 += dyg * xh[j];
        }
        g0.x += d[0] * xh[0]; g0.y += d[1] * xh[1]; g0.z += d[2] * xh[2]; g0.w += d[3] * xh[3];
        g1.x += d[4] * xh[4]; g1.y += d[5] * xh[5]; g1.z += d[6] * xh[6]; g1.w += d[7] * xh[7];
        b0.x += d[0]; b0.y += d[1]; b0.z += d[2]; b0.w += d[3];
        b1.x += d[4]; b1.y += d[5]; b1.z += d[6]; b1.w += d[7];
        gp[0] = g0; gp[1] = g1; bp[0] = b0; bp[1] = b1;
      }
    }
    s1 = warp_sum(s1) / H;
    s2 = warp_sum(s2) / H;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c = lane + 32 * i;
      if (c < nv) {
        float d[8], g[8], o[8];
        unpack8(dpk[i], d);
        unpack8(reinterpret_cast<const uint4*>(gamma)[c], g);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = (xv[i][j] - mean) * rstd;
          o[j] = rstd * (d[j] * g[j] - (RMS ? 0.f : s1) - xh * s2);
        }
        // the producer-bias partial; in embedding mode without type ids (every
        // token of type 0) it holds the type-row gradient instead, added to
        // type_grad once per CTA rather than once per token
        if (dbias_prev != nullptr || (word_grad != nullptr && type_ids == nullptr)) {
          float4* dp = reinterpret_cast<float4*>(pd + c * 8);
          float4 a0 = dp[0], a1 = dp[1];
          a0.x += o[0]; a0.y += o[1]; a0.z += o[2]; a0.w += o[3];
          a1.x += o[4]; a1.y += o[5]; a1.z += o[6]; a1.w += o[7];
          dp[0] = a0; dp[1] = a1;
        }
        if (word_grad != nullptr) {
          const int id = ids[row];
          float* wg = word_grad + static_cast<int64_t>(id) * H + c * 8;
          float* pgp = pos_grad + static_cast<int64_t>(pos_ids[row]) * H + c * 8;
          float* tg = type_ids ? type_grad + static_cast<int64_t>(type_ids[row]) * H + c * 8 : nullptr;
#pragma unroll
          for (int j = 0; j < 8; j += 4) {
            const float4 w4 = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
            if (id != pad_id) red_add_f4(reinterpret_cast<float4*>(wg + j), w4);
            red_add_f4(reinterpret_cast<float4*>(pgp + j), w4);
            if (tg != nullptr) red_add_f4(reinterpret_cast<float4*>(tg + j), w4);
          }
        } else {
          reinterpret_cast<uint4*>(dx + static_cast<int64_t>(row) * H)[c] = pack8(o);
        }
      }
    }
  }
  __syncthreads();
  for (int col = threadIdx.x; col < H; col += blockDim.x) {
    float a = 0.f, b = 0.f, d = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float* base = red + static_cast<size_t>(w) * 3 * H;
      a += base[col];
      b += base[H + col];
      d += base[2 * H + col];
    }
    if (dgamma) atomicAdd(dgamma + col, a);
    if (dbeta && !RMS) atomicAdd(dbeta + col, b);
    if (dbias_prev) atomicAdd(dbias_prev + col, d);
    else if (word_grad != nullptr && type_ids == nullptr) atomicAdd(type_grad + col, d);
  }
}

// Backward of a plain (non-embedding) normalisation with the next row's
// inputs prefetched: each warp keeps its current row's raw x / dy vectors and
// the next row's loads in flight while it computes, so two rows per warp are
// outstanding (the one-row loop above is latency-bound on these shapes).
// Same arithmetic and the same per-warp shared-memory partial sums as
// norm_bwd_kernel.
template <int MAXV, bool RMS>
__global__ void __launch_bounds__(kWarps * 32, (MAXV <= 2 ? 3 : MAXV <= 4 ? 2 : 1))
    norm_bwd_prefetch_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                             const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                             const __nv_bfloat16* __restrict__ gamma, __nv_bfloat16* __restrict__ dx,
                             float* __restrict__ dgamma, float* __restrict__ dbeta,
                             float* __restrict__ dbias_prev, int rows, int H) {
  extern __shared__ float red[];  // [kWarps][3][H] partial sums
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nv = H >> 3;
  float* pg = red + static_cast<size_t>(warp) * 3 * H;
  float* pb = pg + H;
  float* pd = pb + H;
  for (int i = lane; i < 3 * H; i += 32) pg[i] = 0.f;
  __syncwarp();

  const int stride = gridDim.x * kWarps;
  uint4 xr[MAXV], dr[MAXV];
  float mean = 0.f, rstd = 0.f;
  auto load = [&](int row, uint4 (&xa)[MAXV], uint4 (&da)[MAXV], float& m, float& r) {
    if (row >= rows) return;
    m = RMS ? 0.f : mean_in[row];
    r = rstd_in[row];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c = lane + 32 * i;
      if (c < nv) {
        xa[i] = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * H)[c];
        da[i] = reinterpret_cast<const uint4*>(dy + static_cast<int64_t>(row) * H)[c];
      }
    }
  };
  int row = blockIdx.x * kWarps + warp;
  load(row, xr, dr, mean, rstd);
  for (; row < rows; row += stride) {
    uint4 xn[MAXV], dn[MAXV];
    float mean_n = 0.f, rstd_n = 0.f;
    load(row + stride, xn, dn, mean_n, rstd_n);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c = lane + 32 * i;
      if (c < nv) {
        float xv[8], d[8], g[8];
        unpack8(xr[i], xv);
        unpack8(dr[i], d);
        unpack8(reinterpret_cast<const uint4*>(gamma)[c], g);
        float4* gp = reinterpret_cast<float4*>(pg + c * 8);
        float4* bp = reinterpret_cast<float4*>(pb + c * 8);
        float4 g0 = gp[0], g1 = gp[1], b0 = bp[0], b1 = bp[1];
        float xh[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[j] = (xv[j] - mean) * rstd;
          const float dyg = d[j] * g[j];
          s1 += dyg;
          s2 += dyg * xh[j];
        }
        g0.x += d[0] * xh[0]; g0.y += d[1] * xh[1]; g0.z += d[2] * xh[2]; g0.w += d[3] * xh[3];
        g1.x += d[4] * xh[4]; g1.y += d[5] * xh[5]; g1.z += d[6] * xh[6]; g1.w += d[7] * xh[7];
        b0.x += d[0]; b0.y += d[1]; b0.z += d[2]; b0.w += d[3];
        b1.x += d[4]; b1.y += d[5]; b1.z += d[6]; b1.w += d[7];
        gp[0] = g0; gp[1] = g1; bp[0] = b0; bp[1] = b1;
      }
    }
    s1 = warp_sum(s1) / H;
    s2 = warp_sum(s2) / H;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int c = lane + 32 * i;
      if (c < nv) {
        float xv[8], d[8], g[8], o[8];
        unpack8(xr[i], xv);
        unpack8(dr[i], d);
        unpack8(reinterpret_cast<const uint4*>(gamma)[c], g);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = (xv[j] - mean) * rstd;
          o[j] = rstd * (d[j] * g[j] - (RMS ? 0.f : s1) - xh * s2);
        }
        if (dbias_prev != nullptr) {
          float4* dp = reinterpret_cast<float4*>(pd + c * 8);
          float4 a0 = dp[0], a1 = dp[1];
          a0.x += o[0]; a0.y += o[1]; a0.z += o[2]; a0.w += o[3];
          a1.x += o[4]; a1.y += o[5]; a1.z += o[6]; a1.w += o[7];
          dp[0] = a0; dp[1] = a1;
        }
        reinterpret_cast<uint4*>(dx + static_cast<int64_t>(row) * H)[c] = pack8(o);
      }
    }
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      xr[i] = xn[i];
      dr[i] = dn[i];
    }
    mean = mean_n;
    rstd = rstd_n;
  }
  __syncthreads();
  for (int col = threadIdx.x; col < H; col += blockDim.x) {
    float a = 0.f, b = 0.f, d = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float* base = red + static_cast<size_t>(w) * 3 * H;
      a += base[col];
      b += base[H + col];
      d += base[2 * H + col];
    }
    if (dgamma) atomicAdd(dgamma + col, a);
    if (dbeta && !RMS) atomicAdd(dbeta + col, b);
    if (dbias_prev) atomicAdd(dbias_prev + col, d);
  }
}

// Backward of a plain normalisation fed by bulk copies: rows are
// contiguous, so one warp (the producer) moves 8-row chunks of x and dy into a
// four-stage shared-memory ring with cp.async.bulk (one copy per tensor per
// chunk, completion counted on the stage's mbarrier) and loads the chunk's
// mean / rstd; each of the 8 compute warps takes one row of the chunk, frees
// the stage as soon as its row is in registers, and writes dx with 16-byte
// stores. 32 rows (96 KB at H = 768) are in flight per SM with no register
// cost. Parameter-gradient partials accumulate in registers (this lane's
// columns) and meet in shared memory once per CTA. Waits are bounded
// (%globaltimer) and report to the status word; an aborting CTA drains its
// copies before it exits.
namespace bulk {
constexpr int kRows = 8, kStages = 4, kComputeWarps = 8;
constexpr int kThreads = 32 * (kComputeWarps + 1);
}  // namespace bulk

template <int MAXV, bool RMS>
__global__ void __launch_bounds__(bulk::kThreads, 1)
    norm_bwd_bulk_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                         const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
                         const __nv_bfloat16* __restrict__ gamma, __nv_bfloat16* __restrict__ dx,
                         float* __restrict__ dgamma, float* __restrict__ dbeta, float* __restrict__ dbias_prev,
                         int rows, int H, int* status, uint64_t timeout_ns) {
  using namespace bulk;
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nv = H >> 3;
  const size_t tile = static_cast<size_t>(kRows) * H * 2;  // bytes of one tensor's chunk
  float* red = reinterpret_cast<float*>(smem);              // [kComputeWarps][3][H]
  uint8_t* ring = smem + static_cast<size_t>(kComputeWarps) * 3 * H * 4;
  // stage s: x chunk, dy chunk, then -mean / rstd [2][kRows] floats
  const size_t stage_bytes = 2 * tile + 2 * kRows * 4;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + kStages * stage_bytes);
  uint64_t* empty = full + kStages;
  volatile int* abort = reinterpret_cast<volatile int*>(empty + kStages);
  const int chunks = (rows + kRows - 1) / kRows;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 32);
      mbar_init(&empty[s], kComputeWarps * 32);
    }
    *abort = 0;
    fence_mbarrier_init();
  }
  if (warp < kComputeWarps) {
    float* pg = red + static_cast<size_t>(warp) * 3 * H;
    for (int i = lane; i < 3 * H; i += 32) pg[i] = 0.f;
  }
  __syncthreads();

  if (warp == kComputeWarps) {
    // ---------------------------------------------------------------- producer
    int k = 0;
    uint32_t issued[kStages] = {0, 0, 0, 0};
    for (int c = blockIdx.x; c < chunks; c += gridDim.x, ++k) {
      const int s = k % kStages;
      bool ok = true;
      if (lane == 0) {
        ok = !*abort && mbar_wait(&empty[s], ((k / kStages) & 1) ^ 1, timeout_ns);
        if (!ok && !*abort) {
          report_status(status, kStatusTimeoutProducer);
          *abort = 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      const int r0 = c * kRows, nr = min(kRows, rows - r0);
      uint8_t* st = ring + s * stage_bytes;
      if (lane == 0) {
        const uint32_t bytes = static_cast<uint32_t>(nr) * H * 2;
        mbar_expect_tx(&full[s], 2 * bytes);
        bulk_load(st, x + static_cast<int64_t>(r0) * H, bytes, &full[s]);
        bulk_load(st + tile, dy + static_cast<int64_t>(r0) * H, bytes, &full[s]);
        ++issued[s];
      }
      float* stats = reinterpret_cast<float*>(st + 2 * tile);
      if (lane < kRows) {
        const int r = r0 + lane;
        stats[lane] = r < rows && !RMS ? mean_in[r] : 0.f;
        stats[kRows + lane] = r < rows ? rstd_in[r] : 0.f;
      }
      mbar_arrive(&full[s]);
    }
    if (*abort && lane == 0)
      for (int s = 0; s < kStages; ++s)
        if (issued[s] > 0 && !mbar_wait(&full[s], (issued[s] - 1) & 1, timeout_ns))
          report_status(status, kStatusTimeoutDrain);
  } else {
    // ---------------------------------------------------------------- compute
    // parameter-gradient partials of this lane's columns stay in registers
    // (one CTA per SM leaves room) and meet in shared memory once at the end
    float ag[MAXV][8], ab[MAXV][8], ad[MAXV][8];
#pragma unroll
    for (int i = 0; i < MAXV; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) ag[i][j] = ab[i][j] = ad[i][j] = 0.f;
    int k = 0;
    for (int c = blockIdx.x; c < chunks; c += gridDim.x, ++k) {
      const int s = k % kStages;
      bool ok = !*abort && mbar_wait(&full[s], (k / kStages) & 1, timeout_ns);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0 && !*abort) {
          report_status(status, kStatusTimeoutEpilogue);
          *abort = 1;
        }
        break;
      }
      const uint8_t* st = ring + s * stage_bytes;
      const int row = c * kRows + warp;
      uint4 xr[MAXV], dr[MAXV];
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int cc = lane + 32 * i;
        if (cc < nv) {
          xr[i] = reinterpret_cast<const uint4*>(st + static_cast<size_t>(warp) * H * 2)[cc];
          dr[i] = reinterpret_cast<const uint4*>(st + tile + static_cast<size_t>(warp) * H * 2)[cc];
        }
      }
      const float* stats = reinterpret_cast<const float*>(st + 2 * tile);
      const float mean = stats[warp], rstd = stats[kRows + warp];
      mbar_arrive(&empty[s]);  // the row is in registers: the stage may refill
      if (row >= rows) continue;
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int cc = lane + 32 * i;
        if (cc < nv) {
          float xv[8], d[8], g[8];
          unpack8(xr[i], xv);
          unpack8(dr[i], d);
          unpack8(reinterpret_cast<const uint4*>(gamma)[cc], g);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float xh = (xv[j] - mean) * rstd;
            const float dyg = d[j] * g[j];
            s1 += dyg;
            s2 += dyg * xh;
            ag[i][j] += d[j] * xh;
            ab[i][j] += d[j];
          }
        }
      }
      s1 = warp_sum(s1) / H;
      s2 = warp_sum(s2) / H;
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int cc = lane + 32 * i;
        if (cc < nv) {
          float xv[8], d[8], g[8], o[8];
          unpack8(xr[i], xv);
          unpack8(dr[i], d);
          unpack8(reinterpret_cast<const uint4*>(gamma)[cc], g);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float xh = (xv[j] - mean) * rstd;
            o[j] = rstd * (d[j] * g[j] - (RMS ? 0.f : s1) - xh * s2);
            ad[i][j] += o[j];
          }
          reinterpret_cast<uint4*>(dx + static_cast<int64_t>(row) * H)[cc] = pack8(o);
        }
      }
    }
    float* pg = red + static_cast<size_t>(warp) * 3 * H;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int cc = lane + 32 * i;
      if (cc < nv) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          pg[cc * 8 + j] = ag[i][j];
          pg[H + cc * 8 + j] = ab[i][j];
          pg[2 * H + cc * 8 + j] = ad[i][j];
        }
      }
    }
  }
  __syncthreads();
  for (int col = threadIdx.x; col < H; col += blockDim.x) {
    float a = 0.f, b = 0.f, d = 0.f;
#pragma unroll
    for (int w = 0; w < kComputeWarps; ++w) {
      const float* base = red + static_cast<size_t>(w) * 3 * H;
      a += base[col];
      b += base[H + col];
      d += base[2 * H + col];
    }
    if (dgamma) atomicAdd(dgamma + col, a);
    if (dbeta && !RMS) atomicAdd(dbeta + col, b);
    if (dbias_prev) atomicAdd(dbias_prev + col, d);
  }
}

template <bool RMS>
void launch_fwd(int maxv, dim3 grid, cudaStream_t st, const __nv_bfloat16* x, const int* ids,
                const int* pos_ids, const int* type_ids, const __nv_bfloat16* word,
                const __nv_bfloat16* pos, const __nv_bfloat16* type, const __nv_bfloat16* gamma,
                const __nv_bfloat16* beta, __nv_bfloat16* y, float* mean, float* rstd, int rows,
                int H, float eps, __nv_bfloat16* sum_out) {
#define RX_NORM_FWD(V)                                                                        \
  norm_fwd_kernel<V, RMS><<<grid, kWarps * 32, 0, st>>>(x, ids, pos_ids, type_ids, word, pos, \
                                                         type, gamma, beta, y, mean, rstd, rows, \
                                                         H, eps, sum_out)
  if (maxv <= 1) RX_NORM_FWD(1);
  else if (maxv <= 2) RX_NORM_FWD(2);
  else if (maxv <= 3) RX_NORM_FWD(3);
  else if (maxv <= 4) RX_NORM_FWD(4);
  else if (maxv <= 8) RX_NORM_FWD(8);
  else RX_NORM_FWD(16);
#undef RX_NORM_FWD
  RX_CUDA_CHECK(cudaGetLastError());
}

template <bool RMS>
void launch_bwd(int maxv, int grid, int sms, int* status, size_t smem, cudaStream_t st, const __nv_bfloat16* dy,
                const __nv_bfloat16* x, const float* mean, const float* rstd,
                const __nv_bfloat16* gamma, __nv_bfloat16* dx, float* dgamma, float* dbeta,
                float* dbias_prev, int rows, int H, const int* ids, const int* pos_ids,
                const int* type_ids, const __nv_bfloat16* word, const __nv_bfloat16* pos,
                const __nv_bfloat16* type, float* wg, float* pg, float* tg, int pad_id) {
#define RX_NORM_BWD(V)                                                                            \
  do {                                                                                            \
    const size_t bulk_smem = static_cast<size_t>(bulk::kComputeWarps) * 3 * H * 4 +                \
                             bulk::kStages * (2 * static_cast<size_t>(bulk::kRows) * H * 2 +      \
                                              2 * bulk::kRows * 4) + 2 * bulk::kStages * 8 + 16;  \
    if (word == nullptr && bulk_smem <= 200 * 1024 &&                                             \
        reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(dy) % 16 == 0) { \
      auto k = norm_bwd_bulk_kernel<V, RMS>;                                                      \
      RX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,         \
                                         static_cast<int>(bulk_smem)));                           \
      const int chunks = (rows + bulk::kRows - 1) / bulk::kRows;                                  \
      k<<<std::max(1, std::min(chunks, sms)), bulk::kThreads, bulk_smem, st>>>(                   \
          dy, x, mean, rstd, gamma, dx, dgamma, dbeta, dbias_prev, rows, H, status, kWaitBudgetNs); \
    } else if (word == nullptr) {                                                                 \
      auto k = norm_bwd_prefetch_kernel<V, RMS>;                                                  \
      if (smem > 48 * 1024)                                                                       \
        RX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,       \
                                           static_cast<int>(smem)));                              \
      int per_sm = 1; /* one wave of resident CTAs: each warp strides over rows */                \
      RX_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kWarps * 32, smem));  \
      const int g = std::max(1, std::min(grid, std::max(1, per_sm) * sms));                       \
      k<<<g, kWarps * 32, smem, st>>>(dy, x, mean, rstd, gamma, dx, dgamma, dbeta, dbias_prev,    \
                                      rows, H);                                                   \
    } else {                                                                                      \
      auto k = norm_bwd_kernel<V, RMS>;                                                           \
      if (smem > 48 * 1024)                                                                       \
        RX_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,       \
                                           static_cast<int>(smem)));                              \
      k<<<grid, kWarps * 32, smem, st>>>(dy, x, mean, rstd, gamma, dx, dgamma, dbeta, dbias_prev, \
                                         rows, H, ids, pos_ids, type_ids, word, pos, type, wg, pg, \
                                         tg, pad_id);                                             \
    }                                                                                             \
  } while (0)
  if (maxv <= 1) RX_NORM_BWD(1);
  else if (maxv <= 2) RX_NORM_BWD(2);
  else if (maxv <= 3) RX_NORM_BWD(3);
  else if (maxv <= 4) RX_NORM_BWD(4);
  else if (maxv <= 6) RX_NORM_BWD(6);
  else RX_NORM_BWD(8);
#undef RX_NORM_BWD
  RX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace norm

namespace attn {
int* tc_status_word(int device);  // the device status word (attention_tc.cu)
}  // namespace attn

namespace {
template <typename T>
const T* opt_ptr(const c10::optional<at::Tensor>& t) {
  return t.has_value() ? reinterpret_cast<const T*>(t->data_ptr()) : nullptr;
}
template <typename T>
T* opt_mut(const c10::optional<at::Tensor>& t) {
  return t.has_value() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}
int maxv_for(int64_t H) { return static_cast<int>((H / 8 + 31) / 32); }
}  // namespace

// y = norm(x) with bf16 gamma/beta; returns fp32 mean (LayerNorm) and rstd.
void norm_forward(const at::Tensor& x, const at::Tensor& gamma, const c10::optional<at::Tensor>& beta,
                  at::Tensor& y, const c10::optional<at::Tensor>& mean, at::Tensor& rstd,
                  double eps, bool rms) {
  check_bf16(x, "x");
  check_bf16(gamma, "gamma");
  const int64_t H = x.size(-1);
  const int64_t rows = x.numel() / H;
  RX_CHECK(H % 8 == 0 && H <= 4096, "norm width must be a multiple of 8 and <= 4096");
  RX_CHECK(x.is_contiguous() && y.is_contiguous(), "norm tensors must be contiguous");
  if (rows == 0) return;
  c10::cuda::CUDAGuard guard(x.get_device());
  dim3 grid((rows + norm::kWarps - 1) / norm::kWarps);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto* gp = reinterpret_cast<const __nv_bfloat16*>(gamma.data_ptr());
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
  if (rms)
    norm::launch_fwd<true>(maxv_for(H), grid, st, xp, nullptr, nullptr, nullptr, nullptr, nullptr,
                           nullptr, gp, nullptr, yp, nullptr, rstd.data_ptr<float>(),
                           static_cast<int>(rows), static_cast<int>(H), static_cast<float>(eps),
                           nullptr);
  else
    norm::launch_fwd<false>(maxv_for(H), grid, st, xp, nullptr, nullptr, nullptr, nullptr, nullptr,
                            nullptr, gp, opt_ptr<__nv_bfloat16>(beta), yp, opt_mut<float>(mean),
                            rstd.data_ptr<float>(), static_cast<int>(rows), static_cast<int>(H),
                            static_cast<float>(eps), nullptr);
}

void norm_backward(const at::Tensor& dy, const at::Tensor& x, const c10::optional<at::Tensor>& mean,
                   const at::Tensor& rstd, const at::Tensor& gamma, at::Tensor& dx,
                   const c10::optional<at::Tensor>& dgamma, const c10::optional<at::Tensor>& dbeta,
                   const c10::optional<at::Tensor>& dbias_prev, bool rms) {
  check_bf16(dy, "dy");
  check_bf16(x, "x");
  const int64_t H = x.size(-1);
  const int64_t rows = x.numel() / H;
  RX_CHECK(H % 8 == 0 && H <= 2048, "norm backward width must be a multiple of 8 and <= 2048");
  if (rows == 0) return;
  c10::cuda::CUDAGuard guard(x.get_device());
  const int sms = num_sms(x.get_device());
  const int grid = static_cast<int>(std::min<int64_t>((rows + norm::kWarps - 1) / norm::kWarps, 3 * sms));
  const size_t smem = 3 * norm::kWarps * H * sizeof(float);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  auto launch = rms ? norm::launch_bwd<true> : norm::launch_bwd<false>;
  launch(maxv_for(H), grid, sms, attn::tc_status_word(x.get_device()), smem, st,
         reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
         reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), opt_ptr<float>(mean),
         rstd.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(gamma.data_ptr()),
         reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), opt_mut<float>(dgamma),
         opt_mut<float>(dbeta), opt_mut<float>(dbias_prev), static_cast<int>(rows),
         static_cast<int>(H), nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
         nullptr, nullptr, -1);
}

// BERT embeddings: y = LayerNorm(word[ids] + pos[pos_ids] + type[type_ids]).
void embed_ln_forward(const at::Tensor& ids, const at::Tensor& pos_ids,
                      const c10::optional<at::Tensor>& type_ids, const at::Tensor& word,
                      const at::Tensor& pos, const at::Tensor& type, const at::Tensor& gamma,
                      const at::Tensor& beta, at::Tensor& y, at::Tensor& mean, at::Tensor& rstd,
                      double eps) {
  check_bf16(word, "word");
  const int64_t H = word.size(1);
  const int64_t rows = ids.numel();
  RX_CHECK(ids.scalar_type() == at::kInt && pos_ids.scalar_type() == at::kInt, "ids must be int32");
  RX_CHECK(H % 8 == 0 && H <= 4096, "hidden size must be a multiple of 8");
  if (rows == 0) return;
  c10::cuda::CUDAGuard guard(word.get_device());
  dim3 grid((rows + norm::kWarps - 1) / norm::kWarps);
  norm::launch_fwd<false>(
      maxv_for(H), grid, at::cuda::getCurrentCUDAStream().stream(), nullptr, ids.data_ptr<int>(),
      pos_ids.data_ptr<int>(), type_ids.has_value() ? type_ids->data_ptr<int>() : nullptr,
      reinterpret_cast<const __nv_bfloat16*>(word.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(pos.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(type.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(gamma.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(beta.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), mean.data_ptr<float>(),
      rstd.data_ptr<float>(), static_cast<int>(rows), static_cast<int>(H), static_cast<float>(eps),
      nullptr);
}

void embed_ln_backward(const at::Tensor& dy, const at::Tensor& ids, const at::Tensor& pos_ids,
                       const c10::optional<at::Tensor>& type_ids, const at::Tensor& word,
                       const at::Tensor& pos, const at::Tensor& type, const at::Tensor& gamma,
                       const at::Tensor& mean, const at::Tensor& rstd, at::Tensor& word_grad,
                       at::Tensor& pos_grad, at::Tensor& type_grad, at::Tensor& dgamma,
                       at::Tensor& dbeta, int64_t pad_id) {
  const int64_t H = word.size(1);
  const int64_t rows = ids.numel();
  RX_CHECK(H % 8 == 0 && H <= 2048, "hidden size must be a multiple of 8 and <= 2048");
  check_f32(word_grad, "word_grad");
  if (rows == 0) return;
  c10::cuda::CUDAGuard guard(word.get_device());
  const int sms = num_sms(word.get_device());
  const int grid = static_cast<int>(std::min<int64_t>((rows + norm::kWarps - 1) / norm::kWarps, 3 * sms));
  const size_t smem = 3 * norm::kWarps * H * sizeof(float);
  norm::launch_bwd<false>(
      maxv_for(H), grid, sms, nullptr, smem, at::cuda::getCurrentCUDAStream().stream(),
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), nullptr, mean.data_ptr<float>(),
      rstd.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(gamma.data_ptr()), nullptr,
      dgamma.data_ptr<float>(), dbeta.data_ptr<float>(), nullptr, static_cast<int>(rows),
      static_cast<int>(H), ids.data_ptr<int>(), pos_ids.data_ptr<int>(),
      type_ids.has_value() ? type_ids->data_ptr<int>() : nullptr,
      reinterpret_cast<const __nv_bfloat16*>(word.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(pos.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(type.data_ptr()), word_grad.data_ptr<float>(),
      pos_grad.data_ptr<float>(), type_grad.data_ptr<float>(), static_cast<int>(pad_id));
}

}  // namespace rx
