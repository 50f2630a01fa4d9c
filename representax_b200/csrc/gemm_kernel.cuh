// Persistent tcgen05 GEMM for sm_100a with fused epilogues.
//
//   C[M, N] = epilogue(alpha * sum_k A(m, k) * B(n, k))
//
// A is K-major (stored [M, K]) or MN-major (stored [K, M]); B is K-major
// (stored [N, K]) or MN-major (stored [K, N]). The three combinations cover a
// linear layer's forward (K/K), input gradient (K/MN) and weight gradient
// (MN/MN) without materialising any transpose.
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: 128x64 A tile + BNx64 B tile per stage, 128-byte
//               swizzle, 4-stage ring guarded by full/empty mbarriers.
//   warp 1      owns TMEM (2 x BN fp32 columns = a double-buffered 128xBN
//               accumulator) and one thread issues tcgen05.mma (M=128, K=16)
//               and tcgen05.commit.
//   warps 2-9   epilogue: two warps per 32-lane TMEM quadrant, each taking half
//               of the tile's columns; tcgen05.ld gives one output row per
//               thread; fused bias / GELU (also writing gelu'(z) for the
//               backward) / GELU-backward (a product with that saved
//               derivative) / residual, bf16 or fp32 stores, fp32 accumulate or
//               split-K atomic reduction.
// The double-buffered accumulator lets the epilogue of tile i overlap the
// main loop of tile i+1.
//
// Linear-layer role parity: the reference's `Linear.__call__`
// (src/representax/models/components.py:81-94) and its XLA-generated
// backward; this kernel replaces both.
#pragma once
#include "common.h"
#include "philox.cuh"
#include "sm100.cuh"

namespace rx {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kEpilogueWarps = 8;  // two per TMEM lane quadrant, each owning half the columns
constexpr int kMaxGatherRanks = 16;
constexpr int kGatherRows = 32;  // rows per gather chunk (one readiness flag each)
constexpr int kThreads = 64 + 32 * kEpilogueWarps;

// EPI_DROP: inverted dropout of the (biased) value before the residual add;
// element (m, n) keeps its value when word (n & 3) of Philox block
// (m, n >> 2) at the site is >= the threshold.
// EPI_COLSUM (tile-store path only): the column sums of the output are added
// into p.colsum (fp32 [N]) with one atomic per column per 32-row warp piece
// (the bias gradient of the layer whose input gradient is being computed).
enum Epi : int { EPI_BIAS = 1, EPI_GELU = 2, EPI_DGELU = 4, EPI_RESID = 8, EPI_DROP = 16, EPI_COLSUM = 32 };
enum Out : int { OUT_BF16 = 0, OUT_F32 = 1, OUT_F32_ACC = 2, OUT_F32_ATOMIC = 3 };

struct Params {
  int M, N, K;
  int m_tiles, n_tiles, splits, kb_total, kb_per_split, num_units;
  void* C;
  int64_t ldc;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* aux_in;
  int64_t ld_aux_in;
  __nv_bfloat16* aux_out;
  int64_t ld_aux_out;
  const __nv_bfloat16* residual;
  int64_t ld_res;
  float alpha;
  const float* scales;  // fp8: device [2] per-tensor operand scales multiplied into alpha
  DropoutSite drop;
  float* colsum;
  int* status;
  uint64_t timeout_ns;
  // Fused FSDP gather (forward, single-CTA kernel only). The B operand is a
  // weight whose flat elements [g_off, g_off + N * K) are spread over the
  // ranks' shards (rank r holds flat [r * g_seg, (r + 1) * g_seg) at
  // g_src[r], bf16). The epilogue warps first copy 32-row chunks of it into
  // g_dst (this GPU's full copy, which B's tensor map reads) by plain loads
  // from the owners, raising g_ready[chunk]; the producer waits for a tile's
  // chunks before loading it.
  int gather;
  int g_world;
  int64_t g_seg, g_off;
  int64_t g_src[kMaxGatherRanks];
  __nv_bfloat16* g_dst;
  int* g_ready;
};

// Operand kinds: 0 = bf16 x bf16 (kind::f16); 1.. = 8-bit floats
// (kind::f8f6f4), KIND - 1 = (a_fmt | b_fmt << 1) with 0 = E4M3, 1 = E5M2.
constexpr int kKindBf16 = 0;
constexpr int fp8_kind(int a_fmt, int b_fmt) { return 1 + (a_fmt | (b_fmt << 1)); }

// GELU (erf form) and its derivative from one exponential: the normal CDF
// Phi(x) = (1 + erf(x / sqrt 2)) / 2 uses the rational approximation of
// Abramowitz & Stegun, Handbook of Mathematical Functions, eq. 7.1.26
// (|error of erf| <= 1.5e-7, far below bf16's resolution), whose exp(-u^2)
// factor at u = |x| / sqrt 2 is exp(-x^2 / 2), the same exponential the normal
// density phi(x) needs. gelu = x Phi(x); gelu' = Phi(x) + x phi(x).
__device__ __forceinline__ void gelu_and_grad(float x, float& gelu, float& grad) {
  const float u = fabsf(x) * 0.70710678118654752440f;
  float t;  // 1 / (1 + p u) by the approximate reciprocal (a few ulp, far below bf16's resolution)
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.3275911f, u, 1.0f)));
  float poly = fmaf(1.061405429f, t, -1.453152027f);
  poly = fmaf(poly, t, 1.421413741f);
  poly = fmaf(poly, t, -0.284496736f);
  poly = fmaf(poly, t, 0.254829592f);
  poly *= t;
  float e;  // exp(-x^2 / 2) = 2^(-x^2 / 2 * log2(e))
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-0.72134752044448170368f * x * x));
  const float erf_u = 1.0f - poly * e;  // erf(|x| / sqrt 2)
  const float cdf = 0.5f + 0.5f * copysignf(erf_u, x);
  gelu = x * cdf;
  grad = fmaf(x * 0.39894228040143267794f, e, cdf);
}

__device__ __forceinline__ float gelu_erf(float x) {
  float g, d;
  gelu_and_grad(x, g, d);
  return g;
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float (&v)[32]) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w = s[q];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(h[j]);
      v[q * 8 + 2 * j] = f.x;
      v[q * 8 + 2 * j + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[q * 8 + 2 * j], v[q * 8 + 2 * j + 1]);
    d[q] = w;
  }
}

// Write one lane's 32 bf16 values as row `lane` of a 32 x 32 tile staged in
// shared memory with the 64-byte swizzle of the store tensor map.
__device__ __forceinline__ void stage_row32_sw64(uint8_t* buf, int lane, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(v[q * 8 + 2 * j], v[q * 8 + 2 * j + 1]);
    *reinterpret_cast<uint4*>(buf + lane * 64 + ((q ^ ((lane >> 1) & 3)) * 16)) = w;
  }
}

// Coalesced load of a 32 x 32 bf16 tile (rows row0.., columns n_base..) into
// `buf` with the 64-byte swizzle: 16-byte pieces, 4 lanes per 64-byte row
// segment; rows >= rows_valid and columns >= cols_valid read as zero.
__device__ __forceinline__ void warp_load_tile32_sw64(uint8_t* buf, const __nv_bfloat16* src, int64_t ld, int row0,
                                                      int n_base, int rows_valid, int cols_valid, int lane) {
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int c = lane + 32 * it;
    const int row = c >> 2, piece = c & 3;
    const int m = row0 + row, n = n_base + piece * 8;
    uint4 w = make_uint4(0u, 0u, 0u, 0u);
    if (m < rows_valid) {
      const __nv_bfloat16* g = src + static_cast<int64_t>(m) * ld + n;
      if (n + 8 <= cols_valid) {
        w = *reinterpret_cast<const uint4*>(g);
      } else {
        __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&w);
        for (int k = 0; k < 8; ++k) e[k] = n + k < cols_valid ? g[k] : __float2bfloat16_rn(0.f);
      }
    }
    *reinterpret_cast<uint4*>(buf + row * 64 + ((piece ^ ((row >> 1) & 3)) * 16)) = w;
  }
}

// The same 32 x 32 tile in two steps, so the loads of the next tile can be
// in flight while the current one is computed: fetch into registers (lane
// holds pieces lane, lane + 32, lane + 64, lane + 96) ...
__device__ __forceinline__ void warp_fetch_tile32(const __nv_bfloat16* src, int64_t ld, int row0, int n_base,
                                                  int rows_valid, int cols_valid, int lane, uint4 (&w)[4]) {
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int c = lane + 32 * it;
    const int row = c >> 2, piece = c & 3;
    const int m = row0 + row, n = n_base + piece * 8;
    w[it] = make_uint4(0u, 0u, 0u, 0u);
    if (m < rows_valid) {
      const __nv_bfloat16* g = src + static_cast<int64_t>(m) * ld + n;
      if (n + 8 <= cols_valid) {
        w[it] = *reinterpret_cast<const uint4*>(g);
      } else {
        __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(&w[it]);
        for (int k = 0; k < 8; ++k) e[k] = n + k < cols_valid ? g[k] : __float2bfloat16_rn(0.f);
      }
    }
  }
}

// ... then place it in `buf` with the 64-byte swizzle.
__device__ __forceinline__ void warp_put_tile32_sw64(uint8_t* buf, int lane, const uint4 (&w)[4]) {
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int c = lane + 32 * it;
    const int row = c >> 2, piece = c & 3;
    *reinterpret_cast<uint4*>(buf + row * 64 + ((piece ^ ((row >> 1) & 3)) * 16)) = w[it];
  }
}

// Row `lane` of a 64-byte-swizzled 32 x 32 bf16 tile as 32 floats.
__device__ __forceinline__ void read_row32_sw64(const uint8_t* buf, int lane, float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 w = *reinterpret_cast<const uint4*>(buf + lane * 64 + ((q ^ ((lane >> 1) & 3)) * 16));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      v[q * 8 + 2 * j] = f.x;
      v[q * 8 + 2 * j + 1] = f.y;
    }
  }
}

// Epilogue values of one row segment for the staged tile store, with the
// residual (EPI_RESID) or the saved GELU derivative (EPI_DGELU) already in
// `side`; with EPI_GELU the derivative gelu'(z) is returned in `pre`.
template <int EPI>
__device__ __forceinline__ void epilogue_tile_values32(const Params& p, int m, int n_base, const uint32_t (&r)[32],
                                                       const float (&side)[32], float (&v)[32], float (&pre)[32]) {
  const bool row_ok = m < p.M;
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * p.alpha;
  if constexpr ((EPI & EPI_BIAS) != 0) {
    if (n_base + 32 <= p.N) {
      float b[32];
      load_bf16x32(p.bias + n_base, b);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += b[i];
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += n_base + i < p.N ? __bfloat162float(p.bias[n_base + i]) : 0.f;
    }
  }
  if constexpr ((EPI & EPI_DGELU) != 0) {  // side = gelu'(z) saved by the forward
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= side[i];
  }
  if constexpr ((EPI & EPI_GELU) != 0) {  // pre receives gelu'(z) for the backward
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float g, d;
      gelu_and_grad(v[i], g, d);
      pre[i] = d;
      v[i] = g;
    }
  }
  if constexpr ((EPI & EPI_DROP) != 0) {
    if (row_ok) {  // 8-bit decisions: two Philox blocks cover the 32 columns
      const Keep8 k8 = keep8_of(p.drop);
      const uint32_t keep = keep16(p.drop, k8.t8, static_cast<uint32_t>(m), static_cast<uint32_t>(n_base >> 4)) |
                            (keep16(p.drop, k8.t8, static_cast<uint32_t>(m), static_cast<uint32_t>((n_base >> 4) + 1))
                             << 16);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = ((keep >> i) & 1u) ? v[i] * k8.scale : 0.f;
    }
  }
  if constexpr ((EPI & EPI_RESID) != 0) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] += side[i];
  }
}

// Epilogue for one row segment of 32 columns [n_base, n_base + 32).
template <int EPI, int OUT>
__device__ __forceinline__ void epilogue_row32(const Params& p, int m, int n_base,
                                               const uint32_t (&r)[32]) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * p.alpha;
  const bool full = (n_base + 32 <= p.N);
  if (full) {
    if constexpr ((EPI & EPI_BIAS) != 0) {
      float b[32];
      load_bf16x32(p.bias + n_base, b);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += b[i];
    }
    if constexpr ((EPI & EPI_DGELU) != 0) {  // times gelu'(z) saved by the forward
      float d[32];
      load_bf16x32(p.aux_in + static_cast<int64_t>(m) * p.ld_aux_in + n_base, d);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] *= d[i];
    }
    if constexpr ((EPI & EPI_GELU) != 0) {  // aux_out receives gelu'(z)
      float d[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) gelu_and_grad(v[i], v[i], d[i]);
      store_bf16x32(p.aux_out + static_cast<int64_t>(m) * p.ld_aux_out + n_base, d);
    }
    if constexpr ((EPI & EPI_DROP) != 0) {
      const Keep8 k8 = keep8_of(p.drop);
      const uint32_t keep = keep16(p.drop, k8.t8, static_cast<uint32_t>(m), static_cast<uint32_t>(n_base >> 4)) |
                            (keep16(p.drop, k8.t8, static_cast<uint32_t>(m), static_cast<uint32_t>((n_base >> 4) + 1))
                             << 16);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = ((keep >> i) & 1u) ? v[i] * k8.scale : 0.f;
    }
    if constexpr ((EPI & EPI_RESID) != 0) {
      float res[32];
      load_bf16x32(p.residual + static_cast<int64_t>(m) * p.ld_res + n_base, res);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += res[i];
    }
    if constexpr (OUT == OUT_BF16) {
      store_bf16x32(reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(m) * p.ldc + n_base,
                    v);
    } else {
      float* c = reinterpret_cast<float*>(p.C) + static_cast<int64_t>(m) * p.ldc + n_base;
      float4* c4 = reinterpret_cast<float4*>(c);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 w = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        if constexpr (OUT == OUT_F32) {
          c4[q] = w;
        } else if constexpr (OUT == OUT_F32_ACC) {
          float4 o = c4[q];
          c4[q] = make_float4(o.x + w.x, o.y + w.y, o.z + w.z, o.w + w.w);
        } else {
          red_add_f4(c4 + q, w);
        }
      }
    }
    return;
  }
  // Ragged right edge: scalar, bounds-checked, statically indexed so the
  // values stay in registers.
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int n = n_base + i;
    if (n < p.N) {
      float x = v[i];
      if constexpr ((EPI & EPI_BIAS) != 0) x += __bfloat162float(p.bias[n]);
      if constexpr ((EPI & EPI_DGELU) != 0)
        x *= __bfloat162float(p.aux_in[static_cast<int64_t>(m) * p.ld_aux_in + n]);
      if constexpr ((EPI & EPI_GELU) != 0) {
        float d;
        gelu_and_grad(x, x, d);
        p.aux_out[static_cast<int64_t>(m) * p.ld_aux_out + n] = __float2bfloat16_rn(d);
      }
      if constexpr ((EPI & EPI_DROP) != 0) {
        const Keep8 k8 = keep8_of(p.drop);
        const uint32_t keep = keep16(p.drop, k8.t8, static_cast<uint32_t>(m), static_cast<uint32_t>(n >> 4));
        x = ((keep >> (n & 15)) & 1u) ? x * k8.scale : 0.f;
      }
      if constexpr ((EPI & EPI_RESID) != 0)
        x += __bfloat162float(p.residual[static_cast<int64_t>(m) * p.ld_res + n]);
      const int64_t off = static_cast<int64_t>(m) * p.ldc + n;
      if constexpr (OUT == OUT_BF16) {
        reinterpret_cast<__nv_bfloat16*>(p.C)[off] = __float2bfloat16_rn(x);
      } else if constexpr (OUT == OUT_F32) {
        reinterpret_cast<float*>(p.C)[off] = x;
      } else if constexpr (OUT == OUT_F32_ACC) {
        reinterpret_cast<float*>(p.C)[off] += x;
      } else {
        atomicAdd(reinterpret_cast<float*>(p.C) + off, x);
      }
    }
  }
}

// Work unit u -> (row tile origin, column tile index, k-block range). Column
// tiles vary fastest so consecutive CTAs share an A row block in L2.
__device__ __forceinline__ void decode_unit(const Params& p, int u, int& m0, int& n_tile, int& kb0,
                                            int& kb1) {
  n_tile = u % p.n_tiles;
  const int t = u / p.n_tiles;
  const int m_t = t % p.m_tiles;
  const int split = t / p.m_tiles;
  m0 = m_t * BM;
  kb0 = split * p.kb_per_split;
  kb1 = min(p.kb_total, kb0 + p.kb_per_split);
}

__device__ __forceinline__ int ld_acquire_gpu_s32(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Copy gather chunks c = first, first + step, ... of the weight into p.g_dst.
// Runs on the epilogue warps (256 threads, named barrier 1); every 16-byte
// piece comes from the rank owning that flat position (runs split at shard
// boundaries; slots and shards are 64-element aligned, rows 8-element aligned).
__device__ __forceinline__ void gather_weight_chunks(const Params& p, int first, int step, int tid) {
  const int64_t row_elems = p.K;
  const int chunks = (p.N + kGatherRows - 1) / kGatherRows;
  for (int c = first; c < chunks; c += step) {
    const int64_t e0 = p.g_off + static_cast<int64_t>(c) * kGatherRows * row_elems;
    const int64_t e1 = p.g_off + static_cast<int64_t>(min(p.N, (c + 1) * kGatherRows)) * row_elems;
    const int64_t pieces = (e1 - e0) >> 3;  // 8 bf16 per 16-byte piece
    for (int64_t base = 0; base < pieces; base += 256 * 8) {
      uint4 v[8];
      int64_t at[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t q = base + u * 256 + tid;
        at[u] = -1;
        if (q < pieces) {
          const int64_t e = e0 + (q << 3);
          const int owner = static_cast<int>(e / p.g_seg);
          at[u] = e;
          v[u] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.g_src[owner]) +
                                                 (e - owner * p.g_seg));
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (at[u] >= 0) *reinterpret_cast<uint4*>(p.g_dst + (at[u] - p.g_off)) = v[u];
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __threadfence();
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpilogueWarps) : "memory");
    if (tid == 0) asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(p.g_ready + c) : "memory");
  }
}

// Producer side: all chunks holding rows [n0, n0 + bn) of the weight are in place.
__device__ __forceinline__ bool gather_rows_ready(const Params& p, int n0, int bn) {
  const int c1 = (min(p.N, n0 + bn) + kGatherRows - 1) / kGatherRows;
  for (int c = n0 / kGatherRows; c < c1; ++c) {
    if (ld_acquire_gpu_s32(p.g_ready + c) > 0) continue;
    const uint64_t start = globaltimer_ns();
    while (ld_acquire_gpu_s32(p.g_ready + c) <= 0) {
      if (globaltimer_ns() - start > p.timeout_ns) return false;
      __nanosleep(128);
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, int OUT, int KIND = kKindBf16>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const Params p) {
  // Both kinds move 128-byte K rows per stage: 64 bf16 or 128 8-bit values.
  static_assert(KIND == kKindBf16 || (!A_MN && !B_MN), "8-bit operands are K-major only");
  constexpr int K_ELEMS = KIND == kKindBf16 ? BK : 2 * BK;
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  static_assert(TMEM_COLS <= 512, "accumulator does not fit in TMEM");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 32 * kEpilogueWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
        int m0, n_t, kb0, kb1;
        decode_unit(p, u, m0, n_t, kb0, kb1);
        const int n0 = n_t * BN;
        if (p.gather && !gather_rows_ready(p, n0, BN)) {
          report_status(p.status, kStatusTimeoutPeer);
          *abort_flag = 1;
          ok = false;
          break;
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (*abort_flag) { ok = false; break; }
          if (!mbar_wait(&empty[stage], phase ^ 1, p.timeout_ns)) {
            report_status(p.status, kStatusTimeoutProducer);
            *abort_flag = 1;
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          const int k0 = kb * K_ELEMS;
          if constexpr (A_MN) {
            tma_load_2d(a_dst, &tmA, &full[stage], m0, k0);
            tma_load_2d(a_dst + 8192, &tmA, &full[stage], m0 + 64, k0);
          } else {
            tma_load_2d(a_dst, &tmA, &full[stage], k0, m0);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(b_dst + j * 8192, &tmB, &full[stage], n0 + 64 * j, k0);
          } else {
            tma_load_2d(b_dst, &tmB, &full[stage], k0, n0);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Never leave the CTA with a TMA write still landing in its shared memory.
      for (int s = 0; s < STAGES; ++s) {
        if ((issued_mask >> s) & 1u) {
          if (!mbar_wait(&full[s], (issued_parity >> s) & 1u, p.timeout_ns))
            report_status(p.status, kStatusTimeoutDrain);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = KIND == kKindBf16
                                     ? idesc_bf16_f32(BM, BN, A_MN, B_MN)
                                     : idesc_f8_f32(BM, BN, (KIND - 1) & 1, ((KIND - 1) >> 1) & 1);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      bool issued_any = false;
      for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x, ++local) {
        int m0, n_t, kb0, kb1;
        decode_unit(p, u, m0, n_t, kb0, kb1);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (*abort_flag || !mbar_wait(&tempty[acc], acc_phase ^ 1, p.timeout_ns)) {
          report_status(p.status, kStatusTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (*abort_flag || !mbar_wait(&full[stage], phase, p.timeout_ns)) {
            report_status(p.status, kStatusTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? smem_desc_sw128(a_addr + kk * 2048, 8192, 1024)
                                     : smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc_sw128(b_addr + kk * 2048, 8192, 1024)
                                     : smem_desc_sw128(b_addr + kk * 32, 16, 1024);
            // One instruction consumes 32 bytes of K either way: K=16 bf16 or K=32 fp8.
            if constexpr (KIND == kKindBf16)
              umma_f16_ss(d_tmem, ad, bd, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
            else
              umma_f8_ss(d_tmem, ad, bd, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      // Every MMA must have retired before TMEM is released.
      if (issued_any) {
        umma_commit(drain);
        if (!mbar_wait(drain, 0, p.timeout_ns)) report_status(p.status, kStatusTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // (with a fused gather, the epilogue warps first assemble this CTA's share
    // of the weight; they have no tile to store before the first MMAs finish)
    if (p.gather) gather_weight_chunks(p, blockIdx.x, gridDim.x, threadIdx.x - 64);
    const int quad = warp & 3;  // TMEM lanes this warp may access: [32*quad, 32*quad+32)
    const int row_local = quad * 32 + lane;
    constexpr int kChunksPerWarp = BN / 32 / (kEpilogueWarps / 4);
    const int chunk0 = ((warp - 2) / 4) * kChunksPerWarp;  // this warp's column half
    int local = 0;
    float operand_scale = 1.f;
    if constexpr (KIND != kKindBf16) {
      if (p.scales != nullptr) operand_scale = p.scales[0] * p.scales[1];
    }
    for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++local) {
      int m0, n_t, kb0, kb1;
      decode_unit(p, u, m0, n_t, kb0, kb1);
      const int n0 = n_t * BN;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      bool ok = (*abort_flag == 0) && mbar_wait(&tfull[acc], acc_phase, p.timeout_ns);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) report_status(p.status, kStatusTimeoutEpilogue);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int m = m0 + row_local;
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = chunk0; c < chunk0 + kChunksPerWarp; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait();
        if constexpr (KIND != kKindBf16) {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * operand_scale);
        }
        const int n_base = n0 + c * 32;
        if (m < p.M && n_base < p.N) epilogue_row32<EPI, OUT>(p, m, n_base, r);
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, int OUT, int KIND = kKindBf16>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int grid,
            cudaStream_t stream, int device) {
  auto kern = gemm_kernel<BN, STAGES, A_MN, B_MN, EPI, OUT, KIND>;
  constexpr size_t smem = 1024 + STAGES * (BM * BK * 2 + BN * BK * 2) + 256;
  static bool configured[64] = {false};
  if (device < 0 || device >= 64 || !configured[device]) {
    RX_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
    if (device >= 0 && device < 64) configured[device] = true;
  }
  if (p.gather) {
    // CTAs wait for chunks that other CTAs of the grid copy: guarantee co-residency.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    RX_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, p));
    return;
  }
  kern<<<grid, kThreads, smem, stream>>>(ta, tb, p);
  RX_CUDA_CHECK(cudaGetLastError());
}

// ============================================================================
// CTA-pair variant (cta_group::2). A cluster of two CTAs owns a 256 x 256
// output tile: CTA r loads A rows [128r, 128r + 128) and B rows
// [128r, 128r + 128) of the tile into its own shared memory; the even CTA
// issues one M=256, N=256 tcgen05.mma per K=16 step that reads both CTAs'
// operands and leaves each CTA's 128 accumulator rows in its own TMEM. Each
// CTA thus moves half the B tile per stage (32 KB instead of 48 KB), which
// leaves room for 6 stages.
//
// Barriers: every stage's TMA loads (from both CTAs) complete on the even
// CTA's full barrier; the MMA completion is committed to the empty / TMEM-full
// / drain barriers of both CTAs; both CTAs' epilogue warps arrive on the even
// CTA's TMEM-empty barrier.
// ============================================================================
constexpr int kPairStages = 6;

// bf16 outputs leave through shared memory and TMA tile stores: each
// epilogue warp stages its 32 x 32 piece (double-buffered, 64-byte swizzle)
// and one lane issues the store, instead of 32 lanes writing 64 bytes to 32
// different rows.
template <int OUT>
constexpr int pair_stage_bytes() { return OUT == OUT_BF16 ? kEpilogueWarps * 2 * 2048 : 0; }

template <bool A_MN, bool B_MN, int EPI, int OUT>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmAux,
                     const Params p) {
  constexpr int BN = 256;           // pair tile columns
  constexpr int HALF_N = BN / 2;    // B rows loaded by each CTA
  constexpr int STAGES = kPairStages;
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = HALF_N * BK * 2;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  constexpr bool kTileStore = OUT == OUT_BF16;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = base;
  uint8_t* sB = base + STAGES * A_BYTES;
  uint8_t* sC = sB + STAGES * B_BYTES;  // 1024-aligned staging for tile stores
  uint64_t* full = reinterpret_cast<uint64_t*>(sC + pair_stage_bytes<OUT>());
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const int clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpilogueWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_map(&tmA);
    tma_prefetch_map(&tmB);
    if constexpr (kTileStore) tma_prefetch_map(&tmC);
    if constexpr (kTileStore && (EPI & EPI_GELU) != 0) tma_prefetch_map(&tmAux);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto decode = [&](int u, int& m0, int& n0, int& kb0, int& kb1) {
    const int n_t = u % p.n_tiles;
    const int t = u / p.n_tiles;
    const int m_t = t % p.m_tiles;
    const int split = t / p.m_tiles;
    m0 = m_t * (2 * BM);
    n0 = n_t * BN;
    kb0 = split * p.kb_per_split;
    kb1 = min(p.kb_total, kb0 + p.kb_per_split);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t full_leader0 = mapa_shared(smem_u32(&full[0]), 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = cluster; ok && u < p.num_units; u += clusters) {
        int m0, n0, kb0, kb1;
        decode(u, m0, n0, kb0, kb1);
        const int my_m = m0 + static_cast<int>(rank) * BM;
        const int my_n = n0 + static_cast<int>(rank) * HALF_N;
        if (p.gather && !gather_rows_ready(p, my_n, HALF_N)) {
          report_status(p.status, kStatusTimeoutPeer);
          *abort_flag = 1;
          ok = false;
          break;
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (*abort_flag) { ok = false; break; }
          if (!mbar_wait(&empty[stage], phase ^ 1, p.timeout_ns)) {
            report_status(p.status, kStatusTimeoutProducer);
            *abort_flag = 1;
            ok = false;
            break;
          }
          // The even CTA expects the bytes of both CTAs' loads.
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (A_BYTES + B_BYTES));
          const uint32_t bar = full_leader0 + stage * 8;
          uint8_t* a_dst = sA + stage * A_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          const int k0 = kb * BK;
          if constexpr (A_MN) {
            tma_load_2d_pair(a_dst, &tmA, bar, my_m, k0);
            tma_load_2d_pair(a_dst + 8192, &tmA, bar, my_m + 64, k0);
          } else {
            tma_load_2d_pair(a_dst, &tmA, bar, k0, my_m);
          }
          if constexpr (B_MN) {
            tma_load_2d_pair(b_dst, &tmB, bar, my_n, k0);
            tma_load_2d_pair(b_dst + 8192, &tmB, bar, my_n + 64, k0);
          } else {
            tma_load_2d_pair(b_dst, &tmB, bar, k0, my_n);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Every load issued by this CTA was consumed by an MMA before the MMA
      // committed the stage's empty barrier; wait for the last commits.
      for (int s = 0; s < STAGES; ++s) {
        if (!mbar_wait(&empty[stage], phase ^ 1, p.timeout_ns)) {
          report_status(p.status, kStatusTimeoutDrain);
          break;
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(2 * BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int u = cluster; ok && u < p.num_units; u += clusters, ++local) {
        int m0, n0, kb0, kb1;
        decode(u, m0, n0, kb0, kb1);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (*abort_flag || !mbar_wait(&tempty[acc], acc_phase ^ 1, p.timeout_ns)) {
          report_status(p.status, kStatusTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (*abort_flag || !mbar_wait(&full[stage], phase, p.timeout_ns)) {
            report_status(p.status, kStatusTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? smem_desc_sw128(a_addr + kk * 2048, 8192, 1024)
                                     : smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc_sw128(b_addr + kk * 2048, 8192, 1024)
                                     : smem_desc_sw128(b_addr + kk * 32, 16, 1024);
            umma_f16_ss_pair(d_tmem, ad, bd, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(&tfull[acc], 0x3);
      }
      // Signal both CTAs once every MMA of this pair has retired.
      umma_commit_pair(drain, 0x3);
    }
    if (lane == 0 && !mbar_wait(drain, 0, p.timeout_ns)) report_status(p.status, kStatusTimeoutDrain);
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    // (a fused FSDP gather first: see the single-CTA kernel)
    if (p.gather) gather_weight_chunks(p, blockIdx.x, gridDim.x, threadIdx.x - 64);
    const int quad = warp & 3;
    const int row_local = quad * 32 + lane;
    constexpr int kChunksPerWarp = BN / 32 / (kEpilogueWarps / 4);
    const int chunk0 = ((warp - 2) / 4) * kChunksPerWarp;
    const uint32_t tempty_leader = mapa_shared(smem_u32(&tempty[0]), 0);
    int local = 0;
    uint32_t store_seq = 0;
    for (int u = cluster; u < p.num_units; u += clusters, ++local) {
      int m0, n0, kb0, kb1;
      decode(u, m0, n0, kb0, kb1);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      bool ok = (*abort_flag == 0) && mbar_wait(&tfull[acc], acc_phase, p.timeout_ns);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) report_status(p.status, kStatusTimeoutEpilogue);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int m = m0 + static_cast<int>(rank) * BM + row_local;
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      constexpr bool kSide = (EPI & (EPI_RESID | EPI_DGELU)) != 0;
      const __nv_bfloat16* side_src = (EPI & EPI_RESID) != 0 ? p.residual : p.aux_in;
      const int64_t side_ld = (EPI & EPI_RESID) != 0 ? p.ld_res : p.ld_aux_in;
      const int side_row0 = m0 + static_cast<int>(rank) * BM + quad * 32;
      uint4 side_next[4];  // the next chunk's residual / saved-derivative tile, in flight
      if constexpr (kTileStore && kSide) {
        if (n0 + chunk0 * 32 < p.N && side_row0 < p.M)
          warp_fetch_tile32(side_src, side_ld, side_row0, n0 + chunk0 * 32, p.M, p.N, lane, side_next);
      }
#pragma unroll 1
      for (int c = chunk0; c < chunk0 + kChunksPerWarp; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait();
        const int n_base = n0 + c * 32;
        if constexpr (kTileStore) {
          const int row0 = side_row0;
          uint4 side_cur[4];
          if constexpr (kSide) {
#pragma unroll
            for (int q = 0; q < 4; ++q) side_cur[q] = side_next[q];
            if (c + 1 < chunk0 + kChunksPerWarp && n_base + 32 < p.N && row0 < p.M)
              warp_fetch_tile32(side_src, side_ld, row0, n_base + 32, p.M, p.N, lane, side_next);
          }
          if (n_base < p.N && row0 < p.M) {  // warp-uniform
            uint8_t* buf = sC + ((warp - 2) * 2 + (store_seq & 1)) * 2048;
            if (lane == 0) tma_store_wait_read<1>();  // the store that last read `buf` is done reading
            __syncwarp();
            float side[32], v[32], pre[32];
            if constexpr (kSide) {
              warp_put_tile32_sw64(buf, lane, side_cur);
              __syncwarp();
              read_row32_sw64(buf, lane, side);
              __syncwarp();  // every lane has its row before the buffer is overwritten
            }
            epilogue_tile_values32<EPI>(p, m, n_base, r, side, v, pre);
            stage_row32_sw64(buf, lane, v);
            fence_proxy_async_smem();
            __syncwarp();
            if constexpr ((EPI & EPI_COLSUM) != 0) {
              // lane c sums column n_base + c over the piece's rows (rows >= M hold zeros)
              float cs = 0.f;
              const int piece = lane >> 3, within = (lane & 7) * 2;
#pragma unroll 8
              for (int rr = 0; rr < 32; ++rr)
                cs += __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(
                    buf + rr * 64 + ((piece ^ ((rr >> 1) & 3)) * 16) + within));
              if (n_base + lane < p.N) atomicAdd(p.colsum + n_base + lane, cs);
            }
            if (lane == 0) {
              tma_store_2d(&tmC, buf, n_base, row0);
              tma_store_commit();
            }
            ++store_seq;
            if constexpr ((EPI & EPI_GELU) != 0) {
              // gelu'(z) through the other staging buffer: only the store issued
              // two stores ago must have finished reading it
              uint8_t* buf2 = sC + ((warp - 2) * 2 + (store_seq & 1)) * 2048;
              if (lane == 0) tma_store_wait_read<1>();
              __syncwarp();
              stage_row32_sw64(buf2, lane, pre);
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmAux, buf2, n_base, row0);
                tma_store_commit();
              }
              ++store_seq;
            }
          }
        } else {
          if (m < p.M && n_base < p.N) epilogue_row32<EPI, OUT>(p, m, n_base, r);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader + acc * 8);
    }
    if constexpr (kTileStore) {
      if (lane == 0) tma_store_wait<0>();  // every tile store has landed before the CTA exits
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its peer may still signal it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, TMEM_COLS);
}

template <bool A_MN, bool B_MN, int EPI, int OUT>
void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int grid,
                 cudaStream_t stream, int device) {
  auto kern = gemm_pair_kernel<A_MN, B_MN, EPI, OUT>;
  constexpr size_t smem = 1024 + kPairStages * (BM * BK * 2 + 128 * BK * 2) + pair_stage_bytes<OUT>() + 256;
  static_assert(smem <= 232448, "pair GEMM shared memory exceeds the opt-in limit");
  CUtensorMap tc{}, taux{};
  if constexpr (OUT == OUT_BF16) {
    tc = make_tmap_2d_bf16_store(p.C, p.M, p.N, p.ldc);
    if constexpr ((EPI & EPI_GELU) != 0) taux = make_tmap_2d_bf16_store(p.aux_out, p.M, p.N, p.ld_aux_out);
  }
  static bool configured[64] = {false};
  if (device < 0 || device >= 64 || !configured[device]) {
    RX_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
    if (device >= 0 && device < 64) configured[device] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // a fused gather makes CTAs wait for chunks copied by other CTAs: co-resident grid
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = p.gather ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = p.gather ? 2 : 1;
  RX_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, taux, p));
}

using LaunchFn = void (*)(const CUtensorMap&, const CUtensorMap&, const Params&, int, cudaStream_t,
                          int);

// Variant tables, one translation unit each so they compile in parallel.
LaunchFn pick_forward(int epi, int out);
LaunchFn pick_dgrad(int epi, int out);
LaunchFn pick_wgrad(int epi, int out);
LaunchFn pick_forward_pair(int epi, int out);
LaunchFn pick_dgrad_pair(int epi, int out);
LaunchFn pick_wgrad_pair(int epi, int out);

}  // namespace gemm
}  // namespace rx
