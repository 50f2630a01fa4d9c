// Variable-length (packed, padding-free) multi-head attention for sm_100a,
// head dimension 64 or 128, bf16 operands, fp32 softmax and accumulation.
//
// Sequences are packed back to back ([T, heads * D] rows addressed through
// cu_seqlens), so no FLOP is spent on padding tokens. Supported masks: key
// validity (sequence end), causal, and a symmetric sliding window
// |i - j| <= window (ModernBERT local layers). Grouped-query attention maps
// query head h to key/value head h / heads_per_kv.
//
// Forward: one CTA = 4 warps = 64 queries of one (sequence, head); key/value
// tiles of 64 stream through double-buffered cp.async shared memory; online
// softmax in base 2; the log-sum-exp is saved for the backward pass.
// Backward: one CTA = 64 keys of one (sequence, key/value head); loops over
// the query heads of its group and their query tiles, accumulates dK and dV
// in registers, and adds dQ partials with fp32 vector atomics into a
// [T, heads * D] accumulator.
// Warp-level math uses mma.sync m16n8k16 with ldmatrix fragment loads.
//
// Reference parity: `dot_product_attention` with padding / window / causal
// masks (src/representax/models/components.py:187-235), sliding windows
// (src/representax/models/modernvbert/model.py:217-230) and GQA
// (src/representax/models/qwen3_vl/text.py:188-199).
#include "attention_kernels.cuh"
#include <algorithm>

#include "common.h"
#include "sm100.cuh"

namespace rx {
namespace attn {

// Tile constants and the kernel parameter block are shared with the other
// host entry points through attention_kernels.cuh.

// Byte offset of 16-byte chunk `chunk` of row `row` in a [rows][W] bf16 tile
// whose chunks are XOR-swizzled by the row's low 3 bits (bank-conflict-free
// ldmatrix).
template <int W>
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return static_cast<uint32_t>((row * (W / 8) + (chunk ^ (row & 7))) * 16);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Load a [64 rows][D] bf16 tile (rows row0.. of a packed matrix) into
// swizzled shared memory; rows at or beyond `rows_valid` are zero-filled.
template <int D>
__device__ __forceinline__ void load_tile(uint32_t smem, const __nv_bfloat16* base, int64_t ld,
                                          int row0, int rows_valid) {
  constexpr int kChunks = D / 8;
#pragma unroll
  for (int i = 0; i < (64 * kChunks) / kThreads; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    const int r = idx / kChunks;
    const int c = idx % kChunks;
    const bool valid = (row0 + r) < rows_valid;
    const __nv_bfloat16* src = base + static_cast<int64_t>(valid ? row0 + r : 0) * ld + c * 8;
    cp_async16(smem + swz<D>(r, c), src, valid);
  }
}

// Is key j visible from query i (both sequence-relative)?
__device__ __forceinline__ bool visible(const Params& p, int i, int j, int len) {
  if (j >= len) return false;
  if (p.causal && j > i) return false;
  if (p.window >= 0 && (j - i > p.window || i - j > p.window)) return false;
  return true;
}

__device__ __forceinline__ void key_range(const Params& p, int q_lo, int q_hi, int len, int& k_lo,
                                          int& k_hi) {
  k_lo = 0;
  k_hi = len;
  if (p.causal) k_hi = min(k_hi, q_hi);
  if (p.window >= 0) {
    k_lo = max(0, q_lo - p.window);
    k_hi = min(k_hi, q_hi - 1 + p.window + 1);
  }
}

// ===================================================================== forward
template <int D>
__global__ void __launch_bounds__(kThreads, D == 64 ? 4 : 1) attn_fwd_kernel(const Params p) {
  const int qb = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int start = p.cu_seqlens[b];
  const int len = p.cu_seqlens[b + 1] - start;
  if (qb * BM >= len) return;
  const int kvh = h / p.heads_per_kv;

  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK[2] = {sQ + 64 * D * 2, sQ + 2 * 64 * D * 2};
  const uint32_t sV[2] = {sQ + 3 * 64 * D * 2, sQ + 4 * 64 * D * 2};

  const __nv_bfloat16* qbase = p.q + static_cast<int64_t>(start) * p.ldq + h * D;
  const __nv_bfloat16* kbase = p.k + static_cast<int64_t>(start) * p.ldk + kvh * D;
  const __nv_bfloat16* vbase = p.v + static_cast<int64_t>(start) * p.ldv + kvh * D;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int q_lo = qb * BM;
  const int q_hi = min(len, q_lo + BM);
  int k_lo, k_hi;
  key_range(p, q_lo, q_hi, len, k_lo, k_hi);
  const int kb_first = k_lo / BN;
  const int kb_last = (k_hi + BN - 1) / BN;  // exclusive

  load_tile<D>(sQ, qbase, p.ldq, q_lo, len);
  if (kb_first < kb_last) {
    load_tile<D>(sK[0], kbase, p.ldk, kb_first * BN, len);
    load_tile<D>(sV[0], vbase, p.ldv, kb_first * BN, len);
  }
  cp_async_commit();

  // Row state for rows (warp*16 + g) and (+8).
  float m_r[2] = {-INFINITY, -INFINITY};
  float l_r[2] = {0.f, 0.f};
  float o_acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o_acc[i][0] = o_acc[i][1] = o_acc[i][2] = o_acc[i][3] = 0.f;
  uint32_t qf[D / 16][4];
  const int qi0 = q_lo + warp * 16 + g;  // sequence-relative query rows qi0, qi0 + 8

  for (int kb = kb_first; kb < kb_last; ++kb) {
    const int buf = (kb - kb_first) & 1;
    if (kb + 1 < kb_last) {
      load_tile<D>(sK[buf ^ 1], kbase, p.ldk, (kb + 1) * BN, len);
      load_tile<D>(sV[buf ^ 1], vbase, p.ldv, (kb + 1) * BN, len);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kb == kb_first) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int r = warp * 16 + (lane & 15);
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(sQ + swz<D>(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    // S = Q K^T for 16 rows x 64 keys.
    float s[BN / 8][4];
#pragma unroll
    for (int nb = 0; nb < BN / 8; ++nb) {
      s[nb][0] = s[nb][1] = s[nb][2] = s[nb][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < D / 16; kk += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = nb * 8 + (lane & 7);
        const int c = kk * 2 + (lane >> 3);
        ldsm_x4(sK[buf] + swz<D>(r, c), b0, b1, b2, b3);
        mma16816(s[nb], qf[kk], b0, b1);
        mma16816(s[nb], qf[kk + 1], b2, b3);
      }
    }
    // Mask, online softmax.
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < BN / 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = kb * BN + nb * 8 + 2 * t + (e & 1);
        const int i = qi0 + (e >> 1) * 8;
        float x = s[nb][e] * p.scale_log2;
        if (p.rel_lut != nullptr)
          x += __ldg(p.rel_lut + static_cast<int64_t>(h) * (2 * p.lut_len - 1) + (j - i + p.lut_len - 1)) *
               1.4426950408889634f;
        if (!visible(p, i, j, len)) x = -INFINITY;
        s[nb][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2], m_use[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const float m_new = fmaxf(m_r[r], mx[r]);
      m_use[r] = (m_new == -INFINITY) ? 0.f : m_new;
      alpha[r] = (m_r[r] == -INFINITY) ? 0.f : exp2f(m_r[r] - m_use[r]);
      m_r[r] = m_new;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nb = 0; nb < BN / 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pv = exp2f(s[nb][e] - m_use[e >> 1]);
        s[nb][e] = pv;
        rs[e >> 1] += pv;  // the normaliser uses the probabilities before dropout
      }
    }
    if (p.pdrop.threshold != 0u) {
      // Rows qi0 and qi0 + 8 need two 2x2 blocks; the lanes of rows g and g ^ 1
      // (lane ^ 4) need the same two blocks, so each lane generates one and
      // the pair swaps halves: even-g lanes make the block of rows (qi0, qi0+1),
      // odd-g lanes that of rows (qi0 + 7, qi0 + 8).
      const bool odd = (g & 1) != 0;
      const int i_sel = odd ? qi0 + 8 : qi0;
#pragma unroll
      for (int nb = 0; nb < BN / 8; ++nb) {
        const int j = kb * BN + nb * 8 + 2 * t;  // even key index of this thread's pair
        const Philox4 b = dropout_block(p.pdrop, static_cast<uint32_t>(start + (i_sel & ~1)),
                                        (static_cast<uint32_t>(h) << 16) | static_cast<uint32_t>(j >> 1));
        const uint32_t got0 = __shfl_xor_sync(0xffffffffu, odd ? b.x : b.z, 4);
        const uint32_t got1 = __shfl_xor_sync(0xffffffffu, odd ? b.y : b.w, 4);
        // words for (row qi0, cols j, j+1) and (row qi0 + 8, cols j, j+1)
        const uint32_t w00 = odd ? got0 : b.x, w01 = odd ? got1 : b.y;
        const uint32_t w10 = odd ? b.z : got0, w11 = odd ? b.w : got1;
        const uint32_t th = p.pdrop.threshold;
        const float sc = p.pdrop.scale;
        s[nb][0] = w00 >= th ? s[nb][0] * sc : 0.f;
        s[nb][1] = w01 >= th ? s[nb][1] * sc : 0.f;
        s[nb][2] = w10 >= th ? s[nb][2] * sc : 0.f;
        s[nb][3] = w11 >= th ? s[nb][3] * sc : 0.f;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_r[r] = l_r[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) {
      o_acc[nb][0] *= alpha[0];
      o_acc[nb][1] *= alpha[0];
      o_acc[nb][2] *= alpha[1];
      o_acc[nb][3] *= alpha[1];
    }
    // O += P V.
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      uint32_t a[4];
      a[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int nb = 0; nb < D / 8; nb += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = nb + (lane >> 4);
        ldsm_x4_t(sV[buf] + swz<D>(r, c), b0, b1, b2, b3);
        mma16816(o_acc[nb], a, b0, b1);
        mma16816(o_acc[nb + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // Normalise and store.
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int i = qi0 + r * 8;
    if (i >= len) continue;
    const float inv = l_r[r] > 0.f ? 1.f / l_r[r] : 0.f;
    __nv_bfloat16* orow = p.o + static_cast<int64_t>(start + i) * p.ldo + h * D;
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) {
      *reinterpret_cast<uint32_t*>(orow + nb * 8 + 2 * t) =
          pack_bf16(o_acc[nb][2 * r] * inv, o_acc[nb][2 * r + 1] * inv);
    }
    if (t == 0) {
      p.lse[static_cast<int64_t>(h) * p.total_tokens + start + i] =
          l_r[r] > 0.f ? m_r[r] + log2f(l_r[r]) : INFINITY;
    }
  }
}

// ============================================================ backward prep
// dvec[h, t] = sum_d dO[t, h, d] * O[t, h, d]  (one warp per (t, h)).
__global__ void attn_dvec_kernel(const __nv_bfloat16* __restrict__ o, int64_t ldo,
                                 const __nv_bfloat16* __restrict__ dO, int64_t ld_do,
                                 float* __restrict__ dvec, int total, int heads, int head_dim) {
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<int64_t>(total) * heads) return;
  const int64_t tok = gw / heads;
  const int h = static_cast<int>(gw % heads);
  const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(o + tok * ldo + h * head_dim);
  const __nv_bfloat162* d = reinterpret_cast<const __nv_bfloat162*>(dO + tok * ld_do + h * head_dim);
  float s = 0.f;
  for (int i = lane; i < head_dim / 2; i += 32) {
    const float2 fa = __bfloat1622float2(a[i]), fd = __bfloat1622float2(d[i]);
    s += fa.x * fd.x + fa.y * fd.y;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) dvec[static_cast<int64_t>(h) * total + tok] = s;
}

// Backward prep, one pass over the tokens: dvec[h, t] = sum_d dO[t, h, d] *
// O[t, h, d], and the fp32 dQ accumulator row of (t, h) is zeroed. A group of
// D / 8 threads owns one (t, h): each thread loads 16 bytes of O and of dO and
// stores 8 zero floats; the group sums with shuffles.
template <int D>
__global__ void __launch_bounds__(256)
    attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ o, int64_t ldo, const __nv_bfloat16* __restrict__ dO,
                         int64_t ld_do, float* __restrict__ dvec, float* __restrict__ dq_acc, int total, int heads) {
  constexpr int G = D / 8;  // threads per (token, head)
  const int64_t gid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x);
  const int64_t item = gid / G;
  const int c = static_cast<int>(gid % G);
  const bool live = item < static_cast<int64_t>(total) * heads;
  float s = 0.f;
  int64_t tok = 0;
  int h = 0;
  if (live) {
    tok = item / heads;
    h = static_cast<int>(item % heads);
    const uint4 a = reinterpret_cast<const uint4*>(o + tok * ldo + h * D)[c];
    const uint4 d = reinterpret_cast<const uint4*>(dO + tok * ld_do + h * D)[c];
    const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&d);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fa = __bfloat1622float2(a2[j]), fd = __bfloat1622float2(d2[j]);
      s += fa.x * fd.x + fa.y * fd.y;
    }
    float4* z = reinterpret_cast<float4*>(dq_acc + tok * (static_cast<int64_t>(heads) * D) + h * D + c * 8);
    z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int off = G / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (live && c == 0) dvec[static_cast<int64_t>(h) * total + tok] = s;
}

// dq[t, h*D + d] = bf16(dq_acc[t, h*D + d])
__global__ void attn_dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq,
                                       int64_t ld_dq, int total, int width) {
  const int64_t idx = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (idx >= static_cast<int64_t>(total) * width) return;
  const int64_t tok = idx / width, col = idx % width;
  const float4 v = *reinterpret_cast<const float4*>(acc + idx);
  uint2 w;
  w.x = pack_bf16(v.x, v.y);
  w.y = pack_bf16(v.z, v.w);
  *reinterpret_cast<uint2*>(dq + tok * ld_dq + col) = w;
}

// dq = bf16(dq_acc) with the column sums of the rounded values added into
// `colsum` (the query part of a fused QKV bias gradient). One CTA per slice
// of rows; thread (g, c) owns 4 columns of rows g, g + G, ... with eight
// 16-byte loads in flight; row groups meet in shared memory, so each column
// takes one atomic per CTA.
__global__ void __launch_bounds__(1024)
    attn_dq_convert_colsum_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, int64_t ld_dq,
                                  int total, int width, int slice, float* __restrict__ colsum) {
  extern __shared__ float part[];  // [groups][width]
  const int chunks = width >> 2;
  const int groups = blockDim.x / chunks;
  const int c = threadIdx.x % chunks, g = threadIdx.x / chunks;
  const int r0 = blockIdx.x * slice, r1 = min(total, r0 + slice);
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  if (g < groups) {
    for (int r = r0 + g; r < r1; r += 8 * groups) {
      // unconditional loads (rows past the slice re-read its last row; they
      // are neither stored nor summed) so that all eight are in flight at once
      uint4 w[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int rr = min(r + u * groups, r1 - 1);
        w[u] = ldg_v4_issue(reinterpret_cast<const float4*>(acc + static_cast<int64_t>(rr) * width) + c);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) hold_v4(w[u]);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int rr = r + u * groups;
        if (rr < r1) {
          const __nv_bfloat162 lo = __floats2bfloat162_rn(__uint_as_float(w[u].x), __uint_as_float(w[u].y));
          const __nv_bfloat162 hi = __floats2bfloat162_rn(__uint_as_float(w[u].z), __uint_as_float(w[u].w));
          uint2 o;
          o.x = *reinterpret_cast<const uint32_t*>(&lo);
          o.y = *reinterpret_cast<const uint32_t*>(&hi);
          *reinterpret_cast<uint2*>(dq + static_cast<int64_t>(rr) * ld_dq + c * 4) = o;
          const float2 a = __bfloat1622float2(lo), b = __bfloat1622float2(hi);
          s[0] += a.x;
          s[1] += a.y;
          s[2] += b.x;
          s[3] += b.y;
        }
      }
    }
  }
  if (colsum == nullptr) return;
  if (groups == 1) {
    if (g == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) atomicAdd(colsum + c * 4 + j, s[j]);
    }
    return;
  }
  if (g < groups) {
#pragma unroll
    for (int j = 0; j < 4; ++j) part[g * width + c * 4 + j] = s[j];
  }
  __syncthreads();
  for (int col = threadIdx.x; col < width; col += blockDim.x) {
    float t = 0.f;
    for (int q = 0; q < groups; ++q) t += part[q * width + col];
    atomicAdd(colsum + col, t);
  }
}

// ==================================================================== backward
template <int D, bool GQA>
__global__ void __launch_bounds__(kThreads) attn_bwd_kernel(const Params p) {
  const int kbk = blockIdx.x;
  const int kvh = blockIdx.y;  // key/value head; its query heads are looped below
  const int b = blockIdx.z;
  const int start = p.cu_seqlens[b];
  const int len = p.cu_seqlens[b + 1] - start;
  if (kbk * BN >= len) return;

  // K, V, Q, dO tiles + dS^T tile (bf16) + lse/dvec for 64 queries.
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float s_lse[64];
  __shared__ float s_dv[64];
  __shared__ float s_diag[128];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + 64 * D * 2;
  const uint32_t sQ = sK + 2 * 64 * D * 2;
  const uint32_t sdO = sK + 3 * 64 * D * 2;
  const uint32_t sdS = sK + 4 * 64 * D * 2;  // [64 keys][64 queries] bf16, swizzled

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int k_lo = kbk * BN;
  const int k_hi = min(len, k_lo + BN);

  // Query range that can see this key block.
  int q_lo = 0, q_hi = len;
  if (p.causal) q_lo = k_lo;
  if (p.window >= 0) {
    q_lo = max(q_lo, k_lo - p.window);
    q_hi = min(q_hi, k_hi - 1 + p.window + 1);
  }
  const int qb_first = q_lo / BM;
  const int qb_last = (q_hi + BM - 1) / BM;

  const __nv_bfloat16* kbase = p.k + static_cast<int64_t>(start) * p.ldk + kvh * D;
  const __nv_bfloat16* vbase = p.v + static_cast<int64_t>(start) * p.ldv + kvh * D;
  load_tile<D>(sK, kbase, p.ldk, k_lo, len);
  load_tile<D>(sV, vbase, p.ldv, k_lo, len);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();

  // K and V fragments are re-read from shared memory per 32-wide k step of
  // the first products instead of being held for the whole loop: the
  // backward's accumulators already fill the register file.
  float dk_acc[D / 8][4], dv_acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk_acc[i][e] = dv_acc[i][e] = 0.f;

  const int kj0 = k_lo + warp * 16 + g;  // this thread's key rows kj0, kj0 + 8

  const int group = GQA ? p.heads_per_kv : 1;
  for (int h = kvh * group; h < (kvh + 1) * group; ++h)
  for (int qb = qb_first; qb < qb_last; ++qb) {
    const __nv_bfloat16* qbase = p.q + static_cast<int64_t>(start) * p.ldq + h * D;
    const __nv_bfloat16* dobase = p.dO + static_cast<int64_t>(start) * p.ld_do + h * D;
    const int q0 = qb * BM;
    load_tile<D>(sQ, qbase, p.ldq, q0, len);
    load_tile<D>(sdO, dobase, p.ld_do, q0, len);
    cp_async_commit();
    if (threadIdx.x < 64) {
      const int i = q0 + threadIdx.x;
      s_lse[threadIdx.x] = i < len ? p.lse[static_cast<int64_t>(h) * p.total_tokens + start + i] : INFINITY;
      s_dv[threadIdx.x] = i < len ? p.dvec[static_cast<int64_t>(h) * p.total_tokens + start + i] : 0.f;
    }
    cp_async_wait<0>();
    __syncthreads();

    // S^T = K Q^T (16 keys x 64 queries per warp) and dP^T = V dO^T.
    float st[BM / 8][4], dpt[BM / 8][4];
#pragma unroll
    for (int nb = 0; nb < BM / 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[nb][e] = dpt[nb][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; kk += 2) {
      uint32_t kf[2][4], vf[2][4];
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int r = warp * 16 + (lane & 15);
        const int c = (kk + h2) * 2 + (lane >> 4);
        ldsm_x4(sK + swz<D>(r, c), kf[h2][0], kf[h2][1], kf[h2][2], kf[h2][3]);
        ldsm_x4(sV + swz<D>(r, c), vf[h2][0], vf[h2][1], vf[h2][2], vf[h2][3]);
      }
#pragma unroll
      for (int nb = 0; nb < BM / 8; ++nb) {
        uint32_t b0, b1, b2, b3;
        const int r = nb * 8 + (lane & 7);
        const int c = kk * 2 + (lane >> 3);
        ldsm_x4(sQ + swz<D>(r, c), b0, b1, b2, b3);
        mma16816(st[nb], kf[0], b0, b1);
        mma16816(st[nb], kf[1], b2, b3);
        ldsm_x4(sdO + swz<D>(r, c), b0, b1, b2, b3);
        mma16816(dpt[nb], vf[0], b0, b1);
        mma16816(dpt[nb], vf[1], b2, b3);
      }
    }
    // P^T and dS^T.
    const bool drop = p.pdrop.threshold != 0u;
#pragma unroll
    for (int nb = 0; nb < BM / 8; ++nb) {
      // Keys kj0 and kj0 + 8 x queries i0, i0 + 1: two 2x2 blocks, shared with
      // the lane of key row g ^ 1 (lane ^ 4) as in the forward. Words per key
      // row: [0] = query i0, [1] = query i0 + 1.
      uint32_t kw[2][2] = {{0u, 0u}, {0u, 0u}};
      if (drop) {
        const int i0 = q0 + nb * 8 + 2 * t;  // even query index of this thread's pair
        const bool odd = (g & 1) != 0;
        const int j_sel = odd ? kj0 + 8 : kj0;
        const Philox4 b = dropout_block(p.pdrop, static_cast<uint32_t>(start + i0),
                                        (static_cast<uint32_t>(h) << 16) | static_cast<uint32_t>(j_sel >> 1));
        const uint32_t got0 = __shfl_xor_sync(0xffffffffu, odd ? b.x : b.y, 4);
        const uint32_t got1 = __shfl_xor_sync(0xffffffffu, odd ? b.z : b.w, 4);
        // word (i & 1) * 2 + (j & 1): even key -> x (i0), z (i0 + 1); odd key -> y, w
        kw[0][0] = odd ? got0 : b.x;
        kw[0][1] = odd ? got1 : b.z;
        kw[1][0] = odd ? b.y : got0;
        kw[1][1] = odd ? b.w : got1;
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = nb * 8 + 2 * t + (e & 1);
        const int j = kj0 + (e >> 1) * 8;
        const int i = q0 + qi;
        float pv = 0.f;
        float bias = 0.f;
        if (p.rel_lut != nullptr && i < len && j < len)
          bias = __ldg(p.rel_lut + static_cast<int64_t>(h) * (2 * p.lut_len - 1) + (j - i + p.lut_len - 1)) *
                 1.4426950408889634f;
        if (i < len && visible(p, i, j, len)) pv = exp2f(st[nb][e] * p.scale_log2 + bias - s_lse[qi]);
        if (drop) {
          // dS = P * (mask * dP / (1 - p) - D); dV uses the dropped probabilities
          const bool keep = kw[e >> 1][e & 1] >= p.pdrop.threshold;
          const float dp = keep ? dpt[nb][e] * p.pdrop.scale : 0.f;
          dpt[nb][e] = pv * (dp - s_dv[qi]);
          st[nb][e] = keep ? pv * p.pdrop.scale : 0.f;
        } else {
          st[nb][e] = pv;
          dpt[nb][e] = pv * (dpt[nb][e] - s_dv[qi]);
        }
      }
    }
    if (p.drel != nullptr) {
      // dS summed along diagonals d = j - i (127 of them in a 64 x 64 tile)
      // in shared memory, then one global atomic per diagonal.
      for (int x = threadIdx.x; x < 128; x += blockDim.x) s_diag[x] = 0.f;
      __syncthreads();
      const int d0 = k_lo - q0 - 63;  // diagonal of (query q0 + 63, key k_lo)
#pragma unroll
      for (int nb = 0; nb < BM / 8; ++nb) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = q0 + nb * 8 + 2 * t + (e & 1);
          const int j = kj0 + (e >> 1) * 8;
          if (i < len && j < len && dpt[nb][e] != 0.f) atomicAdd(&s_diag[j - i - d0], dpt[nb][e]);
        }
      }
      __syncthreads();
      float* dst = p.drel + static_cast<int64_t>(h) * (2 * p.lut_len - 1) + p.lut_len - 1 + d0;
      for (int x = threadIdx.x; x < 127; x += blockDim.x) {
        const float v = s_diag[x];
        if (v != 0.f) atomicAdd(dst + x, v);
      }
    }
    // dV += P^T dO ; dK += dS^T Q  (k = queries).
#pragma unroll
    for (int kk = 0; kk < BM / 16; ++kk) {
      uint32_t ap[4], ad[4];
      ap[0] = pack_bf16(st[2 * kk][0], st[2 * kk][1]);
      ap[1] = pack_bf16(st[2 * kk][2], st[2 * kk][3]);
      ap[2] = pack_bf16(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      ap[3] = pack_bf16(st[2 * kk + 1][2], st[2 * kk + 1][3]);
      ad[0] = pack_bf16(dpt[2 * kk][0], dpt[2 * kk][1]);
      ad[1] = pack_bf16(dpt[2 * kk][2], dpt[2 * kk][3]);
      ad[2] = pack_bf16(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]);
      ad[3] = pack_bf16(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3]);
#pragma unroll
      for (int nb = 0; nb < D / 8; nb += 2) {
        uint32_t b0, b1, b2, b3;
        const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = nb + (lane >> 4);
        ldsm_x4_t(sdO + swz<D>(r, c), b0, b1, b2, b3);
        mma16816(dv_acc[nb], ap, b0, b1);
        mma16816(dv_acc[nb + 1], ap, b2, b3);
        ldsm_x4_t(sQ + swz<D>(r, c), b0, b1, b2, b3);
        mma16816(dk_acc[nb], ad, b0, b1);
        mma16816(dk_acc[nb + 1], ad, b2, b3);
      }
      // Stash dS^T (rows = this warp's keys) for the dQ product.
      const int key_r = warp * 16 + g;
      const int qcol = kk * 16 + 2 * t;  // element column within the 64-query row
      uint8_t* base = smem + 4 * 64 * D * 2;
      *reinterpret_cast<uint32_t*>(base + swz<64>(key_r, qcol >> 3) + (qcol & 7) * 2) = ad[0];
      *reinterpret_cast<uint32_t*>(base + swz<64>(key_r + 8, qcol >> 3) + (qcol & 7) * 2) = ad[1];
      *reinterpret_cast<uint32_t*>(base + swz<64>(key_r, (qcol + 8) >> 3) + (qcol & 7) * 2) = ad[2];
      *reinterpret_cast<uint32_t*>(base + swz<64>(key_r + 8, (qcol + 8) >> 3) + (qcol & 7) * 2) = ad[3];
    }
    __syncthreads();
    // dQ[64 q x D] += dS K : warp w handles queries w*16..w*16+15, k = keys.
    {
      float dq[D / 8][4];
#pragma unroll
      for (int i = 0; i < D / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        uint32_t a[4];
        {
          const int mi = lane >> 3;
          const int r = kk * 16 + (lane & 7) + (mi >> 1) * 8;  // key row in dS^T
          const int c = warp * 2 + (mi & 1);                     // query chunk
          ldsm_x4_t(sdS + swz<64>(r, c), a[0], a[1], a[2], a[3]);
        }
#pragma unroll
        for (int nb = 0; nb < D / 8; nb += 2) {
          uint32_t b0, b1, b2, b3;
          const int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int c = nb + (lane >> 4);
          ldsm_x4_t(sK + swz<D>(r, c), b0, b1, b2, b3);
          mma16816(dq[nb], a, b0, b1);
          mma16816(dq[nb + 1], a, b2, b3);
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int i = q0 + warp * 16 + g + r * 8;
        if (i < len) {
          float* row = p.dq_acc + static_cast<int64_t>(start + i) * (p.heads * D) + h * D;
#pragma unroll
          for (int nb = 0; nb < D / 8; ++nb) {
            atomicAdd(reinterpret_cast<float2*>(row + nb * 8 + 2 * t),
                      make_float2(dq[nb][2 * r] * p.scale, dq[nb][2 * r + 1] * p.scale));
          }
        }
      }
    }
    __syncthreads();
  }

  // Store dK (scaled) and dV for this warp's 16 keys.
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int j = kj0 + r * 8;
    if (j >= len) continue;
    __nv_bfloat16* dkrow = p.dk + static_cast<int64_t>(start + j) * p.ld_dk + kvh * D;
    __nv_bfloat16* dvrow = p.dv + static_cast<int64_t>(start + j) * p.ld_dv + kvh * D;
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) {
      *reinterpret_cast<uint32_t*>(dkrow + nb * 8 + 2 * t) =
          pack_bf16(dk_acc[nb][2 * r] * p.scale, dk_acc[nb][2 * r + 1] * p.scale);
      *reinterpret_cast<uint32_t*>(dvrow + nb * 8 + 2 * t) =
          pack_bf16(dv_acc[nb][2 * r], dv_acc[nb][2 * r + 1]);
    }
  }
}

template __global__ void attn_fwd_kernel<64>(const Params p);
template __global__ void attn_fwd_kernel<128>(const Params p);
template __global__ void attn_bwd_kernel<64, false>(const Params p);
template __global__ void attn_bwd_kernel<128, false>(const Params p);
template __global__ void attn_bwd_kernel<64, true>(const Params p);
template __global__ void attn_bwd_kernel<128, true>(const Params p);

// tcgen05 kernels (attention_tc.cu): the default path for head dims 64 / 128.
bool tc_attention_enabled();
void tc_forward(Params p, int d, int64_t max_len, cudaStream_t st, int device);
void tc_backward(Params p, int d, int64_t max_len, cudaStream_t st, int device);
int* tc_status_word(int device);
bool ws_backward_enabled();
void tc_backward_ws(Params p, int64_t max_len, cudaStream_t st, int device, int* status);
bool ws_forward_enabled();
void tc_forward_ws(Params p, int64_t max_len, cudaStream_t st, int device, int* status);

}  // namespace attn

namespace {
bool aligned_rows(const at::Tensor& t) {
  return t.stride(1) == 1 && t.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0;
}

void fill_common(attn::Params& p, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                 const at::Tensor& cu_seqlens, int64_t heads, int64_t kv_heads, double scale,
                 bool causal, int64_t window) {
  check_bf16(q, "q");
  check_bf16(k, "k");
  check_bf16(v, "v");
  RX_CHECK(cu_seqlens.scalar_type() == at::kInt && cu_seqlens.is_cuda(), "cu_seqlens must be CUDA int32");
  RX_CHECK(q.dim() == 2 && k.dim() == 2 && v.dim() == 2, "q/k/v must be [T, heads*D] views");
  RX_CHECK(q.stride(1) == 1 && k.stride(1) == 1 && v.stride(1) == 1, "unit inner stride required");
  RX_CHECK(heads > 0 && kv_heads > 0 && q.size(1) % heads == 0, "bad head counts");
  const int64_t d = q.size(1) / heads;
  RX_CHECK(d == 64 || d == 128, "head_dim must be 64 or 128");
  RX_CHECK(k.size(1) == kv_heads * d && v.size(1) == kv_heads * d, "k/v widths do not match kv_heads*head_dim");
  RX_CHECK(heads % kv_heads == 0, "heads must be a multiple of kv_heads");
  for (const at::Tensor* t : {&q, &k, &v})
    RX_CHECK(t->stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
             "q/k/v rows must be 16-byte aligned");
  p.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  p.k = reinterpret_cast<const __nv_bfloat16*>(k.data_ptr());
  p.v = reinterpret_cast<const __nv_bfloat16*>(v.data_ptr());
  p.ldq = q.stride(0);
  p.ldk = k.stride(0);
  p.ldv = v.stride(0);
  p.cu_seqlens = cu_seqlens.data_ptr<int>();
  p.batch = static_cast<int>(cu_seqlens.numel() - 1);
  p.heads = static_cast<int>(heads);
  p.heads_per_kv = static_cast<int>(heads / kv_heads);
  p.total_tokens = static_cast<int>(q.size(0));
  p.scale = static_cast<float>(scale);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.causal = causal ? 1 : 0;
  p.window = static_cast<int>(window);
}

void set_rel_bias(attn::Params& p, const c10::optional<at::Tensor>& lut, const c10::optional<at::Tensor>& grad,
                  int64_t heads, int64_t max_len) {
  if (!lut.has_value()) return;
  check_f32(*lut, "rel_lut");
  RX_CHECK(lut->dim() == 2 && lut->size(0) == heads && lut->is_contiguous() && lut->size(1) % 2 == 1,
           "rel_lut must be contiguous fp32 [heads, 2 L - 1]");
  p.lut_len = static_cast<int>((lut->size(1) + 1) / 2);
  RX_CHECK(max_len <= p.lut_len, "rel_lut covers fewer distances than the longest sequence");
  p.rel_lut = lut->data_ptr<float>();
  if (grad.has_value()) {
    check_f32(*grad, "drel");
    RX_CHECK(grad->sizes() == lut->sizes() && grad->is_contiguous(), "drel must match rel_lut");
    p.drel = grad->data_ptr<float>();
  }
}

template <typename Kernel>
void set_smem(Kernel kernel, int bytes) {
  if (bytes > 48 * 1024)
    RX_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}
}  // namespace

void attention_forward(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o,
                       at::Tensor& lse, const at::Tensor& cu_seqlens, int64_t max_len,
                       int64_t heads, int64_t kv_heads, double scale, bool causal, int64_t window,
                       int64_t drop_seed, int64_t drop_stream, double drop_p,
                       const c10::optional<at::Tensor>& rel_lut) {
  attn::Params p{};
  fill_common(p, q, k, v, cu_seqlens, heads, kv_heads, scale, causal, window);
  RX_CHECK(drop_p >= 0.0 && drop_p < 1.0, "attention dropout must be in [0, 1)");
  RX_CHECK(max_len < (1 << 17) && heads < (1 << 16), "dropout counters need max_len < 2^17, heads < 2^16");
  p.pdrop = make_dropout_site(drop_seed, drop_stream, drop_p);
  set_rel_bias(p, rel_lut, c10::nullopt, heads, max_len);
  check_bf16(o, "o");
  check_f32(lse, "lse");
  RX_CHECK(o.stride(1) == 1 && o.stride(0) % 2 == 0, "bad o layout");
  RX_CHECK(lse.numel() >= heads * q.size(0), "lse too small");
  p.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.ldo = o.stride(0);
  p.lse = lse.data_ptr<float>();
  if (p.batch == 0 || max_len == 0) return;
  c10::cuda::CUDAGuard guard(q.get_device());
  auto st = at::cuda::getCurrentCUDAStream().stream();
  if (attn::tc_attention_enabled() && aligned_rows(o)) {
    const int d = static_cast<int>(q.size(1) / heads);
    if (d == 64 && p.rel_lut == nullptr && attn::ws_forward_enabled())
      attn::tc_forward_ws(p, max_len, st, q.get_device(), attn::tc_status_word(q.get_device()));
    else
      attn::tc_forward(p, d, max_len, st, q.get_device());
    return;
  }
  dim3 grid((max_len + attn::BM - 1) / attn::BM, heads, p.batch);
  if (q.size(1) / heads == 64) {
    attn::attn_fwd_kernel<64><<<grid, attn::kThreads, attn::fwd_smem_bytes<64>(), st>>>(p);
  } else {
    set_smem(attn::attn_fwd_kernel<128>, attn::fwd_smem_bytes<128>());
    attn::attn_fwd_kernel<128><<<grid, attn::kThreads, attn::fwd_smem_bytes<128>(), st>>>(p);
  }
  RX_CUDA_CHECK(cudaGetLastError());
}

void colsum_accumulate(const at::Tensor& x, at::Tensor& out);

// `dbias_qkv` (optional fp32 [heads * D + 2 * kv_heads * D]): the column sums
// of dq | dk | dv are added into it (a fused QKV projection's bias gradient),
// inside the dQ conversion and the warp-specialised backward's dK / dV
// epilogue when that kernel runs, else by column-sum passes over dk and dv.
void attention_backward_bias(const at::Tensor& dO, const at::Tensor& q, const at::Tensor& k,
                             const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse,
                             at::Tensor& dq, at::Tensor& dk, at::Tensor& dv, at::Tensor& dq_acc,
                             at::Tensor& dvec, const at::Tensor& cu_seqlens, int64_t max_len,
                             int64_t heads, int64_t kv_heads, double scale, bool causal,
                             int64_t window, int64_t drop_seed, int64_t drop_stream, double drop_p,
                             const c10::optional<at::Tensor>& rel_lut, const c10::optional<at::Tensor>& drel,
                             const c10::optional<at::Tensor>& dbias_qkv) {
  attn::Params p{};
  fill_common(p, q, k, v, cu_seqlens, heads, kv_heads, scale, causal, window);
  p.pdrop = make_dropout_site(drop_seed, drop_stream, drop_p);
  set_rel_bias(p, rel_lut, drel, heads, max_len);
  const int d = static_cast<int>(q.size(1) / heads);
  check_bf16(dO, "dO");
  check_f32(dq_acc, "dq_acc");
  check_f32(dvec, "dvec");
  RX_CHECK(dq_acc.is_contiguous() && dq_acc.numel() == q.size(0) * heads * d, "bad dq_acc");
  p.dO = reinterpret_cast<const __nv_bfloat16*>(dO.data_ptr());
  p.ld_do = dO.stride(0);
  p.lse = lse.data_ptr<float>();
  p.dvec = dvec.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk.data_ptr());
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv.data_ptr());
  p.ld_dk = dk.stride(0);
  p.ld_dv = dv.stride(0);
  if (dbias_qkv.has_value()) {
    check_f32(*dbias_qkv, "dbias_qkv");
    RX_CHECK(dbias_qkv->is_contiguous() && dbias_qkv->numel() == (heads + 2 * kv_heads) * d,
             "dbias_qkv must be a contiguous fp32 [(heads + 2 kv_heads) * head_dim]");
    p.dbias_qkv = dbias_qkv->data_ptr<float>();
  }
  const int total = p.total_tokens;
  if (p.batch == 0 || max_len == 0 || total == 0) return;
  c10::cuda::CUDAGuard guard(q.get_device());
  auto st = at::cuda::getCurrentCUDAStream().stream();
  {
    RX_CHECK(aligned_rows(o) && aligned_rows(dO), "attention backward: O and dO rows must be 16-byte aligned");
    const int64_t threads_needed = static_cast<int64_t>(total) * heads * (d / 8);
    const int threads = 256;
    const int64_t blocks = (threads_needed + threads - 1) / threads;
    auto* op = reinterpret_cast<const __nv_bfloat16*>(o.data_ptr());
    if (d == 64)
      attn::attn_bwd_prep_kernel<64><<<blocks, threads, 0, st>>>(op, o.stride(0), p.dO, p.ld_do, dvec.data_ptr<float>(),
                                                                 p.dq_acc, total, static_cast<int>(heads));
    else
      attn::attn_bwd_prep_kernel<128><<<blocks, threads, 0, st>>>(op, o.stride(0), p.dO, p.ld_do,
                                                                  dvec.data_ptr<float>(), p.dq_acc, total,
                                                                  static_cast<int>(heads));
    RX_CUDA_CHECK(cudaGetLastError());
  }
  dim3 grid((max_len + attn::BN - 1) / attn::BN, kv_heads, p.batch);
  const bool gqa = kv_heads != heads;
  bool bias_kv_done = false;  // dK / dV column sums taken by the kernel's epilogue
  if (attn::tc_attention_enabled() && aligned_rows(dO) &&
      aligned_rows(dk) && aligned_rows(dv)) {
    if (d == 64 && p.rel_lut == nullptr && attn::ws_backward_enabled()) {
      attn::tc_backward_ws(p, max_len, st, q.get_device(), attn::tc_status_word(q.get_device()));
      bias_kv_done = true;
    } else {
      attn::tc_backward(p, d, max_len, st, q.get_device());
    }
  } else if (d == 64) {
    if (gqa) attn::attn_bwd_kernel<64, true><<<grid, attn::kThreads, attn::bwd_smem_bytes<64>(), st>>>(p);
    else attn::attn_bwd_kernel<64, false><<<grid, attn::kThreads, attn::bwd_smem_bytes<64>(), st>>>(p);
  } else if (gqa) {
    set_smem(attn::attn_bwd_kernel<128, true>, attn::bwd_smem_bytes<128>());
    attn::attn_bwd_kernel<128, true><<<grid, attn::kThreads, attn::bwd_smem_bytes<128>(), st>>>(p);
  } else {
    set_smem(attn::attn_bwd_kernel<128, false>, attn::bwd_smem_bytes<128>());
    attn::attn_bwd_kernel<128, false><<<grid, attn::kThreads, attn::bwd_smem_bytes<128>(), st>>>(p);
  }
  RX_CUDA_CHECK(cudaGetLastError());
  {
    const int width = static_cast<int>(heads * d);
    RX_CHECK(aligned_rows(dq), "attention backward: dq rows must be 16-byte aligned");
    const int chunks = width / 4;
    RX_CHECK(chunks <= 1024, "attention backward: dq rows wider than 4096 columns");
    const int groups = std::max(1, 1024 / chunks);
    const int threads = groups * chunks;
    const int sms = num_sms(q.get_device());
    const int slice = std::max(8 * groups, (total + sms - 1) / sms);
    const int grid = (total + slice - 1) / slice;
    const size_t smem = groups > 1 ? static_cast<size_t>(groups) * width * sizeof(float) : 0;
    auto kern = attn::attn_dq_convert_colsum_kernel;
    if (smem > 48 * 1024)
      RX_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    kern<<<grid, threads, smem, st>>>(p.dq_acc, reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()), dq.stride(0), total,
                                      width, slice, p.dbias_qkv);
    RX_CUDA_CHECK(cudaGetLastError());
  }
  if (p.dbias_qkv != nullptr && !bias_kv_done) {
    const int64_t qd = heads * d, kd = kv_heads * d;
    at::Tensor bk = dbias_qkv->narrow(0, qd, kd), bv = dbias_qkv->narrow(0, qd + kd, kd);
    colsum_accumulate(dk, bk);
    colsum_accumulate(dv, bv);
  }
}

void attention_backward(const at::Tensor& dO, const at::Tensor& q, const at::Tensor& k,
                        const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse,
                        at::Tensor& dq, at::Tensor& dk, at::Tensor& dv, at::Tensor& dq_acc,
                        at::Tensor& dvec, const at::Tensor& cu_seqlens, int64_t max_len,
                        int64_t heads, int64_t kv_heads, double scale, bool causal,
                        int64_t window, int64_t drop_seed, int64_t drop_stream, double drop_p,
                        const c10::optional<at::Tensor>& rel_lut, const c10::optional<at::Tensor>& drel) {
  attention_backward_bias(dO, q, k, v, o, lse, dq, dk, dv, dq_acc, dvec, cu_seqlens, max_len, heads, kv_heads, scale,
                          causal, window, drop_seed, drop_stream, drop_p, rel_lut, drel, c10::nullopt);
}

}  // namespace rx
