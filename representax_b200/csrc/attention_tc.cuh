// Shared pieces of the tcgen05 attention kernels (attention_tc.cu and the
// warp-specialised backward in attention_bwd_ws.cu): tile constants, shared-
// memory layouts of the attention_tc.cu kernels, mask / packing / exp2
// helpers, and the 8-bit Philox dropout keep-bit generators both passes use.
#pragma once

#include "attention_kernels.cuh"
#include "common.h"
#include "sm100.cuh"

namespace rx {
namespace attn {
namespace tc {

constexpr int kThreads = 128;
constexpr int FQ = 128;   // forward: queries per CTA (one per TMEM lane)
// forward: keys per block, FK_FOR<D>: 64 for head dim 64 (TMEM S + O = 128
// columns, 48 KB of shared memory, 64 score registers per thread: four CTAs
// per SM), 128 for head dim 128
template <int D>
constexpr int FK_FOR = D == 64 ? 64 : 128;
constexpr int BKT = 128;  // backward: keys per CTA
constexpr int BQB = 64;   // backward: queries per block
constexpr uint32_t kSub128 = 128 * 128;  // [128 rows][64 bf16] swizzled sub-tile
constexpr uint32_t kSub64 = 64 * 128;    // [64 rows][64 bf16]
constexpr float kLog2e = 1.4426950408889634f;

// Barrier slots (uint64) after the tiles.
enum Bar : int { kBarQ = 0, kBarK, kBarV, kBarS, kBarO, kBarDrain, kBarQ1, kNumBars };

template <int D>
struct FwdLayout {
  static constexpr int DS = D / 64;
  static constexpr int FK = FK_FOR<D>;
  static constexpr uint32_t KSUB = FK * 128;  // [FK keys][64 bf16] swizzled sub-tile
  static constexpr uint32_t Q = 0;
  static constexpr uint32_t K = Q + DS * kSub128;
  static constexpr uint32_t V = K + DS * KSUB;
  static constexpr uint32_t P = V + DS * KSUB;  // [128 q][FK keys] as FK / 64 sub-tiles
  static constexpr uint32_t BARS = P + (FK / 64) * kSub128;
  static constexpr uint32_t BYTES = BARS + kNumBars * 8 + 16 + 1024;  // + TMEM slot + alignment slack
  static constexpr uint32_t TMEM_COLS = FK + D <= 128 ? 128 : 256;  // S: [0, FK), O: [FK, FK + D)
  static constexpr int CTAS_PER_SM = D == 64 ? 4 : 1;
};

template <int D>
struct BwdLayout {
  static constexpr int DS = D / 64;
  static constexpr uint32_t K = 0;
  static constexpr uint32_t V = K + DS * kSub128;
  // Q and dO of query block `it` live in buffer it & 1 (loaded one block ahead)
  static constexpr uint32_t Q = V + DS * kSub128;
  static constexpr uint32_t DO = Q + DS * kSub64;
  static constexpr uint32_t QD_STRIDE = 2 * DS * kSub64;  // buffer 1 = buffer 0 + QD_STRIDE
  static constexpr uint32_t DST = Q + 2 * QD_STRIDE;  // dS^T [128 keys][64 q]
  static constexpr uint32_t PT = DST + kSub128;      // P^T  [128 keys][64 q]; must follow DST
  static constexpr uint32_t LSE = PT + kSub128;      // 64 floats
  static constexpr uint32_t DVEC = LSE + 256;        // 64 floats
  static constexpr uint32_t DIAG = DVEC + 256;       // 192 floats: relative-bias gradient per diagonal
  static constexpr uint32_t BARS = DIAG + 768;
  static constexpr uint32_t BYTES = BARS + kNumBars * 8 + 16 + 1024;
  // S^T [0, 64), dP^T [64, 128), dV [128, 128 + D), dK [128 + D, 128 + 2D);
  // dQ reuses [0, D) once S^T and dP^T have been read.
  static constexpr uint32_t TMEM_COLS = D == 64 ? 256 : 512;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

// Is key j visible from query i (both sequence-relative; j, i < len checked by the caller)?
__device__ __forceinline__ bool mask_ok(const Params& p, int i, int j) {
  if (p.causal && j > i) return false;
  if (p.window >= 0 && (j - i > p.window || i - j > p.window)) return false;
  return true;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// 2^x with the SFU instruction (relative error ~2^-22, far below bf16's
// resolution); 2^-inf = 0.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Row `row` of a K-major [rows][64] bf16 sub-tile with the 128-byte swizzle:
// 16-byte chunk c of the row lives at chunk (c ^ (row & 7)).
__device__ __forceinline__ void store_chunk_sw128(uint8_t* sub, int row, int chunk, uint4 w) {
  *reinterpret_cast<uint4*>(sub + row * 128 + ((chunk ^ (row & 7)) << 4)) = w;
}

// Wait for an outstanding TMA phase (bounded), used when unwinding.
__device__ __forceinline__ void drain_phase(uint64_t* bar, int issued, int waited, const Params& p) {
  if (issued > waited && !mbar_wait(bar, static_cast<uint32_t>(waited & 1), p.timeout_ns))
    report_status(p.status, kStatusTimeoutDrain);
}

// Attention-probability dropout with 8-bit keep decisions (sixteen per
// Philox block, as FlashAttention does): element (query i, key j) of query
// head h in a sequence starting at token `start` keeps its probability when
// byte (j & 3) of word (i & 1) * 2 + ((j >> 2) & 1) of Philox block
// (start + (i & ~1), h << 16 | j >> 3) is >= t8 = round(p * 256); kept values
// are scaled by 256 / (256 - t8), which keeps the expectation exact for the
// quantised probability t8 / 256. Both passes draw the mask from these
// coordinates, so nothing is stored between them. Keep bits live in 64-bit
// registers (bit c = column c), never in an indexed array.
struct Drop8 {
  uint32_t t8;  // 0: off
  float scale;
};

__device__ __forceinline__ Drop8 drop8(const DropoutSite& site) {
  Drop8 d{0u, 1.f};
  if (site.threshold == 0u) return d;
  d.t8 = min((site.threshold + (1u << 23)) >> 24, 255u);
  if (d.t8 == 0u) d.t8 = 1u;  // a requested dropout never rounds to none
  d.scale = 256.f / static_cast<float>(256u - d.t8);
  return d;
}

// Keep decisions of the four bytes of a word, as a nibble (bit b = byte b).
__device__ __forceinline__ uint32_t keep_nibble(uint32_t w, uint32_t t8) {
  return static_cast<uint32_t>((w & 0xffu) >= t8) | (static_cast<uint32_t>(((w >> 8) & 0xffu) >= t8) << 1) |
         (static_cast<uint32_t>(((w >> 16) & 0xffu) >= t8) << 2) | (static_cast<uint32_t>((w >> 24) >= t8) << 3);
}

// OR `n` bits of `bits` into the 128-bit (lo, hi) at column c (c may be
// negative: columns below 0 and above 127 are dropped).
__device__ __forceinline__ void put_bits(uint64_t& lo, uint64_t& hi, uint32_t bits, int n, int c) {
  if (c < 0) {
    if (-c >= n) return;
    bits >>= -c;
    c = 0;
  }
  const uint64_t v = static_cast<uint64_t>(bits);
  if (c < 64) {
    lo |= v << c;
    if (c + n > 64) hi |= v >> (64 - c);
  } else if (c < 128) {
    hi |= v << (c - 64);
  }
}

// Forward (lane = query i; lanes i and i ^ 1 share blocks): keys
// [k0, k0 + nkeys), bit c of (lo, hi) = key k0 + c (c < 128).
__device__ __forceinline__ void fwd_keep_bits(const DropoutSite& site, uint32_t t8, int start, int i, int h, int k0,
                                              int nkeys, int lane, uint64_t& lo, uint64_t& hi) {
  lo = hi = 0ull;
  const bool odd = (lane & 1) != 0;
  const uint32_t a = static_cast<uint32_t>(start + (i & ~1));
  const uint32_t hb = static_cast<uint32_t>(h) << 16;
  const int b0 = k0 >> 3;
  const int nb = ((k0 + nkeys - 1) >> 3) - b0 + 1;  // blocks covering the keys (<= 17)
#pragma unroll 1
  for (int t = 0; t < nb; t += 2) {
    const Philox4 r = dropout_block(site, a, hb | static_cast<uint32_t>(b0 + t + (odd ? 1 : 0)));
    // even lane keeps (x, y) of block t and sends (z, w); odd lane keeps
    // (z, w) of block t + 1 and sends (x, y).
    const uint32_t s0 = __shfl_xor_sync(0xffffffffu, odd ? r.x : r.z, 1);
    const uint32_t s1 = __shfl_xor_sync(0xffffffffu, odd ? r.y : r.w, 1);
    // this lane's row: keys 8 (b0 + t) + 0..7 (block t) and + 8..15 (block t + 1)
    const uint32_t wa0 = odd ? s0 : r.x, wa1 = odd ? s1 : r.y;
    const uint32_t wb0 = odd ? r.z : s0, wb1 = odd ? r.w : s1;
    const uint32_t bits = keep_nibble(wa0, t8) | (keep_nibble(wa1, t8) << 4) | (keep_nibble(wb0, t8) << 8) |
                          (keep_nibble(wb1, t8) << 12);
    put_bits(lo, hi, bits, 16, 8 * (b0 + t) - k0);
  }
}

// Backward (lane = key j; the eight lanes of keys 8k .. 8k + 7 share blocks,
// each generating every eighth query pair and broadcasting its 16 decisions):
// queries [q0, q0 + nq), bit c = query q0 + c (c < 64).
__device__ __forceinline__ uint64_t bwd_keep_bits(const DropoutSite& site, uint32_t t8, int start, int j, int h,
                                                  int q0, int nq, int lane) {
  uint64_t keep = 0ull, unused = 0ull;
  const int r = lane & 7, src0 = lane & ~7, koff = j & 7;
  const uint32_t bcol = (static_cast<uint32_t>(h) << 16) | static_cast<uint32_t>(j >> 3);
  const int a0 = q0 >> 1;
  const int npairs = ((q0 + nq - 1) >> 1) - a0 + 1;  // <= 33
#pragma unroll 1
  for (int t0 = 0; t0 < npairs; t0 += 8) {
    const Philox4 blk = dropout_block(site, static_cast<uint32_t>(start + 2 * (a0 + t0 + r)), bcol);
    // bit (8 * (query & 1) + key offset) of the pair's 16 decisions
    const uint32_t dec = keep_nibble(blk.x, t8) | (keep_nibble(blk.y, t8) << 4) | (keep_nibble(blk.z, t8) << 8) |
                         (keep_nibble(blk.w, t8) << 12);
    uint32_t g = 0u;  // 16 queries: bit 2 s = even query of pair s, bit 2 s + 1 = odd
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const uint32_t d = __shfl_sync(0xffffffffu, dec, src0 + s);
      g |= ((d >> koff) & 1u) << (2 * s);
      g |= ((d >> (8 + koff)) & 1u) << (2 * s + 1);
    }
    put_bits(keep, unused, g, 16, 2 * (a0 + t0) - q0);
  }
  return keep;
}

}  // namespace tc
}  // namespace attn
}  // namespace rx
