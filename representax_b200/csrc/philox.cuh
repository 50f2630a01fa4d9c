// Counter-based random numbers for dropout masks that can be recomputed.
//
// Philox4x32 (Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC 2011) with 7 rounds of two 32x32->64-bit multiplies
// and the paper's Weyl key schedule; the paper reports that 7 rounds already
// pass TestU01 BigCrush (10 is its conservative default), and a dropout mask
// needs no more. A dropout site draws
// one 128-bit block per counter (c0, c1, c2, c3) under its 64-bit seed, so the
// forward kernel and any backward kernel regenerate the same mask from the
// element coordinates alone: nothing is stored.
//
// Keep decisions are 8-bit: a block's 16 bytes decide 16 elements; an
// element is kept when its byte is >= t8 = round(p * 256) (at least 1, at most
// 255) and kept values are scaled by 256 / (256 - t8), which keeps the
// expectation exact for the quantised probability t8 / 256. Hidden
// (activation) dropout maps element (row, col) to byte col & 15 of block
// (row, col >> 4); attention-probability dropout has its own mapping
// (attention_tc.cuh).
#pragma once
#include <stdint.h>

namespace rx {

struct Philox4 {
  uint32_t x, y, z, w;
};

__host__ __device__ __forceinline__ uint32_t mulhilo(uint32_t a, uint32_t b, uint32_t& hi) {
  const uint64_t p = static_cast<uint64_t>(a) * b;
  hi = static_cast<uint32_t>(p >> 32);
  return static_cast<uint32_t>(p);
}

template <int ROUNDS>
__host__ __device__ __forceinline__ Philox4 philox4x32(Philox4 c, uint32_t k0, uint32_t k1) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  constexpr uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < ROUNDS; ++r) {
    uint32_t hi0, hi1;
    const uint32_t lo0 = mulhilo(M0, c.x, hi0);
    const uint32_t lo1 = mulhilo(M1, c.z, hi1);
    c = Philox4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += W0;
    k1 += W1;
  }
  return c;
}

// Parameters of one dropout site.
struct DropoutSite {
  uint64_t seed;
  uint32_t stream;     // distinguishes the sites that share a seed
  uint32_t threshold;  // 0 = dropout off
  float scale;         // 1 / (1 - p)
};

inline DropoutSite make_dropout_site(int64_t seed, int64_t stream, double p) {
  DropoutSite s{};
  if (p <= 0.0) return s;
  s.seed = static_cast<uint64_t>(seed);
  s.stream = static_cast<uint32_t>(stream);
  const double t = p * 4294967296.0;
  s.threshold = t >= 4294967295.0 ? 0xFFFFFFFFu : (t < 1.0 ? 1u : static_cast<uint32_t>(t));
  s.scale = static_cast<float>(1.0 / (1.0 - p));
  return s;
}

__device__ __forceinline__ uint32_t word_of(const Philox4& r, int i) {
  return i == 0 ? r.x : (i == 1 ? r.y : (i == 2 ? r.z : r.w));
}

// Four words for the 128-bit block addressed by (a, b) at this site.
__device__ __forceinline__ Philox4 dropout_block(const DropoutSite& s, uint32_t a, uint32_t b) {
  return philox4x32<7>(Philox4{a, b, s.stream, 0u}, static_cast<uint32_t>(s.seed),
                       static_cast<uint32_t>(s.seed >> 32));
}

// 8-bit keep threshold and scale of a site (t8 = 0: dropout off).
struct Keep8 {
  uint32_t t8;
  float scale;
};

__host__ __device__ __forceinline__ Keep8 keep8_of(const DropoutSite& s) {
  Keep8 k{0u, 1.f};
  if (s.threshold == 0u) return k;
  k.t8 = (s.threshold + (1u << 23)) >> 24;
  if (k.t8 > 255u) k.t8 = 255u;
  if (k.t8 == 0u) k.t8 = 1u;  // a requested dropout never rounds to none
  k.scale = 256.f / static_cast<float>(256u - k.t8);
  return k;
}

// Hidden-dropout keep bits of the 16 columns 16 col16 .. 16 col16 + 15 of
// `row`: bit j set = column 16 col16 + j kept.
__device__ __forceinline__ uint32_t keep16(const DropoutSite& s, uint32_t t8, uint32_t row, uint32_t col16) {
  const Philox4 r = dropout_block(s, row, col16);
  uint32_t m = 0u;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t word = word_of(r, w);
#pragma unroll
    for (int b = 0; b < 4; ++b) m |= static_cast<uint32_t>(((word >> (8 * b)) & 0xffu) >= t8) << (4 * w + b);
  }
  return m;
}

}  // namespace rx
