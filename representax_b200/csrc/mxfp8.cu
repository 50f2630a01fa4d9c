// MXFP8 linear layers on tcgen05: 8-bit operands with one power-of-two scale
// (UE8M0) per 32 consecutive values along the contraction dimension, applied
// by the tensor core itself (kind::mxf8f6f4.block_scale).
//
// Quantiser (one pass over a bf16 matrix x [R, C], 32 x 128 tiles in shared
// memory): for every 32-value block b of a row, e = ceil(log2(amax_b / FMAX))
// (FMAX = 448 for E4M3, 57344 for E5M2), scale byte = e + 127 and
// q = sat(x * 2^-e). It writes, as asked, the row-wise data q [R, C] (blocks
// along C: a forward operand) and / or the transposed data q^T [C, R] (blocks
// along R: the operand of a product that contracts over R), each with its
// scales already in the tensor core's order (below), so the GEMM loads scales
// with plain bulk copies.
//
// Scale layout ("atoms"): for an operand with `rows` rows and K values per
// row, scales sit in [ceil(K / 128)][ceil(rows / 128) + 1][512 bytes]; the
// atom of (row tile t, K group g) holds, for row r = 32 q + l of the tile and
// K block j (0..3) of the group, byte 16 l + 4 q + j. That is 32 rows of 16
// bytes: one tcgen05.cp 32x128b.warpx4 puts row l into TMEM lane l (of every
// lane quarter) with the scales of rows l, l + 32, l + 64, l + 96 in four
// consecutive 32-bit columns, one byte per K block. The extra row tile is
// padding that 192-row tiles read past the end.
//
// GEMM D [M, N] = A [M, K] . B [N, K]^T (both K-major 8-bit, E4M3 or E5M2):
// persistent, one CTA per SM, warp-specialised like the bf16 kernels:
//   warp 0    producer: per stage a 128 x 128 A tile and a 192 x 128 B tile
//             by TMA (128-byte swizzle, no multicast) plus the A scale atom
//             (512 B) and two B atoms (1 KB) by untiled bulk copies;
//   warp 1    owns TMEM (two 192-column fp32 accumulators + 12 scale
//             columns); per stage it copies the scales into TMEM
//             (tcgen05.cp, ordered with the MMAs of the same thread) and issues
//             four block-scaled MMAs (K = 32 each, scale byte j = K block j);
//             a 192-row B tile that starts half-way into a scale atom (odd
//             tile) points its scale address two columns further;
//   warps 2-5 epilogue: tcgen05.ld, bf16 output with bias / residual, or fp32
//             store / accumulate (weight gradients).
// Every wait is bounded by %globaltimer and reports to the status word.
//
// A linear layer y = x W^T runs as E4M3 x E4M3 (x, W row-wise); dx = dy W as
// E5M2 x E4M3 (dy row-wise, W transposed); dW += dy^T x as E5M2 x E4M3 (dy and
// x transposed) into the fp32 gradient.
//
// Reference parity: the reference's fp8 recipe is per-tensor scaled
// (src/representax/precision.py:127-221: E4M3 forward, E5M2 gradients, fp32
// accumulation); this is the same recipe with per-block power-of-two scales.
#include <cuda_fp8.h>

#include <algorithm>

#include "common.h"
#include "sm100.cuh"

namespace rx {
namespace mx {

constexpr int BM = 128, BN = 192, BK = 128, STAGES = 5;
constexpr int kTileA = BM * BK;  // 16 KB
constexpr int kTileB = BN * BK;  // 24 KB
constexpr int kTiles = kTileA + kTileB;
constexpr int kSfA = 512, kSfB = 1024;
constexpr int kSf = kSfA + kSfB;
constexpr int kEpiWarps = 4;
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr size_t kSmem = 1024 + STAGES * kTiles + STAGES * kSf + 256;
constexpr int kAccCols = 2 * BN;  // 384
constexpr int kTmemCols = 512;

enum OutMode : int { kOutBf16 = 0, kOutF32 = 1, kOutF32Acc = 2 };

struct Params {
  int M, N, K;
  int m_tiles, n_tiles, k_groups, num_units;
  const uint8_t* sfa;
  const uint8_t* sfb;
  int sfa_rt, sfb_rt;  // row tiles per K group of the scale arrays (padded)
  uint32_t idesc;      // formats and shape; scale ids are or-ed in per K block
  void* C;
  int64_t ldc;
  int out_mode;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;
  int64_t ldr;
  int* status;
  uint64_t timeout_ns;
};

__global__ void __launch_bounds__(kThreads, 1)
    mx_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sf_base = base + STAGES * kTiles;
  uint64_t* full = reinterpret_cast<uint64_t*>(sf_base + STAGES * kSf);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 32 * kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_map(&tmA);
      tma_prefetch_map(&tmB);
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
        const int mt = u % p.m_tiles, nt = u / p.m_tiles;
        const int m0 = mt * BM, n0 = nt * BN;
        for (int kg = 0; kg < p.k_groups; ++kg) {
          if (*abort_flag || !mbar_wait(&empty[stage], phase ^ 1, p.timeout_ns)) {
            report_status(p.status, kStatusTimeoutProducer);
            *abort_flag = 1;
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kTiles + kSf);
          uint8_t* tiles = base + stage * kTiles;
          uint8_t* sf = sf_base + stage * kSf;
          tma_load_2d(tiles, &tmA, &full[stage], kg * BK, m0);
          tma_load_2d(tiles + kTileA, &tmB, &full[stage], kg * BK, n0);
          bulk_load(sf, p.sfa + (static_cast<int64_t>(kg) * p.sfa_rt + mt) * 512, kSfA, &full[stage]);
          bulk_load(sf + kSfA, p.sfb + (static_cast<int64_t>(kg) * p.sfb_rt + n0 / 128) * 512, kSfB, &full[stage]);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // leave no copy in flight into shared memory that is about to be released
      for (int s = 0; s < STAGES; ++s)
        if (((issued_mask >> s) & 1u) && !mbar_wait(&full[s], (issued_parity >> s) & 1u, p.timeout_ns))
          report_status(p.status, kStatusTimeoutDrain);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t sfa_t = tmem_base + kAccCols, sfb_t = tmem_base + kAccCols + 4;
      int stage = 0, local = 0;
      uint32_t phase = 0;
      bool ok = true, issued_any = false;
      for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x, ++local) {
        const int nt = u / p.m_tiles;
        const uint32_t sfb_col = sfb_t + static_cast<uint32_t>(((nt * BN) % 128) / 32);
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (*abort_flag || !mbar_wait(&tempty[acc], acc_phase ^ 1, p.timeout_ns)) {
          report_status(p.status, kStatusTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kg = 0; kg < p.k_groups; ++kg) {
          if (*abort_flag || !mbar_wait(&full[stage], phase, p.timeout_ns)) {
            report_status(p.status, kStatusTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(base + stage * kTiles), b = a + kTileA;
          const uint32_t sf = smem_u32(sf_base + stage * kSf);
          tmem_cp_32x128b_warpx4(sfa_t, smem_desc_plain(sf, 512, 128));
          tmem_cp_32x128b_warpx4(sfb_t, smem_desc_plain(sf + kSfA, 512, 128));
          tmem_cp_32x128b_warpx4(sfb_t + 4, smem_desc_plain(sf + kSfA + 512, 512, 128));
#pragma unroll
          for (int kk = 0; kk < BK / 32; ++kk) {
            const uint32_t id = p.idesc | (static_cast<uint32_t>(kk) << 4) | (static_cast<uint32_t>(kk) << 29);
            umma_mxf8_ss(d_tmem, smem_desc_sw128(a + kk * 32, 16, 1024), smem_desc_sw128(b + kk * 32, 16, 1024), id,
                         sfa_t | (static_cast<uint32_t>(kk) << 30), sfb_col | (static_cast<uint32_t>(kk) << 30),
                         (kg > 0 || kk > 0) ? 1u : 0u);
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
      if (issued_any) {
        umma_commit(drain);
        if (!mbar_wait(drain, 0, p.timeout_ns)) report_status(p.status, kStatusTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    int local = 0;
    for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++local) {
      const int mt = u % p.m_tiles, nt = u / p.m_tiles;
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
      const int m = mt * BM + quad * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait();
        const int nb = nt * BN + c * 32;
        if (m >= p.M || nb >= p.N) continue;
        const int cols = min(32, p.N - nb);
        if (p.out_mode == kOutBf16) {
          __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(m) * p.ldc + nb;
          const __nv_bfloat16* res = p.residual ? p.residual + static_cast<int64_t>(m) * p.ldr + nb : nullptr;
          if (cols == 32) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float v[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(r[8 * q + j]);
              if (p.bias) {
                const uint4 bw = *reinterpret_cast<const uint4*>(p.bias + nb + 8 * q);
                const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&bw);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float2 f = __bfloat1622float2(b2[j]);
                  v[2 * j] += f.x;
                  v[2 * j + 1] += f.y;
                }
              }
              if (res) {
                const uint4 rw = *reinterpret_cast<const uint4*>(res + 8 * q);
                const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rw);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const float2 f = __bfloat1622float2(r2[j]);
                  v[2 * j] += f.x;
                  v[2 * j + 1] += f.y;
                }
              }
              uint4 o;
              __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
              for (int j = 0; j < 4; ++j) o2[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
              *reinterpret_cast<uint4*>(row + 8 * q) = o;
            }
          } else {
            for (int i = 0; i < cols; ++i) {
              float v = __uint_as_float(r[i]);
              if (p.bias) v += __bfloat162float(p.bias[nb + i]);
              if (res) v += __bfloat162float(res[i]);
              row[i] = __float2bfloat16_rn(v);
            }
          }
        } else {
          float* row = reinterpret_cast<float*>(p.C) + static_cast<int64_t>(m) * p.ldc + nb;
          const bool add = p.out_mode == kOutF32Acc;
          if (cols == 32) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float4 w = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                     __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
              float4* dst = reinterpret_cast<float4*>(row) + q;
              if (add) {
                const float4 o = *dst;
                w = make_float4(o.x + w.x, o.y + w.y, o.z + w.z, o.w + w.w);
              }
              *dst = w;
            }
          } else {
            for (int i = 0; i < cols; ++i) row[i] = add ? row[i] + __uint_as_float(r[i]) : __uint_as_float(r[i]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

// ------------------------------------------------------------------ quantiser
// Block exponent e = ceil(log2(v)) of v = amax / FMAX > 0 read from the float
// bits (exponent field, plus one when any mantissa bit is set), clamped so
// that both 2^e and 2^-e are normal floats; v = 0 gives the smallest scale.
__device__ __forceinline__ int block_exponent(float amax, float fmax) {
  const uint32_t b = __float_as_uint(amax / fmax);
  int e = static_cast<int>((b >> 23) & 0xffu) - 127 + ((b & 0x7fffffu) != 0u ? 1 : 0);
  return max(-127, min(126, e));
}
__device__ __forceinline__ float pow2(int e) { return __uint_as_float(static_cast<uint32_t>(127 + e) << 23); }

template <bool E5M2>
__device__ __forceinline__ uint16_t to_fp8x2(float a, float b) {
  return static_cast<uint16_t>(
      __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, E5M2 ? __NV_E5M2 : __NV_E4M3));
}

__device__ __forceinline__ int64_t atom_offset(int row, int kblock, int rt_pad) {
  const int t = row >> 7, r = row & 127;
  return (static_cast<int64_t>(kblock >> 2) * rt_pad + t) * 512 + 16 * (r & 31) + 4 * (r >> 5) + (kblock & 3);
}

// One CTA: rows [r0, r0 + 32) x columns [c0, c0 + 128) of x. 128 threads.
template <bool E5M2>
__global__ void __launch_bounds__(128)
    mx_quantize_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int R, int C, uint8_t* __restrict__ q,
                       int64_t ldq, uint8_t* __restrict__ sf, int sf_rt, uint8_t* __restrict__ qt, int64_t ldqt,
                       uint8_t* __restrict__ sft, int sft_rt) {
  constexpr float FMAX = E5M2 ? 57344.f : 448.f;
  __shared__ __align__(16) __nv_bfloat16 tile[32][128 + 8];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 128;
  const int t = threadIdx.x;
  // the tile as 32 rows x 16 chunks of 16 bytes (zeros outside x)
  for (int i = t; i < 32 * 16; i += 128) {
    const int rr = i >> 4, cc = (i & 15) * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (r0 + rr < R && c0 + cc < C) v = *reinterpret_cast<const uint4*>(x + static_cast<int64_t>(r0 + rr) * ldx + c0 + cc);
    *reinterpret_cast<uint4*>(&tile[rr][cc]) = v;
  }
  __syncthreads();
  if (q != nullptr) {
    // row-wise: thread = (row rr, 32-column block cb)
    const int rr = t >> 2, cb = t & 3;
    const int row = r0 + rr, col = c0 + cb * 32;
    if (row < R && col < C) {
      float v[32];
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        v[j] = __bfloat162float(tile[rr][cb * 32 + j]);
        amax = fmaxf(amax, fabsf(v[j]));
      }
      const int e = block_exponent(amax, FMAX);
      const float inv = pow2(-e);
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        w[j] = static_cast<uint32_t>(to_fp8x2<E5M2>(v[4 * j] * inv, v[4 * j + 1] * inv)) |
               (static_cast<uint32_t>(to_fp8x2<E5M2>(v[4 * j + 2] * inv, v[4 * j + 3] * inv)) << 16);
      uint8_t* dst = q + static_cast<int64_t>(row) * ldq + col;
      *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
      *reinterpret_cast<uint4*>(dst + 16) = make_uint4(w[4], w[5], w[6], w[7]);
      sf[atom_offset(row, col >> 5, sf_rt)] = static_cast<uint8_t>(e + 127);
    }
  }
  if (qt != nullptr) {
    // transposed: thread = column cc; its 32 rows form one block of q^T's row cc
    const int col = c0 + t;
    if (col < C && r0 < R) {
      float v[32];
      float amax = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        v[j] = __bfloat162float(tile[j][t]);  // rows >= R were loaded as zero
        amax = fmaxf(amax, fabsf(v[j]));
      }
      const int e = block_exponent(amax, FMAX);
      const float inv = pow2(-e);
      uint32_t w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        w[j] = static_cast<uint32_t>(to_fp8x2<E5M2>(v[4 * j] * inv, v[4 * j + 1] * inv)) |
               (static_cast<uint32_t>(to_fp8x2<E5M2>(v[4 * j + 2] * inv, v[4 * j + 3] * inv)) << 16);
      uint8_t* dst = qt + static_cast<int64_t>(col) * ldqt + r0;
      *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
      *reinterpret_cast<uint4*>(dst + 16) = make_uint4(w[4], w[5], w[6], w[7]);
      sft[atom_offset(col, r0 >> 5, sft_rt)] = static_cast<uint8_t>(e + 127);
    }
  }
}

}  // namespace mx

// Scale-array geometry of an operand with `rows` rows and K values per row.
static int64_t mx_rt_pad(int64_t rows) { return (rows + 127) / 128 + 1; }
static int64_t mx_groups(int64_t k) { return (k + 127) / 128; }

// x bf16 [R, C] -> q uint8 [R, C] + sf (row-wise, blocks along C) and / or
// qt uint8 [C, ldqt >= R rounded up to 32] + sft (blocks along R). The scale
// arrays must be zero-initialised uint8 of [groups * rt_pad * 512] bytes.
void mx_quantize(const at::Tensor& x, const c10::optional<at::Tensor>& q, const c10::optional<at::Tensor>& sf,
                 const c10::optional<at::Tensor>& qt, const c10::optional<at::Tensor>& sft, bool e5m2) {
  check_bf16(x, "x");
  RX_CHECK(x.dim() == 2 && x.stride(1) == 1 && x.stride(0) % 8 == 0 &&
               reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
           "x must be a 16-byte aligned row-major [R, C]");
  const int64_t R = x.size(0), C = x.size(1);
  RX_CHECK(C % 32 == 0, "MXFP8 needs C % 32 == 0");
  RX_CHECK(q.has_value() == sf.has_value() && qt.has_value() == sft.has_value(), "give data and scales together");
  auto u8 = [](const at::Tensor& t, const char* what) {
    RX_CHECK(t.is_cuda() && t.scalar_type() == at::kByte, what, " must be a CUDA uint8 tensor");
  };
  uint8_t *qp = nullptr, *sp = nullptr, *qtp = nullptr, *stp = nullptr;
  int64_t ldq = 0, ldqt = 0;
  if (q.has_value()) {
    u8(*q, "q");
    u8(*sf, "sf");
    RX_CHECK(q->size(0) == R && q->size(1) == C && q->stride(1) == 1 && q->stride(0) % 16 == 0, "q must be [R, C]");
    RX_CHECK(sf->numel() == mx_groups(C) * mx_rt_pad(R) * 512, "sf has the wrong size");
    qp = q->data_ptr<uint8_t>();
    sp = sf->data_ptr<uint8_t>();
    ldq = q->stride(0);
  }
  if (qt.has_value()) {
    u8(*qt, "qt");
    u8(*sft, "sft");
    RX_CHECK(R % 32 == 0 || qt->stride(0) >= (R + 31) / 32 * 32, "qt rows must hold R rounded up to 32");
    RX_CHECK(qt->size(0) == C && qt->stride(1) == 1 && qt->stride(0) % 16 == 0, "qt must be [C, >= R]");
    RX_CHECK(sft->numel() == mx_groups(R) * mx_rt_pad(C) * 512, "sft has the wrong size");
    qtp = qt->data_ptr<uint8_t>();
    stp = sft->data_ptr<uint8_t>();
    ldqt = qt->stride(0);
  }
  if (R == 0 || C == 0 || (qp == nullptr && qtp == nullptr)) return;
  c10::cuda::CUDAGuard guard(x.get_device());
  const dim3 grid(static_cast<unsigned>((C + 127) / 128), static_cast<unsigned>((R + 31) / 32));
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  if (e5m2)
    mx::mx_quantize_kernel<true><<<grid, 128, 0, stream>>>(xp, x.stride(0), static_cast<int>(R), static_cast<int>(C), qp,
                                                           ldq, sp, static_cast<int>(mx_rt_pad(R)), qtp, ldqt, stp,
                                                           static_cast<int>(mx_rt_pad(C)));
  else
    mx::mx_quantize_kernel<false><<<grid, 128, 0, stream>>>(xp, x.stride(0), static_cast<int>(R), static_cast<int>(C),
                                                            qp, ldq, sp, static_cast<int>(mx_rt_pad(R)), qtp, ldqt, stp,
                                                            static_cast<int>(mx_rt_pad(C)));
  RX_CUDA_CHECK(cudaGetLastError());
}

// out [M, N] (bf16, or fp32 stored / accumulated) = A [M, K] . B [N, K]^T with
// MX scales sfa / sfb in the atom layout. out_mode: 0 bf16 (+ bias [N], +
// residual [M, N]), 1 fp32 store, 2 fp32 accumulate.
void mx_gemm(const at::Tensor& a, const at::Tensor& sfa, int64_t a_fmt, const at::Tensor& b, const at::Tensor& sfb,
             int64_t b_fmt, int64_t K, at::Tensor& out, int64_t out_mode, const c10::optional<at::Tensor>& bias,
             const c10::optional<at::Tensor>& residual, const at::Tensor& status) {
  RX_CHECK(a.is_cuda() && b.is_cuda() && a.scalar_type() == at::kByte && b.scalar_type() == at::kByte,
           "A and B must be CUDA uint8 (fp8 bits)");
  RX_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1, "A / B must be row-major 2-D");
  RX_CHECK(K % 32 == 0 && K <= a.size(1) && K <= b.size(1), "K must be a multiple of 32 within A and B");
  RX_CHECK((a_fmt == 0 || a_fmt == 1) && (b_fmt == 0 || b_fmt == 1), "formats: 0 = E4M3, 1 = E5M2");
  const int64_t M = a.size(0), N = b.size(0);
  RX_CHECK(sfa.numel() == mx_groups(K) * mx_rt_pad(M) * 512 && sfb.numel() == mx_groups(K) * mx_rt_pad(N) * 512,
           "scale arrays have the wrong size");
  RX_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "out must be [M, N]");
  RX_CHECK(out_mode >= 0 && out_mode <= 2, "bad out_mode");
  if (out_mode == mx::kOutBf16) {
    check_bf16(out, "out");
    RX_CHECK(out.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
             "bf16 out rows must be 16-byte aligned");
  } else {
    check_f32(out, "out");
    RX_CHECK(out.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
             "fp32 out rows must be 16-byte aligned");
    RX_CHECK(!bias.has_value() && !residual.has_value(), "fp32 outputs take no bias / residual");
  }
  if (bias.has_value()) {
    check_bf16(*bias, "bias");
    RX_CHECK(bias->numel() == N && bias->is_contiguous() && N % 8 == 0 &&
                 reinterpret_cast<uintptr_t>(bias->data_ptr()) % 16 == 0,
             "bias must be a 16-byte aligned contiguous [N], N % 8 == 0");
  }
  if (residual.has_value()) {
    check_bf16(*residual, "residual");
    RX_CHECK(residual->size(0) == M && residual->size(1) == N && residual->stride(1) == 1 &&
                 residual->stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(residual->data_ptr()) % 16 == 0,
             "residual must be [M, N] with 16-byte aligned rows");
  }
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(a.get_device());
  mx::Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.m_tiles = static_cast<int>((M + mx::BM - 1) / mx::BM);
  p.n_tiles = static_cast<int>((N + mx::BN - 1) / mx::BN);
  p.k_groups = static_cast<int>(mx_groups(K));
  p.num_units = p.m_tiles * p.n_tiles;
  p.sfa = sfa.data_ptr<uint8_t>();
  p.sfb = sfb.data_ptr<uint8_t>();
  p.sfa_rt = static_cast<int>(mx_rt_pad(M));
  p.sfb_rt = static_cast<int>(mx_rt_pad(N));
  p.idesc = idesc_mxf8(mx::BM, mx::BN, static_cast<int>(a_fmt), static_cast<int>(b_fmt), 0, 0);
  p.C = out.data_ptr();
  p.ldc = out.stride(0);
  p.out_mode = static_cast<int>(out_mode);
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  p.residual = residual.has_value() ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  p.ldr = residual.has_value() ? residual->stride(0) : 0;
  p.status = status_ptr(status);
  p.timeout_ns = kWaitBudgetNs;
  RX_CHECK(reinterpret_cast<uintptr_t>(p.sfa) % 16 == 0 && reinterpret_cast<uintptr_t>(p.sfb) % 16 == 0,
           "scale arrays must be 16-byte aligned");
  // K extent = K (columns beyond it are zero-filled by TMA; their scales are zero)
  const CUtensorMap ta = make_tmap_2d_u8(a.data_ptr(), M, K, a.stride(0), mx::BM);
  const CUtensorMap tb = make_tmap_2d_u8(b.data_ptr(), N, K, b.stride(0), mx::BN);
  const int dev = a.get_device();
  static bool configured[64] = {false};
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    RX_CUDA_CHECK(cudaFuncSetAttribute(mx::mx_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(mx::kSmem)));
    if (dev >= 0 && dev < 64) configured[dev] = true;
  }
  const int grid = std::max(1, std::min(p.num_units, num_sms(dev)));
  mx::mx_gemm_kernel<<<grid, mx::kThreads, mx::kSmem, at::cuda::getCurrentCUDAStream().stream()>>>(ta, tb, p);
  RX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace rx
