// Similarity GEMMs of the MNR objective on the tcgen05 tensor cores, with the
// cross-rank all-gather of candidate embeddings fused into the scoring kernel
// and the reduce-scatter's send fused into the candidate-gradient epilogue.
//
// Precision: the objective works on fp32 unit vectors (the reference keeps
// representations in fp32, src/representax/core/model.py:155). Every fp32
// operand x is split into two bf16 numbers, hi = bf16(x) and lo = bf16(x - hi),
// and a product is accumulated in fp32 as
//     a.b ~= a_hi.b_hi + a_hi.b_lo + a_lo.b_hi
// (three kind::f16 MMAs per K step; the dropped a_lo.b_lo term is below
// 2^-16 relative), so scores and gradients match an fp32 GEMM to ~1e-5.
//
// One kernel, persistent (one CTA per SM), warp-specialised:
//   warp 0      TMA producer: per stage the four 128 x 64 bf16 tiles A_hi,
//               A_lo, B_hi, B_lo (K-major, or MN-major as two 64 x 64 boxes),
//               128-byte swizzle, 3-stage ring; all maps point at this GPU's
//               memory (no peer memory behind any tensor map, no multicast).
//   warp 1      owns TMEM (two 128-column fp32 accumulators) and issues the
//               MMAs (M = 128, N = 128, K = 16, three per K step).
//   warps 2-5   epilogue: tcgen05.ld, scale, fp32 stores either into a local
//               matrix (optionally accumulating) or, row block by row block,
//               into the owning rank's slot buffer by peer stores; or, for
//               hardest-negative mining, no stores at all: each row's best
//               (score, column) over the tile, merged across tiles by one
//               64-bit atomicMax per row (scores never reach memory).
//   warps 6-9   stagers (scoring launch only): convert the local rows and
//               every rank's candidate rows (plain vector loads from the
//               owner's memory over NVLink) into the split bf16 operand
//               buffers of this GPU, 16 rows per chunk, and count finished
//               chunks per owner with a release add. The producer waits
//               (acquire, bounded) for an owner's count before its first TMA
//               load of that owner's rows, so the transfer of later owners
//               overlaps the MMAs on earlier ones. Tiles are visited starting
//               at this rank's own candidate block.
//
// Every wait is bounded by %globaltimer and reports to the status word.
//
// Reference parity: the similarity products and their transposes in
// src/representax/tasks/retrieval/mnr.py:123-230 with the candidate
// all-gather / cotangent reduce-scatter of :140-148.
#include <vector>

#include "common.h"
#include "sm100.cuh"

namespace rx {
namespace mnrtc {

constexpr int BM = 128, BN = 128, BK = 64, STAGES = 3;
constexpr int kTile = BM * BK * 2;  // 16 KB: 128 rows x 64 bf16
constexpr int kStage = 4 * kTile;   // A_hi, A_lo, B_hi, B_lo
constexpr int kEpiWarps = 4, kStageWarps = 4;
constexpr int kThreads = 32 * (2 + kEpiWarps + kStageWarps);
constexpr int kChunkRows = 16;
constexpr size_t kSmem = 1024 + STAGES * kStage + 256;
constexpr int kMaxRanks = 16;  // peer pointers travel in the kernel parameters

struct Params {
  int M, N, K;
  int m_tiles, n_tiles, num_units, n_rot;
  int splits, kb_per_split;  // split-K: unit = tile x split; splits > 1 adds with fp32 atomics
  float* C;
  int64_t ldc;
  bool accumulate;
  bool routed;  // rows m -> (float*)route[m / route_seg] + route_off + (m % route_seg) * ldc
  int64_t route[kMaxRanks];
  int route_seg;
  int64_t route_off;
  float alpha;
  // staging (scoring launch)
  int64_t src[kMaxRanks];  // fp32 [src_rows, K] candidate rows of each rank (this rank's included)
  int src_rows, world, rank;
  const float* a_src;  // fp32 [a_rows, K] local rows
  int a_rows;
  __nv_bfloat16 *a_hi, *a_lo, *b_hi, *b_lo;
  int* ready;  // [world + 1] finished chunks per owner (index world: the local rows)
  int* status;
  uint64_t timeout_ns;
  // mining: best[m] = max over allowed columns n of key(score) << 32 | ~n
  unsigned long long* best;
  const uint8_t* valid;  // [N] allowed candidates (nullptr: all)
  int64_t exclude_off;   // column m + exclude_off is never a candidate
};

// Order-preserving map of an fp32 score onto uint32 (larger score, larger key).
__device__ __forceinline__ uint32_t score_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Order generic-proxy global writes with later async-proxy (TMA) reads.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void stager_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kStageWarps) : "memory");
}

__device__ __forceinline__ uint2 split4(const float4 v, uint2& lo) {
  const __nv_bfloat16 h0 = __float2bfloat16_rn(v.x), h1 = __float2bfloat16_rn(v.y), h2 = __float2bfloat16_rn(v.z),
                      h3 = __float2bfloat16_rn(v.w);
  const __nv_bfloat162 l01 = __floats2bfloat162_rn(v.x - __bfloat162float(h0), v.y - __bfloat162float(h1));
  const __nv_bfloat162 l23 = __floats2bfloat162_rn(v.z - __bfloat162float(h2), v.w - __bfloat162float(h3));
  const __nv_bfloat162 h01 = __halves2bfloat162(h0, h1), h23 = __halves2bfloat162(h2, h3);
  lo = make_uint2(*reinterpret_cast<const uint32_t*>(&l01), *reinterpret_cast<const uint32_t*>(&l23));
  return make_uint2(*reinterpret_cast<const uint32_t*>(&h01), *reinterpret_cast<const uint32_t*>(&h23));
}

// Convert rows [r0, r1) of an fp32 [*, K] matrix into split bf16 rows. Warp
// `sw` of the stager group takes rows r0 + sw, r0 + sw + kStageWarps, ...; its
// (row, 16-byte column) items are walked in batches of 8 per lane with all 8
// loads (peer or local) issued before the first conversion, so each CTA keeps
// ~16 KB of NVLink reads in flight.
constexpr int kStageDepth = 8;
__device__ __forceinline__ void stage_rows(const float* src, __nv_bfloat16* hi, __nv_bfloat16* lo, int r0, int r1,
                                           int K, int sw, int lane) {
  const int q4 = K >> 2;
  const int nrows = (r1 - r0 - sw + kStageWarps - 1) / kStageWarps;
  if (nrows <= 0) return;
  const int items = nrows * q4;
  const float4* s4 = reinterpret_cast<const float4*>(src);
  uint2* h2 = reinterpret_cast<uint2*>(hi);
  uint2* l2 = reinterpret_cast<uint2*>(lo);
  for (int base = 0; base < items; base += 32 * kStageDepth) {
    float4 v[kStageDepth];
    int64_t at[kStageDepth];
#pragma unroll
    for (int u = 0; u < kStageDepth; ++u) {
      const int f = base + u * 32 + lane;
      at[u] = -1;
      if (f < items) {
        const int row = r0 + sw + (f / q4) * kStageWarps;
        at[u] = static_cast<int64_t>(row) * q4 + (f % q4);
        v[u] = s4[at[u]];
      }
    }
#pragma unroll
    for (int u = 0; u < kStageDepth; ++u) {
      if (at[u] >= 0) {
        uint2 l;
        h2[at[u]] = split4(v[u], l);
        l2[at[u]] = l;
      }
    }
  }
}

__device__ __forceinline__ bool wait_count(const int* p, int target, uint64_t timeout_ns) {
  if (ld_acquire_gpu(p) >= target) return true;
  const uint64_t start = globaltimer_ns();
  while (ld_acquire_gpu(p) < target) {
    if (globaltimer_ns() - start > timeout_ns) return false;
    __nanosleep(128);
  }
  return true;
}

__device__ __forceinline__ void decode(const Params& p, int u, int& m0, int& n0, int& kb0, int& kb1) {
  const int tile = u % (p.m_tiles * p.n_tiles), split = u / (p.m_tiles * p.n_tiles);
  const int nt = (tile / p.m_tiles + p.n_rot) % p.n_tiles;
  m0 = (tile % p.m_tiles) * BM;
  n0 = nt * BN;
  kb0 = split * p.kb_per_split;
  kb1 = min((p.K + BK - 1) / BK, kb0 + p.kb_per_split);
}

template <bool A_MN, bool B_MN, bool STAGE>
__global__ void __launch_bounds__(kThreads, 1)
    mnr_gemm_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
                    const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl,
                    const Params p) {
  static_assert(!STAGE || (!A_MN && !B_MN), "staged operands are K-major");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(base + STAGES * kStage);
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
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int chunks_a = STAGE ? (p.a_rows + kChunkRows - 1) / kChunkRows : 0;
  const int chunks_b = STAGE ? (p.src_rows + kChunkRows - 1) / kChunkRows : 0;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0, issued_parity = 0;
      uint32_t ready_mask = 0;  // owners (bit world: local rows) known to be staged
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
        int m0, n0, kb0, kb1;
        decode(p, u, m0, n0, kb0, kb1);
        if constexpr (STAGE) {
          const int o_lo = n0 / p.src_rows, o_hi = (min(n0 + BN, p.N) - 1) / p.src_rows;
          bool waited = false;
          if (!((ready_mask >> p.world) & 1u)) {
            ok = wait_count(p.ready + p.world, chunks_a, p.timeout_ns);
            ready_mask |= 1u << p.world;
            waited = true;
          }
          for (int o = o_lo; ok && o <= o_hi; ++o) {
            if ((ready_mask >> o) & 1u) continue;
            ok = wait_count(p.ready + o, chunks_b, p.timeout_ns);
            ready_mask |= 1u << o;
            waited = true;
          }
          if (!ok) {
            report_status(p.status, kStatusTimeoutPeer);
            *abort_flag = 1;
            break;
          }
          if (waited) fence_proxy_async_global();
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (*abort_flag) { ok = false; break; }
          if (!mbar_wait(&empty[stage], phase ^ 1, p.timeout_ns)) {
            report_status(p.status, kStatusTimeoutProducer);
            *abort_flag = 1;
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kStage);
          uint8_t* dst = base + stage * kStage;
          const int k0 = kb * BK;
          if constexpr (A_MN) {
            tma_load_2d(dst, &tmAh, &full[stage], m0, k0);
            tma_load_2d(dst + 8192, &tmAh, &full[stage], m0 + 64, k0);
            tma_load_2d(dst + kTile, &tmAl, &full[stage], m0, k0);
            tma_load_2d(dst + kTile + 8192, &tmAl, &full[stage], m0 + 64, k0);
          } else {
            tma_load_2d(dst, &tmAh, &full[stage], k0, m0);
            tma_load_2d(dst + kTile, &tmAl, &full[stage], k0, m0);
          }
          if constexpr (B_MN) {
            tma_load_2d(dst + 2 * kTile, &tmBh, &full[stage], n0, k0);
            tma_load_2d(dst + 2 * kTile + 8192, &tmBh, &full[stage], n0 + 64, k0);
            tma_load_2d(dst + 3 * kTile, &tmBl, &full[stage], n0, k0);
            tma_load_2d(dst + 3 * kTile + 8192, &tmBl, &full[stage], n0 + 64, k0);
          } else {
            tma_load_2d(dst + 2 * kTile, &tmBh, &full[stage], k0, n0);
            tma_load_2d(dst + 3 * kTile, &tmBl, &full[stage], k0, n0);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s)
        if (((issued_mask >> s) & 1u) && !mbar_wait(&full[s], (issued_parity >> s) & 1u, p.timeout_ns))
          report_status(p.status, kStatusTimeoutDrain);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN, A_MN, B_MN);
      int stage = 0, local = 0;
      uint32_t phase = 0;
      bool ok = true, issued_any = false;
      for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x, ++local) {
        int m0, n0, kb0, kb1;
        decode(p, u, m0, n0, kb0, kb1);
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
          const uint32_t ah = smem_u32(base + stage * kStage), al = ah + kTile, bh = ah + 2 * kTile,
                         bl = ah + 3 * kTile;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint32_t ao = A_MN ? kk * 2048 : kk * 32, bo = B_MN ? kk * 2048 : kk * 32;
            const uint64_t dah = A_MN ? smem_desc_sw128(ah + ao, 8192, 1024) : smem_desc_sw128(ah + ao, 16, 1024);
            const uint64_t dal = A_MN ? smem_desc_sw128(al + ao, 8192, 1024) : smem_desc_sw128(al + ao, 16, 1024);
            const uint64_t dbh = B_MN ? smem_desc_sw128(bh + bo, 8192, 1024) : smem_desc_sw128(bh + bo, 16, 1024);
            const uint64_t dbl = B_MN ? smem_desc_sw128(bl + bo, 8192, 1024) : smem_desc_sw128(bl + bo, 16, 1024);
            umma_f16_ss(d_tmem, dah, dbh, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
            umma_f16_ss(d_tmem, dah, dbl, IDESC, 1u);
            umma_f16_ss(d_tmem, dal, dbh, IDESC, 1u);
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
  } else if (warp < 2 + kEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    int local = 0;
    for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++local) {
      int m0, n0, kb0, kb1;
      decode(p, u, m0, n0, kb0, kb1);
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
      const int m = m0 + quad * 32 + lane;
      float* row = nullptr;
      if (m < p.M) {
        row = p.routed
                  ? reinterpret_cast<float*>(p.route[m / p.route_seg]) + p.route_off +
                        static_cast<int64_t>(m % p.route_seg) * p.ldc
                  : p.C + static_cast<int64_t>(m) * p.ldc;
      }
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      if (p.best != nullptr) {
        // hardest-candidate mining: ties go to the smaller column (~n is larger)
        unsigned long long best = 0ull;
        const int64_t skip = static_cast<int64_t>(m) + p.exclude_off;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + c * 32, r);
          tmem_ld_wait();
          const int nb = n0 + c * 32;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int n = nb + i;
            if (n >= p.N || n == skip || (p.valid != nullptr && p.valid[n] == 0)) continue;
            const unsigned long long key =
                (static_cast<unsigned long long>(score_key(__uint_as_float(r[i]))) << 32) | (0xffffffffu - n);
            best = key > best ? key : best;
          }
        }
        if (m < p.M && best != 0ull) atomicMax(p.best + m, best);
        tc_fence_before();
        mbar_arrive(&tempty[acc]);
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait();
        const int nb = n0 + c * 32;
        if (row == nullptr || nb >= p.N) continue;
        if (nb + 32 <= p.N) {
          float4* dst = reinterpret_cast<float4*>(row + nb);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            float4 w = make_float4(__uint_as_float(r[4 * q]) * p.alpha, __uint_as_float(r[4 * q + 1]) * p.alpha,
                                   __uint_as_float(r[4 * q + 2]) * p.alpha, __uint_as_float(r[4 * q + 3]) * p.alpha);
            if (p.splits > 1) {
              atomicAdd(dst + q, w);
            } else {
              if (p.accumulate) {
                const float4 o = dst[q];
                w = make_float4(o.x + w.x, o.y + w.y, o.z + w.z, o.w + w.w);
              }
              dst[q] = w;
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (nb + i < p.N) {
              const float v = __uint_as_float(r[i]) * p.alpha;
              if (p.splits > 1)
                atomicAdd(row + nb + i, v);
              else
                row[nb + i] = p.accumulate ? row[nb + i] + v : v;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  } else if constexpr (STAGE) {
    // ------------------------------------------------------------ stagers
    const int sw = warp - 2 - kEpiWarps;
    const int total = chunks_a + p.world * chunks_b;
    for (int c = blockIdx.x; c < total; c += gridDim.x) {
      int owner_slot;
      if (c < chunks_a) {
        const int r0 = c * kChunkRows;
        stage_rows(p.a_src, p.a_hi, p.a_lo, r0, min(p.a_rows, r0 + kChunkRows), p.K, sw, lane);
        owner_slot = p.world;
      } else {
        const int cc = c - chunks_a;
        const int owner = (p.rank + cc / chunks_b) % p.world;
        const int r0 = (cc % chunks_b) * kChunkRows;
        const float* src = reinterpret_cast<const float*>(p.src[owner]);
        const int64_t shift = static_cast<int64_t>(owner) * p.src_rows * p.K;
        stage_rows(src, p.b_hi + shift, p.b_lo + shift, r0, min(p.src_rows, r0 + kChunkRows), p.K, sw, lane);
        owner_slot = owner;
      }
      fence_proxy_async_global();
      __threadfence();
      stager_sync();
      if (sw == 0 && lane == 0) red_release_gpu_add(p.ready + owner_slot, 1);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, 2 * BN);
}

// fp32 -> (hi, lo) bf16 split of a contiguous array (n % 4 == 0).
__global__ void split_kernel(const float4* __restrict__ src, uint2* __restrict__ hi, uint2* __restrict__ lo,
                             int64_t n4) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint2 l;
    hi[i] = split4(src[i], l);
    lo[i] = l;
  }
}

template <bool A_MN, bool B_MN, bool STAGE>
void launch(const CUtensorMap& ah, const CUtensorMap& al, const CUtensorMap& bh, const CUtensorMap& bl,
            const Params& p, int device, cudaStream_t stream) {
  auto kern = mnr_gemm_kernel<A_MN, B_MN, STAGE>;
  static bool configured[64] = {false};
  if (device < 0 || device >= 64 || !configured[device]) {
    RX_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmem)));
    if (device >= 0 && device < 64) configured[device] = true;
  }
  // The scoring launch uses every SM (CTAs without a tile still stage rows).
  const int grid = STAGE ? num_sms(device) : std::max(1, std::min(p.num_units, num_sms(device)));
  // The scoring launch's CTAs wait for chunks staged by other CTAs of the same
  // grid: launch it cooperatively so they are guaranteed to be co-resident.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = STAGE ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  RX_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ah, al, bh, bl, p));
}

}  // namespace mnrtc

namespace {

// K-major operand [rows, K] (box 64 K x 128 rows) or MN-major operand
// [K, mn] (box 64 mn x 64 K).
CUtensorMap operand_map(const at::Tensor& t, bool mn_major) {
  check_bf16(t, "split operand");
  RX_CHECK(t.dim() == 2 && t.stride(1) == 1, "split operands must be 2-D row-major");
  return make_tmap_2d_bf16(t.data_ptr(), t.size(0), t.size(1), t.stride(0), 64, mn_major ? 64 : 128);
}

mnrtc::Params base_params(int64_t M, int64_t N, int64_t K, double alpha, const at::Tensor& status) {
  mnrtc::Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.m_tiles = static_cast<int>((M + mnrtc::BM - 1) / mnrtc::BM);
  p.n_tiles = static_cast<int>((N + mnrtc::BN - 1) / mnrtc::BN);
  p.num_units = p.m_tiles * p.n_tiles;
  p.splits = 1;
  p.kb_per_split = static_cast<int>((K + mnrtc::BK - 1) / mnrtc::BK);
  p.alpha = static_cast<float>(alpha);
  p.status = status_ptr(status);
  p.timeout_ns = kWaitBudgetNs;
  p.route_seg = 1;
  return p;
}

}  // namespace

// Split an fp32 tensor into bf16 hi / lo parts of the same shape.
void mnr_split(const at::Tensor& src, at::Tensor& hi, at::Tensor& lo) {
  check_f32(src, "src");
  check_bf16(hi, "hi");
  check_bf16(lo, "lo");
  RX_CHECK(src.is_contiguous() && hi.is_contiguous() && lo.is_contiguous(), "split tensors must be contiguous");
  RX_CHECK(src.numel() == hi.numel() && src.numel() == lo.numel() && src.numel() % 4 == 0,
           "split sizes must match and be a multiple of 4");
  if (src.numel() == 0) return;
  c10::cuda::CUDAGuard guard(src.get_device());
  const int64_t n4 = src.numel() / 4;
  const int grid = static_cast<int>(std::min<int64_t>((n4 + 255) / 256, 8 * num_sms(src.get_device())));
  mnrtc::split_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      reinterpret_cast<const float4*>(src.data_ptr<float>()), reinterpret_cast<uint2*>(hi.data_ptr()),
      reinterpret_cast<uint2*>(lo.data_ptr()), n4);
  RX_CUDA_CHECK(cudaGetLastError());
}

// Scores = alpha * rows . cands^T with the candidate all-gather fused in.
// rows: local fp32 [M, K]; src_ptrs: device addresses (host integers) of every
// rank's fp32 [src_rows, K] candidate rows (this rank's included); the split
// bf16 copies land in a_hi/a_lo [M, K] and b_hi/b_lo [world * src_rows, K]
// (kept by the caller for the gradient products); ready: int32[world + 1],
// zeroed here on the stream before the launch.
void mnr_tc_scores(const at::Tensor& rows, const std::vector<int64_t>& src_ptrs, int64_t src_rows, int64_t rank,
                   at::Tensor& a_hi, at::Tensor& a_lo, at::Tensor& b_hi, at::Tensor& b_lo, at::Tensor& ready,
                   at::Tensor& scores, double alpha, const at::Tensor& status) {
  check_f32(rows, "rows");
  check_f32(scores, "scores");
  RX_CHECK(rows.dim() == 2 && rows.is_contiguous(), "rows must be contiguous [M, K]");
  const int64_t world = static_cast<int64_t>(src_ptrs.size());
  RX_CHECK(world >= 1 && world <= mnrtc::kMaxRanks && rank >= 0 && rank < world, "bad world / rank");
  for (int64_t r = 0; r < world; ++r) RX_CHECK(src_ptrs[r] != 0 && src_ptrs[r] % 16 == 0, "src pointers must be 16-byte aligned");
  const int64_t M = rows.size(0), K = rows.size(1), N = world * src_rows;
  RX_CHECK(K % 8 == 0, "embedding width must be a multiple of 8 (16-byte rows of the split operands)");
  RX_CHECK(a_hi.size(0) == M && a_hi.size(1) == K && a_lo.sizes() == a_hi.sizes(), "a split buffers are [M, K]");
  RX_CHECK(b_hi.size(0) == N && b_hi.size(1) == K && b_lo.sizes() == b_hi.sizes(), "b split buffers are [N, K]");
  RX_CHECK(scores.size(0) == M && scores.size(1) == N && scores.stride(1) == 1 && scores.stride(0) % 4 == 0,
           "scores must be [M, N] with a 16-byte aligned row stride");
  RX_CHECK(ready.is_cuda() && ready.scalar_type() == at::kInt && ready.numel() >= world + 1, "ready is int32[world+1]");
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(rows.get_device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  RX_CUDA_CHECK(cudaMemsetAsync(ready.data_ptr(), 0, sizeof(int) * (world + 1), stream));
  mnrtc::Params p = base_params(M, N, K, alpha, status);
  p.C = scores.data_ptr<float>();
  p.ldc = scores.stride(0);
  for (int64_t r = 0; r < world; ++r) p.src[r] = src_ptrs[r];
  p.src_rows = static_cast<int>(src_rows);
  p.world = static_cast<int>(world);
  p.rank = static_cast<int>(rank);
  p.a_src = rows.data_ptr<float>();
  p.a_rows = static_cast<int>(M);
  p.a_hi = reinterpret_cast<__nv_bfloat16*>(a_hi.data_ptr());
  p.a_lo = reinterpret_cast<__nv_bfloat16*>(a_lo.data_ptr());
  p.b_hi = reinterpret_cast<__nv_bfloat16*>(b_hi.data_ptr());
  p.b_lo = reinterpret_cast<__nv_bfloat16*>(b_lo.data_ptr());
  p.ready = ready.data_ptr<int>();
  p.n_rot = static_cast<int>((rank * src_rows) / mnrtc::BN);
  mnrtc::launch<false, false, true>(operand_map(a_hi, false), operand_map(a_lo, false), operand_map(b_hi, false),
                                    operand_map(b_lo, false), p, rows.get_device(), stream);
}

// C (+)= alpha * A . B^T on split operands. A is [M, K] (a_mn false) or
// [K, M] (a_mn true); B is [N, K] or [K, N]. The output is `out` [M, N], or,
// with `route_ptrs` (device addresses as host integers), row m goes to
// route_ptrs[m / route_seg] + route_off + (m % route_seg) * ldc (fp32 elements).
void mnr_tc_gemm(const at::Tensor& a_hi, const at::Tensor& a_lo, bool a_mn, const at::Tensor& b_hi,
                 const at::Tensor& b_lo, bool b_mn, int64_t M, int64_t N, int64_t K,
                 const c10::optional<at::Tensor>& out, const std::vector<int64_t>& route_ptrs, int64_t route_seg,
                 int64_t route_off, int64_t ldc, double alpha, bool accumulate, const at::Tensor& status) {
  RX_CHECK(a_lo.sizes() == a_hi.sizes() && b_lo.sizes() == b_hi.sizes(), "hi / lo shapes differ");
  RX_CHECK(a_hi.size(0) == (a_mn ? K : M) && a_hi.size(1) == (a_mn ? M : K), "A has the wrong shape");
  RX_CHECK(b_hi.size(0) == (b_mn ? K : N) && b_hi.size(1) == (b_mn ? N : K), "B has the wrong shape");
  RX_CHECK(out.has_value() != !route_ptrs.empty(), "give exactly one of out / route_ptrs");
  RX_CHECK(ldc % 4 == 0 && ldc >= N, "ldc must cover N and keep rows 16-byte aligned");
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(a_hi.get_device());
  mnrtc::Params p = base_params(M, N, K, alpha, status);
  p.ldc = ldc;
  p.accumulate = accumulate;
  if (out.has_value()) {
    check_f32(*out, "out");
    RX_CHECK(out->size(0) == M && out->stride(0) == ldc && out->stride(1) == 1, "out must be [M, N] with stride ldc");
    p.C = out->data_ptr<float>();
  } else {
    const int64_t n = static_cast<int64_t>(route_ptrs.size());
    RX_CHECK(n <= mnrtc::kMaxRanks && route_seg >= 1 && (M + route_seg - 1) / route_seg <= n, "route_ptrs too short");
    RX_CHECK(route_off % 4 == 0, "route_off must keep rows 16-byte aligned");
    for (int64_t r = 0; r < n; ++r) {
      RX_CHECK(route_ptrs[r] % 16 == 0, "route pointers must be 16-byte aligned");
      p.route[r] = route_ptrs[r];
    }
    p.routed = true;
    p.route_seg = static_cast<int>(route_seg);
    p.route_off = route_off;
  }
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  const int dev = a_hi.get_device();
  if (out.has_value()) {
    // Split K when the tiles alone cannot fill the GPU (e.g. a per-rank dQ:
    // 512 x 768 outputs over K = 4096); the partial sums meet in fp32 atomics.
    const int tiles = p.m_tiles * p.n_tiles, kb = p.kb_per_split;
    int splits = std::min(num_sms(dev) / std::max(tiles, 1), kb / 4);
    if (splits > 1) {
      p.kb_per_split = (kb + splits - 1) / splits;
      splits = (kb + p.kb_per_split - 1) / p.kb_per_split;
    }
    if (splits > 1) {
      if (!accumulate) out->zero_();
      p.splits = splits;
      p.num_units = tiles * splits;
    }
  }
  const CUtensorMap ah = operand_map(a_hi, a_mn), al = operand_map(a_lo, a_mn), bh = operand_map(b_hi, b_mn),
                    bl = operand_map(b_lo, b_mn);
  if (!a_mn && !b_mn) {
    mnrtc::launch<false, false, false>(ah, al, bh, bl, p, dev, stream);
  } else if (!a_mn && b_mn) {
    mnrtc::launch<false, true, false>(ah, al, bh, bl, p, dev, stream);
  } else if (a_mn && b_mn) {
    mnrtc::launch<true, true, false>(ah, al, bh, bl, p, dev, stream);
  } else {
    mnrtc::launch<true, false, false>(ah, al, bh, bl, p, dev, stream);
  }
}

// Hardest candidate per row: best[m] = max over n of key(A[m] . B[n]) << 32 | (2^32 - 1 - n),
// over candidates with valid[n] != 0 (all when `valid` is absent) and
// n != m + exclude_off. A / B are split [M, K] / [N, K] operands; best is
// int64 [M], zeroed here (0 = no candidate). The score matrix is never stored.
void mnr_tc_argmax(const at::Tensor& a_hi, const at::Tensor& a_lo, const at::Tensor& b_hi, const at::Tensor& b_lo,
                   at::Tensor& best, const c10::optional<at::Tensor>& valid, int64_t exclude_off,
                   const at::Tensor& status) {
  RX_CHECK(a_lo.sizes() == a_hi.sizes() && b_lo.sizes() == b_hi.sizes(), "hi / lo shapes differ");
  RX_CHECK(a_hi.dim() == 2 && b_hi.dim() == 2 && a_hi.size(1) == b_hi.size(1), "A [M, K] and B [N, K] must share K");
  const int64_t M = a_hi.size(0), N = b_hi.size(0), K = a_hi.size(1);
  RX_CHECK(N < 0xffffffffll, "too many candidates");
  RX_CHECK(best.is_cuda() && best.scalar_type() == at::kLong && best.is_contiguous() && best.numel() == M,
           "best must be a contiguous int64 [M]");
  c10::cuda::CUDAGuard guard(a_hi.get_device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  if (M == 0) return;
  RX_CUDA_CHECK(cudaMemsetAsync(best.data_ptr(), 0, sizeof(int64_t) * M, stream));
  if (N == 0) return;
  mnrtc::Params p = base_params(M, N, K, 1.0, status);
  p.best = reinterpret_cast<unsigned long long*>(best.data_ptr());
  p.exclude_off = exclude_off;
  if (valid.has_value()) {
    RX_CHECK(valid->is_cuda() && (valid->scalar_type() == at::kBool || valid->scalar_type() == at::kByte) &&
                 valid->is_contiguous() && valid->numel() == N,
             "valid must be a contiguous bool / uint8 [N]");
    p.valid = reinterpret_cast<const uint8_t*>(valid->data_ptr());
  }
  mnrtc::launch<false, false, false>(operand_map(a_hi, false), operand_map(a_lo, false), operand_map(b_hi, false),
                                     operand_map(b_lo, false), p, a_hi.get_device(), stream);
}

}  // namespace rx
