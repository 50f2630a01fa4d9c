// Warp-specialised, persistent attention forward on tcgen05 (head dim 64).
//
// Work item: 128 queries of one (sequence, query head). Two CTAs per SM, each
// a pipeline that walks items blockIdx.x, blockIdx.x + gridDim.x, ... and,
// inside an item, blocks of 64 keys:
//   S   = Q K^T                (TMEM, M = 128 queries, N = 64 keys; two buffers)
//   P   = exp2(S * scale_log2 - m)   (one thread per query row, online softmax)
//   O  += P V                  (TMEM, N = 64; two buffers, one per item in flight)
// Roles (10 warps):
//   warp 0     producer: TMA of the item's Q tile (reloaded as soon as the
//              last score MMA of the previous item has read it) and of K / V
//              blocks through three stages;
//   warp 1     TMEM owner (256 columns: S[2] 0-127, O[2] 128-255) and the one
//              thread issuing MMAs: S(j + 1) is issued before P V(j), so the
//              tensor core computes the next scores while the softmax warps
//              work on block j;
//   warps 2-9  two threads per query row (TMEM lane quadrant = warp % 4),
//              warps 2-5 on key columns 0-31 of a block and 6-9 on 32-63: masks,
//              the row maximum (the halves exchange theirs through shared
//              memory), online softmax in registers, P into one of two shared-
//              memory buffers; the rare O rescale (when a block raises the
//              running maximum by more than 2^8) waits for the previous P V and
//              scales each half's O columns; then, once per item, O / l as bf16
//              (l summed over both halves) and the base-2 log-sum-exp.
// O and the normaliser always share one maximum, so the result is exact.
// Every wait is bounded (%globaltimer); a wait that runs out records a status
// code and raises a CTA-wide abort flag; each role leaves its loop, copies and
// MMAs in flight are drained, TMEM is freed and the kernel returns.
//
// Reference parity: `dot_product_attention` with padding / window / causal
// masks and GQA (src/representax/models/components.py:187-235,
// src/representax/models/qwen3_vl/text.py:188-199); dropout draws the 8-bit
// Philox decisions that the backward regenerates (attention_tc.cuh).
#include <algorithm>

#include "attention_tc.cuh"

namespace rx {
namespace attn {
namespace wsf {

using tc::Drop8;
using tc::drop8;
using tc::ex2;
using tc::fwd_keep_bits;
using tc::kSub128;
using tc::pack2;
using tc::store_chunk_sw128;

constexpr int D = 64;
constexpr int BQ = 128;  // queries per item (TMEM lanes)
constexpr int BKB = 64;  // keys per block
constexpr int KST = 3;   // K / V stages
constexpr int kWarps = 10, kThreads = 32 * kWarps;
constexpr int kSoftWarp0 = 2;  // warps 2-5: key columns 0-31 of a block, 6-9: columns 32-63
constexpr int kSoftThreads = 256;
constexpr uint32_t kSubK = BKB * 128;  // [64 keys][64 bf16] swizzled tile

// Shared-memory layout (offsets from a 1024-byte aligned base).
constexpr uint32_t QT = 0;                      // Q [128][64]
constexpr uint32_t KV = QT + kSub128;           // stage s: K at KV + s * 16K, V at + 8K
constexpr uint32_t PB = KV + KST * 2 * kSubK;   // buffer b: P [128][64] at PB + b * 16K
constexpr uint32_t XM = PB + 2 * kSub128;      // row maxima of the two column halves: [2 blocks][2][128]
constexpr uint32_t XL = XM + 2 * 2 * BQ * 4;    // row normalisers of the two halves: [2][128]
constexpr uint32_t BARS = XL + 2 * BQ * 4;
enum : int {
  kQFull = 0, kQEmpty, kKvFull, kKvEmpty = kKvFull + KST, kSFull = kKvEmpty + KST, kPFull = kSFull + 2,
  kPEmpty = kPFull + 2, kODone = kPEmpty + 2, kOFull, kOEmpty = kOFull + 2, kRowMax = kOEmpty + 2, kRowSum,
  kDrain, kNumBars
};
constexpr uint32_t BYTES = BARS + kNumBars * 8 + 16 + 1024;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t T_S = 0, T_O = 128;

// One work item: queries [q_lo, q_hi) of sequence b, head h; keys [k_lo, k_hi).
struct Item {
  int start, len, h, q_lo, q_hi, k_lo, k_hi, nblk;
};

__device__ __forceinline__ bool item_at(const Params& p, int u, int tiles, Item& it) {
  const int h = u % p.heads;
  const int rest = u / p.heads;
  const int qt = rest % tiles, b = rest / tiles;
  const int start = p.cu_seqlens[b];
  const int len = p.cu_seqlens[b + 1] - start;
  const int q_lo = qt * BQ;
  if (q_lo >= len) return false;
  it.start = start;
  it.len = len;
  it.h = h;
  it.q_lo = q_lo;
  it.q_hi = min(len, q_lo + BQ);
  int k_lo = 0, k_hi = len;
  if (p.causal) k_hi = min(k_hi, it.q_hi);
  if (p.window >= 0) {
    k_lo = max(0, q_lo - p.window);
    k_hi = min(k_hi, it.q_hi + p.window);
  }
  it.k_lo = k_lo;
  it.k_hi = k_hi;
  it.nblk = (k_hi - k_lo + BKB - 1) / BKB;  // >= 1: query q_lo always sees itself
  return true;
}

__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, const Params& p, volatile int* abort,
                                              int code) {
  if (*abort) return false;
  if (mbar_wait(bar, parity, p.timeout_ns)) return true;
  report_status(p.status, code);
  *abort = 1;
  return false;
}

__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_ws_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const Params p, int tiles, int num_items) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = tc::align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + BARS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(&bars[kQFull], 1);
    mbar_init(&bars[kQEmpty], 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(&bars[kKvFull + s], 1);
      mbar_init(&bars[kKvEmpty + s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[kSFull + i], 1);
      mbar_init(&bars[kPFull + i], kSoftThreads);
      mbar_init(&bars[kPEmpty + i], 1);
      mbar_init(&bars[kOFull + i], 1);
      mbar_init(&bars[kOEmpty + i], kSoftThreads);
    }
    mbar_init(&bars[kODone], 1);
    mbar_init(&bars[kRowMax], kSoftThreads);
    mbar_init(&bars[kRowSum], kSoftThreads);
    mbar_init(&bars[kDrain], 1);
    *abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_map(&tmQ);
      tma_prefetch_map(&tmK);
      tma_prefetch_map(&tmV);
      uint32_t ib = 0, nb = 0, q_issued = 0;
      uint32_t kv_issued[KST] = {0, 0, 0};
      bool ok = true;
      for (int u = blockIdx.x; ok && u < num_items; u += gridDim.x) {
        Item it;
        if (!item_at(p, u, tiles, it)) continue;
        if (!wait_or_abort(&bars[kQEmpty], (ib & 1) ^ 1, p, abort, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&bars[kQFull], kSub128);
        tma_load_2d(base + QT, &tmQ, &bars[kQFull], it.h * D, it.start + it.q_lo);
        ++q_issued;
        const int kvh = it.h / p.heads_per_kv;
        for (int j = 0; j < it.nblk; ++j, ++nb) {
          const int s = nb % KST;
          if (!wait_or_abort(&bars[kKvEmpty + s], ((nb / KST) & 1) ^ 1, p, abort, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          uint8_t* kv = base + KV + s * 2 * kSubK;
          mbar_arrive_expect_tx(&bars[kKvFull + s], 2 * kSubK);
          tma_load_2d(kv, &tmK, &bars[kKvFull + s], kvh * D, it.start + it.k_lo + j * BKB);
          tma_load_2d(kv + kSubK, &tmV, &bars[kKvFull + s], kvh * D, it.start + it.k_lo + j * BKB);
          ++kv_issued[s];
        }
        ++ib;
      }
      if (!ok) {  // let every issued copy land before the CTA can exit
        if (q_issued > 0 && !mbar_wait(&bars[kQFull], (q_issued - 1) & 1, p.timeout_ns))
          report_status(p.status, kStatusTimeoutDrain);
        for (int s = 0; s < KST; ++s)
          if (kv_issued[s] > 0 && !mbar_wait(&bars[kKvFull + s], (kv_issued[s] - 1) & 1, p.timeout_ns))
            report_status(p.status, kStatusTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_O = idesc_bf16_f32(128, D, false, true);  // O: M = queries, N = D, V MN-major
      const uint32_t sQ = smem_u32(base + QT);
      uint32_t ib = 0, nb = 0;
      bool ok = true, issued = false;
      // S(n) = Q K^T of the item's block j into S buffer n & 1
      auto scores = [&](uint32_t n, int j, const Item& it) -> bool {
        const uint32_t s = n % KST, b2 = n & 1;
        if (!wait_or_abort(&bars[kKvFull + s], (n / KST) & 1, p, abort, kStatusTimeoutMma) ||
            !wait_or_abort(&bars[kPFull + b2], ((n >> 1) & 1) ^ 1, p, abort, kStatusTimeoutMma))
          return false;
        tc_fence_after();
        const int n16 = (min(BKB, it.k_hi - (it.k_lo + j * BKB)) + 15) & ~15;
        const uint32_t idesc_s = idesc_bf16_f32(128, n16, false, false);
        const uint32_t sK = smem_u32(base + KV + s * 2 * kSubK);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_f16_ss(tmem + T_S + b2 * BKB, smem_desc_sw128(sQ + kk * 32, 16, 1024),
                      smem_desc_sw128(sK + kk * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&bars[kSFull + b2]);
        issued = true;
        return true;
      };
      for (int u = blockIdx.x; ok && u < num_items; u += gridDim.x) {
        Item it;
        if (!item_at(p, u, tiles, it)) continue;
        const uint32_t ob = ib & 1;
        if (!wait_or_abort(&bars[kQFull], ib & 1, p, abort, kStatusTimeoutMma) || !scores(nb, 0, it)) {
          ok = false;
          break;
        }
        if (it.nblk == 1) umma_commit(&bars[kQEmpty]);  // Q is read by the score MMAs only
        for (int j = 0; j < it.nblk; ++j) {
          const uint32_t n = nb + j;
          if (j + 1 < it.nblk) {
            if (!scores(n + 1, j + 1, it)) {
              ok = false;
              break;
            }
            if (j + 2 == it.nblk) umma_commit(&bars[kQEmpty]);
          }
          // O += P V of block n
          const uint32_t s = n % KST, b2 = n & 1;
          if (!wait_or_abort(&bars[kPFull + b2], (n >> 1) & 1, p, abort, kStatusTimeoutMma) ||
              (j == 0 && !wait_or_abort(&bars[kOEmpty + ob], ((ib >> 1) & 1) ^ 1, p, abort, kStatusTimeoutMma))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int n16 = (min(BKB, it.k_hi - (it.k_lo + j * BKB)) + 15) & ~15;
          const uint32_t sV = smem_u32(base + KV + s * 2 * kSubK) + kSubK, sP = smem_u32(base + PB + b2 * kSub128);
          for (int kk = 0; kk < n16 / 16; ++kk)
            umma_f16_ss(tmem + T_O + ob * D, smem_desc_sw128(sP + kk * 32, 16, 1024),
                        smem_desc_sw128(sV + kk * 2048, kSubK, 1024), IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&bars[kPEmpty + b2]);
          umma_commit(&bars[kKvEmpty + s]);
          umma_commit(&bars[kODone]);
        }
        if (!ok) break;
        umma_commit(&bars[kOFull + ob]);
        nb += it.nblk;
        ++ib;
      }
      if (issued) {
        umma_commit(&bars[kDrain]);
        if (!mbar_wait(&bars[kDrain], 0, p.timeout_ns)) report_status(p.status, kStatusTimeoutDrain);
      }
    }
  } else if (warp >= kSoftWarp0 && warp < kSoftWarp0 + 8) {
    // ------------------------------------------------------------ softmax / epilogue
    const int quad = warp & 3;
    const int half = (warp - kSoftWarp0) >> 2;  // key columns [32 half, 32 half + 32) of each block
    const int row = quad * 32 + lane;
    const int c_base = half * 32;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    float* xmax = reinterpret_cast<float*>(base + XM);  // [block & 1][half][row]
    float* xl = reinterpret_cast<float*>(base + XL);    // [half][row]
    const float sl2 = p.scale_log2;
    const Drop8 dr = drop8(p.pdrop);
    const bool drop = dr.t8 != 0u;
    uint32_t ib = 0, nb = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < num_items; u += gridDim.x) {
      Item it;
      if (!item_at(p, u, tiles, it)) continue;
      const uint32_t ob = ib & 1;
      const int i = it.q_lo + row;  // this thread's query (sequence-relative)
      const bool warp_live = it.q_lo + quad * 32 < it.len;
      int vis_lo = 0, vis_hi = it.len;  // keys this query may see
      if (p.causal) vis_hi = min(vis_hi, i + 1);
      if (p.window >= 0) {
        vis_lo = max(0, i - p.window);
        vis_hi = min(vis_hi, i + p.window + 1);
      }
      // m_run is the same in both halves (built from the exchanged maxima);
      // l_run is this half's share of the normaliser.
      float m_run = -INFINITY, l_run = 0.f;  // scaled base-2 units
      for (int j = 0; j < it.nblk; ++j) {
        const uint32_t n = nb + j, b2 = n & 1;
        const int k0 = it.k_lo + j * BKB;
        const int n16 = (min(BKB, it.k_hi - k0) + 15) & ~15;
        const bool cols_live = c_base < n16;
        // keep bits depend only on coordinates: draw them before the scores land
        uint64_t keep_lo = ~0ull, keep_hi = ~0ull;
        if (drop && warp_live && cols_live)
          fwd_keep_bits(p.pdrop, dr.t8, it.start, i, it.h, k0 + c_base, min(32, n16 - c_base), lane, keep_lo,
                        keep_hi);
        ok = wait_or_abort(&bars[kSFull + b2], (n >> 1) & 1, p, abort, kStatusTimeoutEpilogue) &&
             wait_or_abort(&bars[kPEmpty + b2], ((n >> 1) & 1) ^ 1, p, abort, kStatusTimeoutEpilogue);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        uint32_t r[32];
        float mx = -INFINITY;
        if (warp_live && cols_live) {
          tmem_ld_32x32b_x32(tmem + T_S + b2 * BKB + c_base + lane_off, r);
          tmem_ld_wait();
          const int clo = vis_lo - k0 - c_base, chi = vis_hi - k0 - c_base;  // visible columns of this half
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float v = (e >= clo && e < chi && c_base + e < n16) ? __uint_as_float(r[e]) : -INFINITY;
            r[e] = __float_as_uint(v);
            mx = fmaxf(mx, v);
          }
        }
        // the row maximum of the block: both halves publish theirs, then read
        // the other's (double-buffered by block parity; bounded mbarrier wait)
        xmax[(b2 * 2 + half) * BQ + row] = mx;
        mbar_arrive(&bars[kRowMax]);
        ok = __all_sync(0xffffffffu, wait_or_abort(&bars[kRowMax], n & 1, p, abort, kStatusTimeoutEpilogue));
        if (!ok) break;
        mx = fmaxf(mx, xmax[(b2 * 2 + (half ^ 1)) * BQ + row]) * sl2;  // scaled base-2 units
        float alpha = 1.f;
        bool rescale = false;
        if (mx > -INFINITY) {
          if (m_run == -INFINITY) {
            m_run = mx;  // nothing accumulated for this row yet
          } else if (mx > m_run + 8.f) {
            alpha = ex2(m_run - mx);
            m_run = mx;
            l_run *= alpha;
            rescale = true;
          }
        }
        if (warp_live && __any_sync(0xffffffffu, rescale)) {
          // O must hold every earlier block: wait for P V of block n - 1, then
          // scale this half's 32 columns of the O rows
          ok = __all_sync(0xffffffffu, wait_or_abort(&bars[kODone], (n - 1) & 1, p, abort, kStatusTimeoutEpilogue));
          if (!ok) break;
          tc_fence_after();
          uint32_t o[32];
          tmem_ld_32x32b_x32(tmem + T_O + ob * D + c_base + lane_off, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x32(tmem + T_O + ob * D + c_base + lane_off, o);
          tmem_st_wait();
        }
        if (warp_live && cols_live) {
          const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
          float rs = 0.f;
          uint8_t* prow = base + PB + b2 * kSub128;
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            if (c_base + ch * 8 < n16) {
              float e8[8];
#pragma unroll
              for (int t = 0; t < 8; ++t) {
                const int c = ch * 8 + t;
                const float e = ex2(fmaf(__uint_as_float(r[c]), sl2, neg_m));
                rs += e;  // the normaliser uses the probabilities before dropout
                e8[t] = (!drop || ((keep_lo >> c) & 1ull)) ? e * (drop ? dr.scale : 1.f) : 0.f;
              }
              store_chunk_sw128(prow, row, half * 4 + ch, make_uint4(pack2(e8[0], e8[1]), pack2(e8[2], e8[3]),
                                                                     pack2(e8[4], e8[5]), pack2(e8[6], e8[7])));
            }
          }
          l_run += rs;
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bars[kPFull + b2]);
      }
      if (!ok) break;
      // O / l and the log-sum-exp of this item's queries (each half stores its 32 columns)
      xl[half * BQ + row] = l_run;
      mbar_arrive(&bars[kRowSum]);
      ok = __all_sync(0xffffffffu, wait_or_abort(&bars[kRowSum], ib & 1, p, abort, kStatusTimeoutEpilogue) &&
                                       wait_or_abort(&bars[kOFull + ob], (ib >> 1) & 1, p, abort,
                                                     kStatusTimeoutEpilogue));
      if (!ok) break;
      const float l_tot = l_run + xl[(half ^ 1) * BQ + row];
      tc_fence_after();
      if (warp_live) {
        const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
        uint32_t o[32];
        tmem_ld_32x32b_x32(tmem + T_O + ob * D + c_base + lane_off, o);
        tmem_ld_wait();
        if (i < it.len) {
          uint4* dst = reinterpret_cast<uint4*>(p.o + static_cast<int64_t>(it.start + i) * p.ldo + it.h * D + c_base);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float* f = reinterpret_cast<const float*>(o + q * 8);
            dst[q] = make_uint4(pack2(f[0] * inv, f[1] * inv), pack2(f[2] * inv, f[3] * inv),
                                pack2(f[4] * inv, f[5] * inv), pack2(f[6] * inv, f[7] * inv));
          }
          if (half == 0)
            p.lse[static_cast<int64_t>(it.h) * p.total_tokens + it.start + i] =
                l_tot > 0.f ? m_run + log2f(l_tot) : INFINITY;
        }
      }
      tc_fence_before();
      mbar_arrive(&bars[kOEmpty + ob]);
      nb += it.nblk;
      ++ib;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace wsf

namespace {
// Off by default: on the BERT GradCache chunk (128 sequences, lengths 32-256,
// 12 heads) it measured 0.123 ms against 0.072 ms for the per-tile kernel
// (attn_tc_fwd_kernel, four CTAs per SM); with items of one to four key
// blocks the per-item pipeline fill is not amortised.
bool g_wsf_enabled = false;
}  // namespace

bool ws_forward_enabled() { return g_wsf_enabled; }
void set_ws_forward_enabled(bool on) { g_wsf_enabled = on; }

// Launch the warp-specialised forward (head dim 64, no relative bias): two
// persistent CTAs per SM.
void tc_forward_ws(Params p, int64_t max_len, cudaStream_t st, int device, int* status) {
  p.status = status;
  p.timeout_ns = kWaitBudgetNs;
  const int64_t T = p.total_tokens;
  const int kv_heads = p.heads / p.heads_per_kv;
  const CUtensorMap tq = make_tmap_2d_bf16(p.q, T, static_cast<int64_t>(p.heads) * wsf::D, p.ldq, 64, wsf::BQ);
  const CUtensorMap tk = make_tmap_2d_bf16(p.k, T, static_cast<int64_t>(kv_heads) * wsf::D, p.ldk, 64, wsf::BKB);
  const CUtensorMap tv = make_tmap_2d_bf16(p.v, T, static_cast<int64_t>(kv_heads) * wsf::D, p.ldv, 64, wsf::BKB);
  const int tiles = static_cast<int>((max_len + wsf::BQ - 1) / wsf::BQ);
  const int64_t items = static_cast<int64_t>(p.batch) * tiles * p.heads;
  RX_CHECK(items < (int64_t(1) << 31), "attention forward: too many work items");
  if (items == 0) return;
  static bool done[64] = {false};
  if (device < 0 || device >= 64 || !done[device]) {
    RX_CUDA_CHECK(cudaFuncSetAttribute(wsf::attn_fwd_ws_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(wsf::BYTES)));
    if (device >= 0 && device < 64) done[device] = true;
  }
  const int grid = static_cast<int>(std::min<int64_t>(items, 2ll * num_sms(device)));
  wsf::attn_fwd_ws_kernel<<<grid, wsf::kThreads, wsf::BYTES, st>>>(tq, tk, tv, p, tiles, static_cast<int>(items));
  RX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace attn
}  // namespace rx
