// Warp-specialised, persistent attention backward on tcgen05 (head dim 64).
//
// Work item: 128 keys of one (sequence, key/value head); a CTA (one per SM)
// walks items blockIdx.x, blockIdx.x + gridDim.x, ... and, inside an item, the
// blocks of 64 queries of every query head of the group. Per block:
//   S^T  = K Q^T,  dP^T = V dO^T                        (TMEM, M = 128 keys)
//   P^T  = exp2(S^T * scale_log2 - lse)   dS^T = P^T (dP^T - Dvec) * scale
//   dV  += P^T dO,  dK += dS^T Q                          (TMEM accumulators)
//   dQ   = dS K                                           (TMEM, rows 0-63)
// Roles (14 warps; 10 and 11 idle, so the drain warps sit on TMEM lane quadrants 0 and 1):
//   warp 0     producer: TMA of K / V (two item buffers) and of Q / dO (four
//              block stages); the block's -lse and Dvec * scale rows go to
//              shared memory by plain loads (their rows are not 16-byte
//              aligned, so no tensor copy);
//   warp 1     TMEM owner (all 512 columns) and the one thread issuing MMAs:
//              S(n + 1) is issued before the gradient MMAs of block n, so the
//              tensor core computes the next block's scores while the softmax
//              warps work on the current one;
//   warps 2-9  one key row per thread (TMEM lane quadrant = warp % 4), warps
//              2-5 on query columns 0-31 and 6-9 on 32-63: P^T and dS^T into one
//              of two shared-memory buffers, then, once per item, the dK (warps
//              2-5) / dV (warps 6-9) epilogue (bf16 rows, bias column sums);
//   warps 12-13 dQ drain: query rows 0-63 of the dQ accumulator (two TMEM
//              buffers), released before the fp32 vector atomics into dq_acc.
// TMEM columns: S^T[2] 0-127, dP^T[2] 128-255, dV 256-319, dK 320-383,
// dQ[2] 384-511.
// Every wait is bounded (%globaltimer); a wait that runs out records a status
// code and raises a CTA-wide abort flag; each role leaves its loop, copies and
// MMAs in flight are drained, TMEM is freed and the kernel returns. The
// softmax warps meet each other only on mbarriers (bounded), never on a named
// barrier, so a warp that unwinds cannot strand the others.
//
// Reference parity: the gradient of `dot_product_attention` with padding /
// window / causal masks and GQA (src/representax/models/components.py:187-235,
// src/representax/models/qwen3_vl/text.py:188-199); dropout masks are the
// 8-bit Philox decisions of the forward kernel (attention_tc.cuh).
#include <algorithm>

#include "attention_tc.cuh"

namespace rx {
namespace attn {
namespace ws {

using tc::bwd_keep_bits;
using tc::Drop8;
using tc::drop8;
using tc::ex2;
using tc::kSub128;
using tc::kSub64;
using tc::pack2;
using tc::store_chunk_sw128;

constexpr int D = 64;
constexpr int BK = 128;  // keys per item (TMEM lanes)
constexpr int BQ = 64;   // queries per block
constexpr int QST = 4;   // Q / dO stages
constexpr int kWarps = 14, kThreads = 32 * kWarps;
constexpr int kSoftWarp0 = 2, kDrainWarp0 = 12;  // softmax warps 2-9, dQ drain 12-13
constexpr int kSoftThreads = 256;

// Shared-memory layout (offsets from a 1024-byte aligned base).
constexpr uint32_t KV = 0;                          // buffer b: K at KV + b * 32K, V at + 16K
constexpr uint32_t QD = KV + 2 * 2 * kSub128;       // stage s: Q at QD + s * 16K, dO at + 8K
constexpr uint32_t PB = QD + QST * 2 * kSub64;      // buffer b: dS^T at PB + b * 32K, P^T at + 16K
constexpr uint32_t LS = PB + 2 * 2 * kSub128;       // stage s: -lse[64], Dvec * scale[64]
constexpr uint32_t CS = LS + QST * 2 * BQ * 4;      // dK | dV column sums of an item (128 floats)
constexpr uint32_t BARS = CS + 2 * D * 4;
enum : int {
  kKvFull = 0, kKvEmpty = 2, kQdFull = 4, kQdEmpty = kQdFull + QST, kSFull = kQdEmpty + QST, kPFull = kSFull + 2,
  kPEmpty = kPFull + 2, kDqFull = kPEmpty + 2, kDqEmpty = kDqFull + 2, kAccFull = kDqEmpty + 2, kAccEmpty,
  kDrain, kCsAdded, kCsCleared, kNumBars
};
constexpr uint32_t BYTES = BARS + kNumBars * 8 + 16 + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t T_S = 0, T_DP = 128, T_DV = 256, T_DK = 320, T_DQ = 384;

// One work item: keys [kt0, kt_hi) of sequence b, key/value head kvh.
struct Item {
  int start, len, kt0, kt_hi, kvh;
  int q_first, q_end, nqb, blocks;
};

__device__ __forceinline__ bool item_at(const Params& p, int u, int kv_heads, int tiles, Item& it) {
  const int kvh = u % kv_heads;
  const int rest = u / kv_heads;
  const int kt = rest % tiles, b = rest / tiles;
  const int start = p.cu_seqlens[b];
  const int len = p.cu_seqlens[b + 1] - start;
  const int kt0 = kt * BK;
  if (kt0 >= len) return false;
  it.start = start;
  it.len = len;
  it.kt0 = kt0;
  it.kt_hi = min(len, kt0 + BK);
  it.kvh = kvh;
  int q_first = 0, q_end = len;
  if (p.causal) q_first = kt0;
  if (p.window >= 0) {
    q_first = max(q_first, kt0 - p.window);
    q_end = min(q_end, it.kt_hi + p.window);
  }
  it.q_first = q_first;
  it.q_end = q_end;
  it.nqb = q_end > q_first ? (q_end - q_first + BQ - 1) / BQ : 0;
  it.blocks = it.nqb * p.heads_per_kv;
  return true;
}

// Bounded wait that honours the CTA abort flag; on a timeout it records
// `code` and raises the flag. Returns false when the caller must unwind.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, const Params& p, volatile int* abort,
                                              int code) {
  if (*abort) return false;
  if (mbar_wait(bar, parity, p.timeout_ns)) return true;
  report_status(p.status, code);
  *abort = 1;
  return false;
}

// Column sums of a warp's 32 x 32 block (lane = row, v[i] = column i): after
// the butterfly, lane l holds the sum over all rows of column l.
__device__ __forceinline__ float warp_column_sum(float (&v)[32]) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool upper = (threadIdx.x & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = upper ? v[i] : v[i + o];
      const float keep = upper ? v[i + o] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return v[0];
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_ws_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const Params p, int tiles, int num_items) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = tc::align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + BARS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = warp_id(), lane = lane_id();
  const int kv_heads = p.heads / p.heads_per_kv;
  const int width_q = p.heads * D;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars[kKvFull + i], 1);
      mbar_init(&bars[kKvEmpty + i], 1);
      mbar_init(&bars[kSFull + i], 1);
      mbar_init(&bars[kPFull + i], kSoftThreads);
      mbar_init(&bars[kPEmpty + i], 1);
      mbar_init(&bars[kDqFull + i], 1);
      mbar_init(&bars[kDqEmpty + i], 64);
    }
    for (int s = 0; s < QST; ++s) {
      mbar_init(&bars[kQdFull + s], 32);
      mbar_init(&bars[kQdEmpty + s], 1);
    }
    mbar_init(&bars[kAccFull], 1);
    mbar_init(&bars[kAccEmpty], kSoftThreads);
    mbar_init(&bars[kDrain], 1);
    mbar_init(&bars[kCsAdded], kSoftThreads);
    mbar_init(&bars[kCsCleared], kSoftThreads);
    *abort = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  float* s_colsum = reinterpret_cast<float*>(base + CS);
  if (threadIdx.x < 2 * D) s_colsum[threadIdx.x] = 0.f;
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
      tma_prefetch_map(&tmDO);
    }
    uint32_t n = 0, ib = 0;  // blocks / items issued by this CTA
    uint32_t kv_issued[2] = {0, 0}, qd_issued[QST] = {0, 0, 0, 0};
    bool ok = true;
    for (int u = blockIdx.x; ok && u < num_items; u += gridDim.x) {
      Item it;
      if (!item_at(p, u, kv_heads, tiles, it) || it.blocks == 0) continue;
      const int kvb = ib & 1;
      if (lane == 0) {
        ok = wait_or_abort(&bars[kKvEmpty + kvb], ((ib >> 1) & 1) ^ 1, p, abort, kStatusTimeoutProducer);
        if (ok) {
          uint8_t* kv = base + KV + kvb * 2 * kSub128;
          mbar_arrive_expect_tx(&bars[kKvFull + kvb], 2 * kSub128);
          tma_load_2d(kv, &tmK, &bars[kKvFull + kvb], it.kvh * D, it.start + it.kt0);
          tma_load_2d(kv + kSub128, &tmV, &bars[kKvFull + kvb], it.kvh * D, it.start + it.kt0);
          ++kv_issued[kvb];
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      for (int j = 0; ok && j < it.blocks; ++j, ++n) {
        const int s = n % QST;
        const int hq = it.kvh * p.heads_per_kv + j / it.nqb;
        const int q0 = it.q_first + (j % it.nqb) * BQ;
        // this block's -lse / Dvec rows: loads issued before the stage is free
        float lv[2], dv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int q = q0 + lane + 32 * e;
          const int64_t at = static_cast<int64_t>(hq) * p.total_tokens + it.start + q;
          lv[e] = q < it.len ? -p.lse[at] : -INFINITY;
          dv[e] = q < it.len ? p.dvec[at] * p.scale : 0.f;
        }
        if (lane == 0) ok = wait_or_abort(&bars[kQdEmpty + s], ((n / QST) & 1) ^ 1, p, abort, kStatusTimeoutProducer);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (lane == 0) {  // copies first; every lane arrives after its shared-memory stores
          uint8_t* qd = base + QD + s * 2 * kSub64;
          mbar_expect_tx(&bars[kQdFull + s], 2 * kSub64);
          tma_load_2d(qd, &tmQ, &bars[kQdFull + s], hq * D, it.start + q0);
          tma_load_2d(qd + kSub64, &tmDO, &bars[kQdFull + s], hq * D, it.start + q0);
          ++qd_issued[s];
        }
        float* nlse = reinterpret_cast<float*>(base + LS + s * 2 * BQ * 4);
        float* dvs = nlse + BQ;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          nlse[lane + 32 * e] = lv[e];
          dvs[lane + 32 * e] = dv[e];
        }
        mbar_arrive(&bars[kQdFull + s]);
      }
      ++ib;
    }
    if (!ok && lane == 0) {
      // let every issued copy land before the CTA can exit
      for (int b = 0; b < 2; ++b)
        if (kv_issued[b] > 0 && !mbar_wait(&bars[kKvFull + b], (kv_issued[b] - 1) & 1, p.timeout_ns))
          report_status(p.status, kStatusTimeoutDrain);
      for (int s = 0; s < QST; ++s)
        if (qd_issued[s] > 0 && !mbar_wait(&bars[kQdFull + s], (qd_issued[s] - 1) & 1, p.timeout_ns))
          report_status(p.status, kStatusTimeoutDrain);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_KV = idesc_bf16_f32(128, D, false, true);  // dV, dK: M = keys, N = D
      constexpr uint32_t IDESC_Q = idesc_bf16_f32(128, D, true, true);    // dQ: M = queries (64 used)
      uint32_t n = 0, ib = 0;
      bool ok = true, issued = false;
      // gradient MMAs of block m (item-local index jj) of the current item
      auto grads = [&](uint32_t m, int jj, const Item& it, uint32_t sK) -> bool {
        const uint32_t b2 = m & 1, s = m % QST;
        if (!wait_or_abort(&bars[kPFull + b2], (m >> 1) & 1, p, abort, kStatusTimeoutMma)) return false;
        if (jj == 0 && !wait_or_abort(&bars[kAccEmpty], (ib & 1) ^ 1, p, abort, kStatusTimeoutMma)) return false;
        if (!wait_or_abort(&bars[kDqEmpty + b2], ((m >> 1) & 1) ^ 1, p, abort, kStatusTimeoutMma)) return false;
        tc_fence_after();
        const int q0 = it.q_first + (jj % it.nqb) * BQ;
        const int nq16 = (min(BQ, it.q_end - q0) + 15) & ~15;
        const int nk16 = (it.kt_hi - it.kt0 + 15) & ~15;
        const uint32_t sQ = smem_u32(base + QD + s * 2 * kSub64), sDO = sQ + kSub64;
        const uint32_t sDST = smem_u32(base + PB + b2 * 2 * kSub128), sPT = sDST + kSub128;
        for (int kk = 0; kk < nq16 / 16; ++kk) {
          const uint32_t acc = (jj > 0 || kk > 0) ? 1u : 0u;
          umma_f16_ss(tmem + T_DV, smem_desc_sw128(sPT + kk * 32, 16, 1024),
                      smem_desc_sw128(sDO + kk * 2048, kSub64, 1024), IDESC_KV, acc);
          umma_f16_ss(tmem + T_DK, smem_desc_sw128(sDST + kk * 32, 16, 1024),
                      smem_desc_sw128(sQ + kk * 2048, kSub64, 1024), IDESC_KV, acc);
        }
        // dQ = dS K: A is the MN-major view of dS^T whose second 64-row chunk
        // is the P^T buffer (output rows 64-127, never read)
        for (int kk = 0; kk < nk16 / 16; ++kk)
          umma_f16_ss(tmem + T_DQ + b2 * D, smem_desc_sw128(sDST + kk * 2048, kSub128, 1024),
                      smem_desc_sw128(sK + kk * 2048, kSub128, 1024), IDESC_Q, kk > 0 ? 1u : 0u);
        umma_commit(&bars[kPEmpty + b2]);
        umma_commit(&bars[kQdEmpty + s]);
        umma_commit(&bars[kDqFull + b2]);
        return true;
      };
      for (int u = blockIdx.x; ok && u < num_items; u += gridDim.x) {
        Item it;
        if (!item_at(p, u, kv_heads, tiles, it) || it.blocks == 0) continue;
        const int kvb = ib & 1;
        if (!wait_or_abort(&bars[kKvFull + kvb], (ib >> 1) & 1, p, abort, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        const uint32_t sK = smem_u32(base + KV + kvb * 2 * kSub128), sV = sK + kSub128;
        const uint32_t n0 = n;
        for (int j = 0; j < it.blocks; ++j, ++n) {
          const uint32_t b2 = n & 1, s = n % QST;
          if (!wait_or_abort(&bars[kQdFull + s], (n / QST) & 1, p, abort, kStatusTimeoutMma) ||
              !wait_or_abort(&bars[kPFull + b2], ((n >> 1) & 1) ^ 1, p, abort, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int q0 = it.q_first + (j % it.nqb) * BQ;
          const int nq16 = (min(BQ, it.q_end - q0) + 15) & ~15;
          const uint32_t idesc_s = idesc_bf16_f32(128, nq16, false, false);
          const uint32_t sQ = smem_u32(base + QD + s * 2 * kSub64), sDO = sQ + kSub64;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            umma_f16_ss(tmem + T_S + b2 * BQ, smem_desc_sw128(sK + kk * 32, 16, 1024),
                        smem_desc_sw128(sQ + kk * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
            umma_f16_ss(tmem + T_DP + b2 * BQ, smem_desc_sw128(sV + kk * 32, 16, 1024),
                        smem_desc_sw128(sDO + kk * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
          }
          umma_commit(&bars[kSFull + b2]);
          issued = true;
          if (j > 0 && !grads(n - 1, j - 1, it, sK)) {
            ok = false;
            break;
          }
        }
        if (!ok || !grads(n - 1, static_cast<int>(n - 1 - n0), it, sK)) {
          ok = false;
          break;
        }
        umma_commit(&bars[kKvEmpty + kvb]);
        umma_commit(&bars[kAccFull]);
        ++ib;
      }
      if (issued) {
        umma_commit(&bars[kDrain]);
        if (!mbar_wait(&bars[kDrain], 0, p.timeout_ns)) report_status(p.status, kStatusTimeoutDrain);
      }
    }
  } else if (warp >= kSoftWarp0 && warp < kSoftWarp0 + 8) {
    // ------------------------------------------------------------ softmax / dS, dK dV epilogue
    const int quad = warp & 3;
    const int half = (warp - kSoftWarp0) >> 2;  // query columns [32 half, 32 half + 32); epilogue: dK / dV
    const int krow = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const float sl2 = p.scale_log2, scale = p.scale;
    const Drop8 dr = drop8(p.pdrop);
    const bool drop = dr.t8 != 0u;
    uint32_t n = 0, ib = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < num_items; u += gridDim.x) {
      Item it;
      if (!item_at(p, u, kv_heads, tiles, it)) continue;
      const int key = it.kt0 + krow;
      const bool warp_live = it.kt0 + quad * 32 < it.len;
      if (it.blocks == 0) {  // no query sees these keys: zero gradients
        if (key < it.len) {
          __nv_bfloat16* row = half == 0 ? p.dk + static_cast<int64_t>(it.start + key) * p.ld_dk + it.kvh * D
                                         : p.dv + static_cast<int64_t>(it.start + key) * p.ld_dv + it.kvh * D;
#pragma unroll
          for (int q = 0; q < D / 8; ++q) reinterpret_cast<uint4*>(row)[q] = make_uint4(0u, 0u, 0u, 0u);
        }
        continue;
      }
      int vis_lo = 0, vis_hi = key < it.len ? it.len : 0;  // queries that may see this key
      if (p.causal) vis_lo = key;
      if (p.window >= 0) {
        vis_lo = max(vis_lo, key - p.window);
        vis_hi = min(vis_hi, key + p.window + 1);
      }
      for (int jj = 0; jj < it.blocks; ++jj, ++n) {
        const uint32_t b2 = n & 1, s = n % QST;
        const int hq = it.kvh * p.heads_per_kv + jj / it.nqb;
        const int q0 = it.q_first + (jj % it.nqb) * BQ;
        const int nq16 = (min(BQ, it.q_end - q0) + 15) & ~15;
        const int c_base = half * 32;  // this warp's query columns
        const bool cols_live = c_base < nq16;
        // keep bits depend only on coordinates: draw them before the scores land
        uint64_t keep = ~0ull;
        if (drop && warp_live && cols_live)
          keep = bwd_keep_bits(p.pdrop, dr.t8, it.start, key, hq, q0 + c_base, min(32, nq16 - c_base), lane);
        ok = wait_or_abort(&bars[kSFull + b2], (n >> 1) & 1, p, abort, kStatusTimeoutEpilogue) &&
             wait_or_abort(&bars[kQdFull + s], (n / QST) & 1, p, abort, kStatusTimeoutEpilogue) &&
             wait_or_abort(&bars[kPEmpty + b2], ((n >> 1) & 1) ^ 1, p, abort, kStatusTimeoutEpilogue);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const float* s_nlse = reinterpret_cast<const float*>(base + LS + s * 2 * BQ * 4);
        const float* s_dvs = s_nlse + BQ;
        uint8_t* dst = base + PB + b2 * 2 * kSub128;
        uint8_t* pt = dst + kSub128;
        if (warp_live) {
          if (cols_live) {
            const int clo = vis_lo - q0, chi = vis_hi - q0;  // visible query columns of this block
            uint32_t rs[32], rd[32];
            tmem_ld_32x32b_x32(tmem + T_S + b2 * BQ + c_base + lane_off, rs);
            tmem_ld_32x32b_x32(tmem + T_DP + b2 * BQ + c_base + lane_off, rd);
            tmem_ld_wait();
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
              const int c0 = c_base + ch * 8;
              if (c0 < nq16) {
                float pv[8], dv[8];
#pragma unroll
                for (int t = 0; t < 8; ++t) {
                  const int c = c0 + t;
                  const float sc = __uint_as_float(rs[ch * 8 + t]);
                  const float pr = (c >= clo && c < chi) ? ex2(fmaf(sc, sl2, s_nlse[c])) : 0.f;
                  if (!drop) {
                    pv[t] = pr;
                    dv[t] = pr * fmaf(__uint_as_float(rd[ch * 8 + t]), scale, -s_dvs[c]);  // P (dP - Dvec) * scale
                  } else {
                    // dV uses the dropped probabilities; dS = P (mask * dP / (1 - p) - Dvec)
                    const bool kept = ((keep >> (ch * 8 + t)) & 1ull) != 0ull;
                    const float dp = kept ? __uint_as_float(rd[ch * 8 + t]) * dr.scale : 0.f;
                    pv[t] = kept ? pr * dr.scale : 0.f;
                    dv[t] = pr * fmaf(dp, scale, -s_dvs[c]);
                  }
                }
                store_chunk_sw128(pt, krow, c0 >> 3, make_uint4(pack2(pv[0], pv[1]), pack2(pv[2], pv[3]),
                                                                pack2(pv[4], pv[5]), pack2(pv[6], pv[7])));
                store_chunk_sw128(dst, krow, c0 >> 3, make_uint4(pack2(dv[0], dv[1]), pack2(dv[2], dv[3]),
                                                                 pack2(dv[4], dv[5]), pack2(dv[6], dv[7])));
              }
            }
          }
        } else {
          // keys past the sequence: zero rows (dS^T rows enter dQ = dS K)
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            store_chunk_sw128(pt, krow, half * 4 + ch, make_uint4(0u, 0u, 0u, 0u));
            store_chunk_sw128(dst, krow, half * 4 + ch, make_uint4(0u, 0u, 0u, 0u));
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bars[kPFull + b2]);
      }
      if (!ok) break;
      // dK (warps 2-5) or dV (warps 6-9) of this item's keys
      ok = __all_sync(0xffffffffu, wait_or_abort(&bars[kAccFull], ib & 1, p, abort, kStatusTimeoutEpilogue));
      if (!ok) break;
      tc_fence_after();
      const int which = half;  // 0: dK, 1: dV
      if (warp_live) {
        __nv_bfloat16* out = which == 0 ? p.dk + static_cast<int64_t>(it.start + key) * p.ld_dk + it.kvh * D
                                        : p.dv + static_cast<int64_t>(it.start + key) * p.ld_dv + it.kvh * D;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tmem + (which == 0 ? T_DK : T_DV) + c * 32 + lane_off, o);
          tmem_ld_wait();
          if (key < it.len) {
            uint4* d4 = reinterpret_cast<uint4*>(out + c * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float* f = reinterpret_cast<const float*>(o + q * 8);
              d4[q] = make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
            }
          }
          if (p.dbias_qkv != nullptr) {
            // bias gradient: column sums of the bf16 rows this CTA wrote
            float f[32];
#pragma unroll
            for (int e = 0; e < 32; ++e)
              f[e] = key < it.len ? __bfloat162float(__float2bfloat16_rn(__uint_as_float(o[e]))) : 0.f;
            atomicAdd(s_colsum + which * D + c * 32 + lane, warp_column_sum(f));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bars[kAccEmpty]);
      if (p.dbias_qkv != nullptr) {
        // the eight warps meet on mbarriers (bounded waits, unlike a named
        // barrier, so a warp that unwinds cannot strand the others)
        mbar_arrive(&bars[kCsAdded]);
        ok = __all_sync(0xffffffffu, wait_or_abort(&bars[kCsAdded], ib & 1, p, abort, kStatusTimeoutEpilogue));
        if (!ok) break;
        const int t = half * 128 + quad * 32 + lane;  // 0..255; the dK warps' 128 threads publish the sums
        if (t < 2 * D) {                              // of dK columns then dV columns
          const float v = s_colsum[t];
          s_colsum[t] = 0.f;
          const int qd_w = p.heads * D, kd_w = kv_heads * D;
          atomicAdd(p.dbias_qkv + qd_w + (t < D ? 0 : kd_w) + it.kvh * D + (t & (D - 1)), v);
        }
        mbar_arrive(&bars[kCsCleared]);
        ok = __all_sync(0xffffffffu, wait_or_abort(&bars[kCsCleared], ib & 1, p, abort, kStatusTimeoutEpilogue));
        if (!ok) break;
      }
      ++ib;
    }
  } else if (warp >= kDrainWarp0 && warp < kDrainWarp0 + 2) {
    // ------------------------------------------------------------ dQ drain
    const int quad = warp & 3;  // 0 or 1: query rows 0-63
    const int r = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    uint32_t n = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < num_items; u += gridDim.x) {
      Item it;
      if (!item_at(p, u, kv_heads, tiles, it) || it.blocks == 0) continue;
      for (int jj = 0; jj < it.blocks; ++jj, ++n) {
        const uint32_t b2 = n & 1;
        const int hq = it.kvh * p.heads_per_kv + jj / it.nqb;
        const int q0 = it.q_first + (jj % it.nqb) * BQ;
        ok = __all_sync(0xffffffffu,
                        wait_or_abort(&bars[kDqFull + b2], (n >> 1) & 1, p, abort, kStatusTimeoutEpilogue));
        if (!ok) break;
        tc_fence_after();
        uint32_t o0[32], o1[32];
        tmem_ld_32x32b_x32(tmem + T_DQ + b2 * D + lane_off, o0);
        tmem_ld_32x32b_x32(tmem + T_DQ + b2 * D + 32 + lane_off, o1);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&bars[kDqEmpty + b2]);
        const int q = q0 + r;
        if (q < it.q_end) {  // only queries that see a key of this item have dS rows
          float4* d4 = reinterpret_cast<float4*>(p.dq_acc + static_cast<int64_t>(it.start + q) * width_q + hq * D);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            red_add_f4(d4 + e, make_float4(__uint_as_float(o0[4 * e]), __uint_as_float(o0[4 * e + 1]),
                                          __uint_as_float(o0[4 * e + 2]), __uint_as_float(o0[4 * e + 3])));
#pragma unroll
          for (int e = 0; e < 8; ++e)
            red_add_f4(d4 + 8 + e, make_float4(__uint_as_float(o1[4 * e]), __uint_as_float(o1[4 * e + 1]),
                                              __uint_as_float(o1[4 * e + 2]), __uint_as_float(o1[4 * e + 3])));
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace ws

namespace {
bool g_ws_enabled = true;
}  // namespace

bool ws_backward_enabled() { return g_ws_enabled; }
void set_ws_backward_enabled(bool on) { g_ws_enabled = on; }

// Launch the warp-specialised backward (head dim 64, no relative bias; dq_acc
// zeroed and dvec computed by the caller). One persistent CTA per SM.
void tc_backward_ws(Params p, int64_t max_len, cudaStream_t st, int device, int* status) {
  p.status = status;
  p.timeout_ns = kWaitBudgetNs;
  const int64_t T = p.total_tokens;
  const int kv_heads = p.heads / p.heads_per_kv;
  const CUtensorMap tq = make_tmap_2d_bf16(p.q, T, static_cast<int64_t>(p.heads) * ws::D, p.ldq, 64, ws::BQ);
  const CUtensorMap tdo = make_tmap_2d_bf16(p.dO, T, static_cast<int64_t>(p.heads) * ws::D, p.ld_do, 64, ws::BQ);
  const CUtensorMap tk = make_tmap_2d_bf16(p.k, T, static_cast<int64_t>(kv_heads) * ws::D, p.ldk, 64, ws::BK);
  const CUtensorMap tv = make_tmap_2d_bf16(p.v, T, static_cast<int64_t>(kv_heads) * ws::D, p.ldv, 64, ws::BK);
  const int tiles = static_cast<int>((max_len + ws::BK - 1) / ws::BK);
  const int64_t items = static_cast<int64_t>(p.batch) * tiles * kv_heads;
  RX_CHECK(items < (int64_t(1) << 31), "attention backward: too many work items");
  if (items == 0) return;
  static bool done[64] = {false};
  if (device < 0 || device >= 64 || !done[device]) {
    RX_CUDA_CHECK(cudaFuncSetAttribute(ws::attn_bwd_ws_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(ws::BYTES)));
    if (device >= 0 && device < 64) done[device] = true;
  }
  const int grid = static_cast<int>(std::min<int64_t>(items, num_sms(device)));
  ws::attn_bwd_ws_kernel<<<grid, ws::kThreads, ws::BYTES, st>>>(tq, tk, tv, tdo, p, tiles, static_cast<int>(items));
  RX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace attn
}  // namespace rx
