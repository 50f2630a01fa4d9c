// Packed variable-length attention on the tcgen05 tensor cores (sm_100a).
//
// Same contract as the mma.sync kernels of attention.cu: packed [T, heads*D]
// rows addressed through cu_seqlens (no FLOP spent on padding), key-validity /
// causal / symmetric sliding-window masks, grouped-query heads, and the base-2
// log-sum-exp of the scaled scores saved for the backward, attention-
// probability dropout (Philox masks with 8-bit decisions, regenerated in the
// backward; see below), and MPNet's relative position bias (a
// per-head table over signed distances, added to the logits; its gradient is
// summed per diagonal in shared memory, then one global add per diagonal).
// Head dimension 64 and 128.
//
// Forward: one CTA = 128 queries of one (sequence, head), 4 warps.
//   Thread 0 issues TMA loads of Q (128 x D) and of 128-key blocks of K and V
//   into 128-byte-swizzled shared memory and issues S = Q K^T (M=128, N=128)
//   into TMEM. Each thread owns one query row (its TMEM lane): it reads its
//   128 scores with tcgen05.ld, applies the masks and the online softmax in
//   registers (no cross-thread reductions), and writes P as bf16 into
//   swizzled shared memory; thread 0 then issues O += P V (M=128, N=D, V as an
//   MN-major operand) into a second TMEM region. The running maximum only
//   moves when a block raises it by more than 2^8, so the O rescale (a TMEM
//   read-modify-write) is rare; O and the normaliser always share one maximum,
//   so the result is exact.
// Backward: one CTA = 128 keys of one (sequence, kv head), 4 warps; loops over
//   the query heads of the group and 64-query blocks:
//     S^T = K Q^T, dP^T = V dO^T                    (TMEM, M=128 keys, N=64)
//     P^T = exp2(S^T * scale_log2 - lse), dS^T = P^T (dP^T - Dvec) * scale
//                                                   (thread = key row, to smem)
//     dV += P^T dO, dK += dS^T Q                     (TMEM accumulators)
//     dQ  = dS K                                    (M=128: the upper 64 rows
//                                                    read unrelated data and
//                                                    are never used)
//   and adds the 64 dQ rows into an fp32 accumulator with vector atomics.
//
// Every wait is bounded (%globaltimer); a wait that runs out records an error
// code in the status word, the CTA drains its in-flight copies and MMAs,
// frees its TMEM and returns.
//
// Reference parity: `dot_product_attention` with padding / window / causal
// masks (src/representax/models/components.py:187-235), sliding windows
// (src/representax/models/modernvbert/model.py:217-230) and GQA
// (src/representax/models/qwen3_vl/text.py:188-199).
#include "attention_tc.cuh"  // tile constants, layouts, mask / dropout helpers

namespace rx {
namespace attn {
namespace tc {

// ===================================================================== forward
template <int D>
__global__ void __launch_bounds__(kThreads, FwdLayout<D>::CTAS_PER_SM)
    attn_tc_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const Params p) {
  using L = FwdLayout<D>;
  constexpr int DS = L::DS;
  constexpr int FK = L::FK;
  constexpr int NC = FK / 32;  // 32-column TMEM chunks of a score block
  const int h = blockIdx.y, b = blockIdx.z;
  const int start = p.cu_seqlens[b];
  const int len = p.cu_seqlens[b + 1] - start;
  const int q_lo = blockIdx.x * FQ;
  if (q_lo >= len) return;
  const int q_hi = min(len, q_lo + FQ);
  const int kvh = h / p.heads_per_kv;
  int k_lo = 0, k_hi = len;
  if (p.causal) k_hi = min(k_hi, q_hi);
  if (p.window >= 0) {
    k_lo = max(0, q_lo - p.window);
    k_hi = min(k_hi, q_hi + p.window);
  }
  const int nblk = (k_hi - k_lo + FK - 1) / FK;  // >= 1: query q_lo always sees itself

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + L::BARS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t sQ = smem_u32(base + L::Q), sK = smem_u32(base + L::K), sV = smem_u32(base + L::V),
                 sP = smem_u32(base + L::P);

  // Thread 0 issues every copy and MMA and is the only thread that waits on
  // their mbarriers; the others meet it at a block barrier. Bookkeeping of
  // issued / waited phases lets an aborting CTA drain what is in flight.
  int k_issued = 0, k_waited = 0, v_issued = 0, v_waited = 0, q_waited = 0;
  if (tid == 0) {
    for (int i = 0; i < kNumBars; ++i) mbar_init(&bars[i], 1);
    fence_mbarrier_init();
    mbar_arrive_expect_tx(&bars[kBarQ], DS * kSub128);
    for (int s = 0; s < DS; ++s) tma_load_2d(base + L::Q + s * kSub128, &tmQ, &bars[kBarQ], h * D + 64 * s, start + q_lo);
    mbar_arrive_expect_tx(&bars[kBarK], DS * L::KSUB);
    for (int s = 0; s < DS; ++s) tma_load_2d(base + L::K + s * L::KSUB, &tmK, &bars[kBarK], kvh * D + 64 * s, start + k_lo);
    mbar_arrive_expect_tx(&bars[kBarV], DS * L::KSUB);
    for (int s = 0; s < DS; ++s) tma_load_2d(base + L::V + s * L::KSUB, &tmV, &bars[kBarV], kvh * D + 64 * s, start + k_lo);
    k_issued = v_issued = 1;
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + FK;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const int row = warp * 32 + lane;
  const int i = q_lo + row;  // this thread's query (sequence-relative)
  const bool warp_live = q_lo + warp * 32 < len;
  constexpr uint32_t IDESC_O = idesc_bf16_f32(128, D, false, true);
  const float sl2 = p.scale_log2;
  // Keys this query may see: [vis_lo, vis_hi) (sequence-relative).
  int vis_lo = 0, vis_hi = len;
  if (p.causal) vis_hi = min(vis_hi, i + 1);
  if (p.window >= 0) {
    vis_lo = max(0, i - p.window);
    vis_hi = min(vis_hi, i + p.window + 1);
  }
  // Relative position bias (MPNet): logits[h, i, j] += rel_lut[h, j - i + lut_len - 1],
  // folded into the raw score as bias / scale.
  const float* lut_h =
      p.rel_lut == nullptr ? nullptr : p.rel_lut + static_cast<int64_t>(h) * (2 * p.lut_len - 1) + (p.lut_len - 1);
  const float inv_scale = 1.f / p.scale;
  const Drop8 dr = drop8(p.pdrop);
  const bool drop = dr.t8 != 0u;

  float m_run = -INFINITY, l_run = 0.f;  // in scaled base-2 units
  bool ok = true, mma_issued = false;
  for (int j = 0; j < nblk; ++j) {
    const int k0 = k_lo + j * FK;
    const uint32_t ph = static_cast<uint32_t>(j & 1);
    // Keys of this block that can be visible, rounded up to the MMA's N / K step.
    const int n16 = (min(FK, k_hi - k0) + 15) & ~15;
    const int nch = (n16 + 31) >> 5;  // 32-column TMEM chunks holding scores
    bool ok0 = true;
    if (tid == 0) {
      if (j == 0) {
        ok0 = mbar_wait(&bars[kBarQ], 0, p.timeout_ns);
        q_waited = ok0 ? 1 : 0;
      }
      if (ok0) {
        ok0 = mbar_wait(&bars[kBarK], static_cast<uint32_t>(k_waited & 1), p.timeout_ns);
        if (ok0) ++k_waited;
      }
      if (ok0) {
        tc_fence_after();
        const uint32_t idesc_s = idesc_bf16_f32(128, n16, false, false);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off_q = (kk >> 2) * kSub128 + (kk & 3) * 32;
          const uint32_t off_k = (kk >> 2) * L::KSUB + (kk & 3) * 32;
          umma_f16_ss(tS, smem_desc_sw128(sQ + off_q, 16, 1024), smem_desc_sw128(sK + off_k, 16, 1024), idesc_s,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars[kBarS]);
        mma_issued = true;
      }
    }
    // Dropout keep bits depend only on coordinates: draw them while the
    // copies and the S MMA are in flight.
    uint64_t keep_lo = ~0ull, keep_hi = ~0ull;
    __syncwarp();
    if (drop && warp_live) fwd_keep_bits(p.pdrop, dr.t8, start, i, h, k0, n16, lane, keep_lo, keep_hi);
    if (tid == 0) {
      if (ok0) ok0 = mbar_wait(&bars[kBarS], ph, p.timeout_ns);
      if (!ok0) report_status(p.status, kStatusTimeoutMma);
      // The S MMA has retired, so the K buffer is free for the next block.
      if (ok0 && j + 1 < nblk) {
        mbar_arrive_expect_tx(&bars[kBarK], DS * L::KSUB);
        for (int s = 0; s < DS; ++s)
          tma_load_2d(base + L::K + s * L::KSUB, &tmK, &bars[kBarK], kvh * D + 64 * s, start + k0 + FK);
        ++k_issued;
      }
    }
    if (__syncthreads_or(!ok0)) {
      ok = false;
      break;
    }
    tc_fence_after();

    __syncwarp();
    if (warp_live) {
      uint32_t r[NC][32];
#pragma unroll
      for (int c = 0; c < NC; ++c)
        if (c < nch) tmem_ld_32x32b_x32(tS + lane_off + c * 32, r[c]);
      tmem_ld_wait();
      const int clo = vis_lo - k0, chi = vis_hi - k0;  // visible columns of this block
      float mx = -INFINITY;
      if (lut_h == nullptr) {
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          if (c < nch) {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int col = c * 32 + e;
              const float v = (col >= clo && col < chi) ? __uint_as_float(r[c][e]) : -INFINITY;
              r[c][e] = __float_as_uint(v);
              mx = fmaxf(mx, v);
            }
          }
        }
      } else {
        const float* lut_row = lut_h + (k0 - i);  // bias of column c at lut_row[c]
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          if (c < nch) {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int col = c * 32 + e;
              const bool vis = col >= clo && col < chi && i < len;
              const float v = vis ? __uint_as_float(r[c][e]) + __ldg(lut_row + col) * inv_scale : -INFINITY;
              r[c][e] = __float_as_uint(v);
              mx = fmaxf(mx, v);
            }
          }
        }
      }
      mx *= sl2;  // scaled base-2 units (-inf stays -inf)
      float alpha = 1.f;
      bool rescale = false;
      if (mx > -INFINITY) {
        if (m_run == -INFINITY) {
          m_run = mx;  // the row of O is still zero: earlier blocks contributed nothing
        } else if (mx > m_run + 8.f) {
          alpha = ex2(m_run - mx);
          m_run = mx;
          l_run *= alpha;
          rescale = true;
        }
      }
      if (__any_sync(0xffffffffu, rescale)) {
        // The previous P V has retired (waited below), so O is stable in TMEM.
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tO + lane_off + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x32(tO + lane_off + c * 32, o);
        }
        tmem_st_wait();
      }
      const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
      float rs = 0.f;
      uint8_t* prow = base + L::P;
      if (!drop) {
#pragma unroll
        for (int ch = 0; ch < FK / 8; ++ch) {
          if (ch * 8 < n16) {
            float e8[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              const int c = ch * 8 + t;
              e8[t] = ex2(fmaf(__uint_as_float(r[c >> 5][c & 31]), sl2, neg_m));
              rs += e8[t];
            }
            store_chunk_sw128(prow + (ch >> 3) * kSub128, row, ch & 7,
                              make_uint4(pack2(e8[0], e8[1]), pack2(e8[2], e8[3]), pack2(e8[4], e8[5]),
                                         pack2(e8[6], e8[7])));
          }
        }
      } else {
        const float dscale = dr.scale;
#pragma unroll
        for (int ch = 0; ch < FK / 8; ++ch) {
          if (ch * 8 < n16) {
            float e8[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              const int c = ch * 8 + t;
              const float e = ex2(fmaf(__uint_as_float(r[c >> 5][c & 31]), sl2, neg_m));
              rs += e;  // the normaliser uses the probabilities before dropout
              const uint64_t bit = c < 64 ? (keep_lo >> c) : (keep_hi >> (c - 64));
              e8[t] = (bit & 1ull) ? e * dscale : 0.f;
            }
            store_chunk_sw128(prow + (ch >> 3) * kSub128, row, ch & 7,
                              make_uint4(pack2(e8[0], e8[1]), pack2(e8[2], e8[3]), pack2(e8[4], e8[5]),
                                         pack2(e8[6], e8[7])));
          }
        }
      }
      l_run += rs;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    if (tid == 0) {
      tc_fence_after();
      ok0 = mbar_wait(&bars[kBarV], static_cast<uint32_t>(v_waited & 1), p.timeout_ns);
      if (ok0) {
        ++v_waited;
        for (int kk = 0; kk < n16 / 16; ++kk) {
          const uint32_t a_off = (kk >> 2) * kSub128 + (kk & 3) * 32;
          umma_f16_ss(tO, smem_desc_sw128(sP + a_off, 16, 1024), smem_desc_sw128(sV + kk * 2048, L::KSUB, 1024),
                      IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars[kBarO]);
        ok0 = mbar_wait(&bars[kBarO], ph, p.timeout_ns);
      }
      if (!ok0) report_status(p.status, kStatusTimeoutMma);
      // P V has retired: V (and P) are free.
      if (ok0 && j + 1 < nblk) {
        mbar_arrive_expect_tx(&bars[kBarV], DS * L::KSUB);
        for (int s = 0; s < DS; ++s)
          tma_load_2d(base + L::V + s * L::KSUB, &tmV, &bars[kBarV], kvh * D + 64 * s, start + k0 + FK);
        ++v_issued;
      }
    }
    if (__syncthreads_or(!ok0)) {
      ok = false;
      break;
    }
    tc_fence_after();
  }

  __syncwarp();
  if (ok && warp_live) {
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    __nv_bfloat16* orow = p.o + static_cast<int64_t>(start + i) * p.ldo + h * D;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t o[32];
      tmem_ld_32x32b_x32(tO + lane_off + c * 32, o);
      tmem_ld_wait();
      if (i < len) {
        uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float* f = reinterpret_cast<const float*>(o + q * 8);
          dst[q] = make_uint4(pack2(f[0] * inv, f[1] * inv), pack2(f[2] * inv, f[3] * inv),
                              pack2(f[4] * inv, f[5] * inv), pack2(f[6] * inv, f[7] * inv));
        }
      }
    }
    if (i < len)
      p.lse[static_cast<int64_t>(h) * p.total_tokens + start + i] = l_run > 0.f ? m_run + log2f(l_run) : INFINITY;
  }

  if (!ok && tid == 0) {
    // Unwind: no TMA write may still be landing and no MMA may still be
    // writing TMEM when the CTA releases them.
    if (q_waited == 0) drain_phase(&bars[kBarQ], 1, 0, p);
    drain_phase(&bars[kBarK], k_issued, k_waited, p);
    drain_phase(&bars[kBarV], v_issued, v_waited, p);
    if (mma_issued) {
      umma_commit(&bars[kBarDrain]);
      if (!mbar_wait(&bars[kBarDrain], 0, p.timeout_ns)) report_status(p.status, kStatusTimeoutDrain);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, L::TMEM_COLS);
}

// ==================================================================== backward
template <int D>
__global__ void __launch_bounds__(kThreads, D == 64 ? 2 : 1)
    attn_tc_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const Params p) {
  using L = BwdLayout<D>;
  constexpr int DS = L::DS;
  const int kvh = blockIdx.y, b = blockIdx.z;
  const int start = p.cu_seqlens[b];
  const int len = p.cu_seqlens[b + 1] - start;
  const int kt0 = blockIdx.x * BKT;
  if (kt0 >= len) return;
  const int kt_hi = min(len, kt0 + BKT);
  const int nk16 = (kt_hi - kt0 + 15) & ~15;  // key rows in use (the dQ MMA's K)
  // Queries that can see a key of this tile.
  int q_first = 0, q_end = len;
  if (p.causal) q_first = kt0;
  if (p.window >= 0) {
    q_first = max(q_first, kt0 - p.window);
    q_end = min(q_end, kt_hi + p.window);
  }
  const int nqb = q_end > q_first ? (q_end - q_first + BQB - 1) / BQB : 0;
  const int total_it = nqb * p.heads_per_kv;
  const int width_q = p.heads * D;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + L::BARS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  float* s_nlse = reinterpret_cast<float*>(base + L::LSE);   // -lse of the block's queries
  float* s_dvs = reinterpret_cast<float*>(base + L::DVEC);   // Dvec * scale
  float* s_diag = p.drel != nullptr ? reinterpret_cast<float*>(base + L::DIAG) : nullptr;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t sK = smem_u32(base + L::K), sV = smem_u32(base + L::V), sQ0 = smem_u32(base + L::Q),
                 sDO0 = smem_u32(base + L::DO), sDST = smem_u32(base + L::DST), sPT = smem_u32(base + L::PT);

  int kv_waited = 0;
  int qd_issued[2] = {0, 0}, qd_waited[2] = {0, 0};  // per Q/dO buffer
  auto issue_qd = [&](int it) {
    const int hq = kvh * p.heads_per_kv + it / nqb;
    const int q0 = q_first + (it % nqb) * BQB;
    const int buf = it & 1;
    uint64_t* bar = &bars[buf ? kBarQ1 : kBarQ];
    mbar_arrive_expect_tx(bar, 2 * DS * kSub64);
    for (int s = 0; s < DS; ++s) {
      tma_load_2d(base + L::Q + buf * L::QD_STRIDE + s * kSub64, &tmQ, bar, hq * D + 64 * s, start + q0);
      tma_load_2d(base + L::DO + buf * L::QD_STRIDE + s * kSub64, &tmDO, bar, hq * D + 64 * s, start + q0);
    }
    ++qd_issued[buf];
  };
  if (s_diag != nullptr)
    for (int t = tid; t < BKT + BQB; t += kThreads) s_diag[t] = 0.f;
  if (tid == 0) {
    for (int i = 0; i < kNumBars; ++i) mbar_init(&bars[i], 1);
    fence_mbarrier_init();
    if (total_it > 0) {
      mbar_arrive_expect_tx(&bars[kBarK], 2 * DS * kSub128);
      for (int s = 0; s < DS; ++s) {
        tma_load_2d(base + L::K + s * kSub128, &tmK, &bars[kBarK], kvh * D + 64 * s, start + kt0);
        tma_load_2d(base + L::V + s * kSub128, &tmV, &bars[kBarK], kvh * D + 64 * s, start + kt0);
      }
      issue_qd(0);
      if (total_it > 1) issue_qd(1);
    }
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + 64, tDV = tmem + 128, tDK = tmem + 128 + D, tDQ = tmem;
  const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
  const int krow = warp * 32 + lane;
  const int key = kt0 + krow;  // this thread's key (sequence-relative)
  const bool warp_live = kt0 + warp * 32 < len;
  constexpr uint32_t IDESC_KV = idesc_bf16_f32(128, D, false, true);
  constexpr uint32_t IDESC_Q = idesc_bf16_f32(128, D, true, true);
  const float sl2 = p.scale_log2, scale = p.scale;
  // Queries that may see this key: [vis_lo, vis_hi) (empty past the sequence end).
  int vis_lo = 0, vis_hi = key < len ? len : 0;
  if (p.causal) vis_lo = key;
  if (p.window >= 0) {
    vis_lo = max(vis_lo, key - p.window);
    vis_hi = min(vis_hi, key + p.window + 1);
  }
  const Drop8 dr = drop8(p.pdrop);
  const bool drop = dr.t8 != 0u;
  const bool general = drop || p.rel_lut != nullptr;

  bool ok = true, mma_issued = false;
  for (int it = 0; it < total_it; ++it) {
    const int hq = kvh * p.heads_per_kv + it / nqb;
    const int q0 = q_first + (it % nqb) * BQB;
    const uint32_t ph = static_cast<uint32_t>(it & 1);
    const int buf = it & 1;
    const uint32_t sQ = sQ0 + buf * L::QD_STRIDE, sDO = sDO0 + buf * L::QD_STRIDE;
    const int nq16 = (min(BQB, q_end - q0) + 15) & ~15;  // query columns in use
    if (tid < BQB) {
      const int q = q0 + tid;
      const int64_t at = static_cast<int64_t>(hq) * p.total_tokens + start + q;
      s_nlse[tid] = q < len ? -p.lse[at] : -INFINITY;
      s_dvs[tid] = q < len ? p.dvec[at] * scale : 0.f;
    }
    bool ok0 = true;
    if (tid == 0) {
      if (it == 0) {
        ok0 = mbar_wait(&bars[kBarK], 0, p.timeout_ns);
        kv_waited = ok0 ? 1 : 0;
      }
      if (ok0) {
        ok0 = mbar_wait(&bars[buf ? kBarQ1 : kBarQ], static_cast<uint32_t>(qd_waited[buf] & 1), p.timeout_ns);
        if (ok0) ++qd_waited[buf];
      }
      if (ok0) {
        tc_fence_after();
        const uint32_t idesc_s = idesc_bf16_f32(128, nq16, false, false);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off128 = (kk >> 2) * kSub128 + (kk & 3) * 32;
          const uint32_t off64 = (kk >> 2) * kSub64 + (kk & 3) * 32;
          umma_f16_ss(tS, smem_desc_sw128(sK + off128, 16, 1024), smem_desc_sw128(sQ + off64, 16, 1024), idesc_s,
                      kk > 0 ? 1u : 0u);
          umma_f16_ss(tDP, smem_desc_sw128(sV + off128, 16, 1024), smem_desc_sw128(sDO + off64, 16, 1024), idesc_s,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars[kBarS]);
        mma_issued = true;
      }
    }
    // Dropout keep bits depend only on coordinates: draw them while the
    // S^T / dP^T MMAs are in flight.
    uint64_t keep = ~0ull;
    __syncwarp();
    if (drop && warp_live) keep = bwd_keep_bits(p.pdrop, dr.t8, start, key, hq, q0, nq16, lane);
    if (tid == 0) {
      if (ok0) ok0 = mbar_wait(&bars[kBarS], ph, p.timeout_ns);
      if (!ok0) report_status(p.status, kStatusTimeoutMma);
    }
    // Also publishes this block's -lse / Dvec rows to every thread.
    if (__syncthreads_or(!ok0)) {
      ok = false;
      break;
    }
    tc_fence_after();

    uint8_t* pt = base + L::PT;
    uint8_t* dst = base + L::DST;
    __syncwarp();
    if (warp_live) {
      uint32_t rs[2][32], rd[2][32];
      tmem_ld_32x32b_x32(tS + lane_off, rs[0]);
      tmem_ld_32x32b_x32(tDP + lane_off, rd[0]);
      if (nq16 > 32) {
        tmem_ld_32x32b_x32(tS + lane_off + 32, rs[1]);
        tmem_ld_32x32b_x32(tDP + lane_off + 32, rd[1]);
      }
      tmem_ld_wait();
      const int clo = vis_lo - q0, chi = vis_hi - q0;  // visible query columns of this block
      if (!general) {
#pragma unroll
        for (int ch = 0; ch < BQB / 8; ++ch) {
          if (ch * 8 < nq16) {
            float pv[8], dv[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              const int c = ch * 8 + t;
              const float s = __uint_as_float(rs[c >> 5][c & 31]);
              const float dp = __uint_as_float(rd[c >> 5][c & 31]);
              const float pr = (c >= clo && c < chi) ? ex2(fmaf(s, sl2, s_nlse[c])) : 0.f;
              pv[t] = pr;
              dv[t] = pr * fmaf(dp, scale, -s_dvs[c]);  // P (dP - Dvec) * scale
            }
            store_chunk_sw128(pt, krow, ch, make_uint4(pack2(pv[0], pv[1]), pack2(pv[2], pv[3]),
                                                       pack2(pv[4], pv[5]), pack2(pv[6], pv[7])));
            store_chunk_sw128(dst, krow, ch, make_uint4(pack2(dv[0], dv[1]), pack2(dv[2], dv[3]),
                                                        pack2(dv[4], dv[5]), pack2(dv[6], dv[7])));
          }
        }
      } else {
        // Dropout and / or relative bias: dV uses the dropped probabilities and
        // dS = P * (mask * dP / (1 - p) - Dvec); the bias gradient is dS summed
        // along each diagonal.
        const float dscale = dr.scale;
        const float* lut_col =
            p.rel_lut == nullptr ? nullptr
                                 : p.rel_lut + static_cast<int64_t>(hq) * (2 * p.lut_len - 1) + (p.lut_len - 1) +
                                       (key - q0);  // bias of column c at lut_col[-c]
        const float inv_scale = 1.f / scale;
#pragma unroll
        for (int ch = 0; ch < BQB / 8; ++ch) {
          if (ch * 8 < nq16) {
            float pv[8], dv[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              const int c = ch * 8 + t;
              const bool vis = c >= clo && c < chi;
              float s = __uint_as_float(rs[c >> 5][c & 31]);
              if (vis && lut_col != nullptr) s += __ldg(lut_col - c) * inv_scale;
              const float pr = vis ? ex2(fmaf(s, sl2, s_nlse[c])) : 0.f;
              const bool kept = ((keep >> c) & 1ull) != 0ull;
              const float dp = kept ? __uint_as_float(rd[c >> 5][c & 31]) * dscale : 0.f;
              const float ds = pr * fmaf(dp, scale, -s_dvs[c]);
              pv[t] = kept ? pr * dscale : 0.f;
              dv[t] = ds;
              // diagonal key - q, offset so the tile's smallest (key kt0, query q0 + 63) is 0
              if (s_diag != nullptr && ds != 0.f) atomicAdd(s_diag + (krow - c + BQB - 1), ds * inv_scale);
            }
            store_chunk_sw128(pt, krow, ch, make_uint4(pack2(pv[0], pv[1]), pack2(pv[2], pv[3]),
                                                       pack2(pv[4], pv[5]), pack2(pv[6], pv[7])));
            store_chunk_sw128(dst, krow, ch, make_uint4(pack2(dv[0], dv[1]), pack2(dv[2], dv[3]),
                                                        pack2(dv[4], dv[5]), pack2(dv[6], dv[7])));
          }
        }
      }
    } else {
      // Keys past the sequence: zero rows (dS^T rows enter dQ = dS K).
#pragma unroll
      for (int ch = 0; ch < BQB / 8; ++ch) {
        store_chunk_sw128(pt, krow, ch, make_uint4(0u, 0u, 0u, 0u));
        store_chunk_sw128(dst, krow, ch, make_uint4(0u, 0u, 0u, 0u));
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (s_diag != nullptr) {
      // One global add per diagonal of the tile; the buffer is cleared for the next block.
      float* drel_h = p.drel + static_cast<int64_t>(hq) * (2 * p.lut_len - 1) + (p.lut_len - 1);
      for (int t = tid; t < BKT + BQB - 1; t += kThreads) {
        const float v = s_diag[t];
        if (v != 0.f) {
          atomicAdd(drel_h + (kt0 - (q0 + BQB - 1) + t), v);
          s_diag[t] = 0.f;
        }
      }
    }

    if (tid == 0) {
      tc_fence_after();
      for (int kk = 0; kk < nq16 / 16; ++kk) {
        const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
        umma_f16_ss(tDV, smem_desc_sw128(sPT + kk * 32, 16, 1024), smem_desc_sw128(sDO + kk * 2048, kSub64, 1024),
                    IDESC_KV, acc);
        umma_f16_ss(tDK, smem_desc_sw128(sDST + kk * 32, 16, 1024), smem_desc_sw128(sQ + kk * 2048, kSub64, 1024),
                    IDESC_KV, acc);
      }
      // dQ = dS K: A = dS (M = queries, MN-major view of dS^T; its second
      // 64-row chunk is the P^T buffer, whose output rows are ignored).
      for (int kk = 0; kk < nk16 / 16; ++kk) {
        umma_f16_ss(tDQ, smem_desc_sw128(sDST + kk * 2048, L::PT - L::DST, 1024),
                    smem_desc_sw128(sK + kk * 2048, kSub128, 1024), IDESC_Q, kk > 0 ? 1u : 0u);
      }
      umma_commit(&bars[kBarO]);
      ok0 = mbar_wait(&bars[kBarO], ph, p.timeout_ns);
      if (!ok0) report_status(p.status, kStatusTimeoutMma);
      // This block's Q and dO buffer is free: fetch block it + 2 into it (block
      // it + 1 was fetched one iteration ago and is landing in the other buffer).
      if (ok0 && it + 2 < total_it) issue_qd(it + 2);
    }
    if (__syncthreads_or(!ok0)) {
      ok = false;
      break;
    }
    tc_fence_after();
    __syncwarp();
    if (warp < BQB / 32) {
      const int q = q0 + warp * 32 + lane;
      float* dq = p.dq_acc + static_cast<int64_t>(start + q) * width_q + hq * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tDQ + lane_off + c * 32, o);
        tmem_ld_wait();
        // Only queries that can see this key tile have dS rows written this
        // iteration (q_end <= len).
        if (q < q_end) {
          float4* d4 = reinterpret_cast<float4*>(dq + c * 32);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            red_add_f4(d4 + e, make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]),
                                          __uint_as_float(o[4 * e + 2]), __uint_as_float(o[4 * e + 3])));
        }
      }
    }
    tc_fence_before();
  }

  __syncwarp();
  if (ok && warp_live) {
    const bool have = total_it > 0;
    __nv_bfloat16* dk_row = p.dk + static_cast<int64_t>(start + key) * p.ld_dk + kvh * D;
    __nv_bfloat16* dv_row = p.dv + static_cast<int64_t>(start + key) * p.ld_dv + kvh * D;
#pragma unroll 1
    for (int which = 0; which < 2; ++which) {
      const uint32_t t_acc = which == 0 ? tDK : tDV;
      __nv_bfloat16* out = which == 0 ? dk_row : dv_row;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (have) {
          tmem_ld_32x32b_x32(t_acc + lane_off + c * 32, o);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        if (key < len) {
          uint4* d = reinterpret_cast<uint4*>(out + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float* f = reinterpret_cast<const float*>(o + q * 8);
            d[q] = make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
          }
        }
      }
    }
  }

  if (!ok && tid == 0) {
    if (total_it > 0 && kv_waited == 0) drain_phase(&bars[kBarK], 1, 0, p);
    drain_phase(&bars[kBarQ], qd_issued[0], qd_waited[0], p);
    drain_phase(&bars[kBarQ1], qd_issued[1], qd_waited[1], p);
    if (mma_issued) {
      umma_commit(&bars[kBarDrain]);
      if (!mbar_wait(&bars[kBarDrain], 0, p.timeout_ns)) report_status(p.status, kStatusTimeoutDrain);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, L::TMEM_COLS);
}

template <typename Kernel>
void configure(Kernel kernel, uint32_t bytes, int device, bool (&done)[64]) {
  if (device < 0 || device >= 64 || !done[device]) {
    RX_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)));
    if (device >= 0 && device < 64) done[device] = true;
  }
}

}  // namespace tc

// ------------------------------------------------------------------- host side
namespace {
bool g_tc_enabled = true;
int* g_status[64] = {nullptr};
}  // namespace

bool tc_attention_enabled() { return g_tc_enabled; }
void set_tc_attention_enabled(bool on) { g_tc_enabled = on; }
void register_tc_status(int device, int* status) {
  if (device >= 0 && device < 64) g_status[device] = status;
}
int* tc_status_word(int device) { return (device >= 0 && device < 64) ? g_status[device] : nullptr; }

// Launch the tcgen05 forward for a filled parameter block (no dropout, no bias).
void tc_forward(Params p, int d, int64_t max_len, cudaStream_t st, int device) {
  p.status = (device >= 0 && device < 64) ? g_status[device] : nullptr;
  p.timeout_ns = kWaitBudgetNs;
  const int64_t T = p.total_tokens;
  const int kv_heads = p.heads / p.heads_per_kv;
  const CUtensorMap tq = make_tmap_2d_bf16(p.q, T, static_cast<int64_t>(p.heads) * d, p.ldq, 64, tc::FQ);
  const int fk = d == 64 ? tc::FK_FOR<64> : tc::FK_FOR<128>;
  const CUtensorMap tk = make_tmap_2d_bf16(p.k, T, static_cast<int64_t>(kv_heads) * d, p.ldk, 64, fk);
  const CUtensorMap tv = make_tmap_2d_bf16(p.v, T, static_cast<int64_t>(kv_heads) * d, p.ldv, 64, fk);
  dim3 grid(static_cast<unsigned>((max_len + tc::FQ - 1) / tc::FQ), p.heads, p.batch);
  if (d == 64) {
    static bool done[64] = {false};
    tc::configure(tc::attn_tc_fwd_kernel<64>, tc::FwdLayout<64>::BYTES, device, done);
    tc::attn_tc_fwd_kernel<64><<<grid, tc::kThreads, tc::FwdLayout<64>::BYTES, st>>>(tq, tk, tv, p);
  } else {
    static bool done[64] = {false};
    tc::configure(tc::attn_tc_fwd_kernel<128>, tc::FwdLayout<128>::BYTES, device, done);
    tc::attn_tc_fwd_kernel<128><<<grid, tc::kThreads, tc::FwdLayout<128>::BYTES, st>>>(tq, tk, tv, p);
  }
  RX_CUDA_CHECK(cudaGetLastError());
}

// Launch the tcgen05 backward (dq_acc zeroed and dvec computed by the caller).
void tc_backward(Params p, int d, int64_t max_len, cudaStream_t st, int device) {
  p.status = (device >= 0 && device < 64) ? g_status[device] : nullptr;
  p.timeout_ns = kWaitBudgetNs;
  const int64_t T = p.total_tokens;
  const int kv_heads = p.heads / p.heads_per_kv;
  const CUtensorMap tq = make_tmap_2d_bf16(p.q, T, static_cast<int64_t>(p.heads) * d, p.ldq, 64, tc::BQB);
  const CUtensorMap tdo = make_tmap_2d_bf16(p.dO, T, static_cast<int64_t>(p.heads) * d, p.ld_do, 64, tc::BQB);
  const CUtensorMap tk = make_tmap_2d_bf16(p.k, T, static_cast<int64_t>(kv_heads) * d, p.ldk, 64, tc::BKT);
  const CUtensorMap tv = make_tmap_2d_bf16(p.v, T, static_cast<int64_t>(kv_heads) * d, p.ldv, 64, tc::BKT);
  dim3 grid(static_cast<unsigned>((max_len + tc::BKT - 1) / tc::BKT), kv_heads, p.batch);
  if (d == 64) {
    static bool done[64] = {false};
    tc::configure(tc::attn_tc_bwd_kernel<64>, tc::BwdLayout<64>::BYTES, device, done);
    tc::attn_tc_bwd_kernel<64><<<grid, tc::kThreads, tc::BwdLayout<64>::BYTES, st>>>(tq, tk, tv, tdo, p);
  } else {
    static bool done[64] = {false};
    tc::configure(tc::attn_tc_bwd_kernel<128>, tc::BwdLayout<128>::BYTES, device, done);
    tc::attn_tc_bwd_kernel<128><<<grid, tc::kThreads, tc::BwdLayout<128>::BYTES, st>>>(tq, tk, tv, tdo, p);
  }
  RX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace attn
}  // namespace rx
