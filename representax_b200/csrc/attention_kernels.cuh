// Shared declarations of the packed-attention kernels (defined in
// attention.cu): tile constants, the parameter block, and the kernel entry
// symbols, so more than one host entry point can launch the same kernels.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "philox.cuh"

namespace rx {
namespace attn {

// Head dimension D (64 or 128) is a template parameter of the kernels.
constexpr int BM = 64;
constexpr int BN = 64;
constexpr int kThreads = 128;

// Dynamic shared memory: forward Q + 2 x (K, V); backward K, V, Q, dO, dS^T.
template <int D>
constexpr int fwd_smem_bytes() { return 5 * 64 * D * 2; }
template <int D>
constexpr int bwd_smem_bytes() { return 4 * 64 * D * 2 + 64 * 64 * 2; }

struct Params {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t ldq, ldk, ldv;  // row strides in elements
  __nv_bfloat16* o;
  int64_t ldo;
  float* lse;  // [heads, T] base-2 log-sum-exp of the scaled scores
  const int* cu_seqlens;
  int batch, heads, heads_per_kv, total_tokens;  // heads = query heads
  float scale_log2;  // softmax_scale * log2(e)
  float scale;
  int causal;
  int window;  // -1: no window
  // Attention-probability dropout (threshold 0 = off). Element (query i,
  // key j) of head h in a sequence starting at token `start` uses word
  // (i & 1) * 2 + (j & 1) of Philox block (start + (i & ~1), h << 16 | j >> 1):
  // 2 x 2 blocks, so the forward (row-major) and backward (transposed) tiles
  // both use two words of every block they generate.
  DropoutSite pdrop;
  // Relative position bias (MPNet): logits[h, i, j] += rel_lut[h, j - i + lut_len - 1]
  // (fp32 [heads, 2 * lut_len - 1]); the backward adds dS into drel (same shape).
  const float* rel_lut;
  float* drel;
  int lut_len;
  // backward
  const __nv_bfloat16* dO;
  int64_t ld_do;
  const float* dvec;  // [heads, T] rowsum(dO * O)
  float* dq_acc;      // [T, heads * D] fp32, pre-zeroed
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int64_t ld_dk, ld_dv;
  // Optional fp32 [heads * D + 2 * kv_heads * D] accumulator of the column
  // sums of (dQ | dK | dV): the gradient of a fused QKV projection's bias.
  float* dbias_qkv;
  // Bounded waits of the tcgen05 kernels (attention_tc.cu): error word and budget.
  int* status;
  uint64_t timeout_ns;
};


// Four forward CTAs per SM at head dim 64 (<= 128 registers per thread).
template <int D>
__global__ void __launch_bounds__(kThreads, D == 64 ? 4 : 1) attn_fwd_kernel(const Params p);
// GQA: loop over the query heads of each key/value head (heads_per_kv > 1).
template <int D, bool GQA>
__global__ void __launch_bounds__(kThreads) attn_bwd_kernel(const Params p);
extern template __global__ void attn_fwd_kernel<64>(const Params p);
extern template __global__ void attn_fwd_kernel<128>(const Params p);
extern template __global__ void attn_bwd_kernel<64, false>(const Params p);
extern template __global__ void attn_bwd_kernel<128, false>(const Params p);
extern template __global__ void attn_bwd_kernel<64, true>(const Params p);
extern template __global__ void attn_bwd_kernel<128, true>(const Params p);
// dvec[h, t] = <dO[t, h, :], O[t, h, :]>, one warp per (t, h); D = 64 or 128.
__global__ void attn_dvec_kernel(const __nv_bfloat16* __restrict__ o, int64_t ldo,
                                 const __nv_bfloat16* __restrict__ dO, int64_t ld_do,
                                 float* __restrict__ dvec, int total, int heads, int head_dim);
__global__ void attn_dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq,
                                       int64_t ld_dq, int total, int width);
// dq = bf16(dq_acc) and, when colsum != nullptr, colsum[c] += sum_t dq[t, c].
__global__ void attn_dq_convert_colsum_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq,
                                              int64_t ld_dq, int total, int width, int slice,
                                              float* __restrict__ colsum);

}  // namespace attn
}  // namespace rx
