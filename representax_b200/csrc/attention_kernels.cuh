// Shared declarations of the packed-attention kernels (defined in
// attention.cu): tile constants, the parameter block, and the kernel entry
// symbols, so more than one host entry point can launch the same kernels.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace rx {
namespace attn {

constexpr int D = 64;
constexpr int BM = 64;
constexpr int BN = 64;
constexpr int kThreads = 128;
constexpr int kChunks = D / 8;  // 16-byte chunks per row

struct Params {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t ldq, ldk, ldv;  // row strides in elements
  __nv_bfloat16* o;
  int64_t ldo;
  float* lse;  // [heads, T] base-2 log-sum-exp of the scaled scores
  const int* cu_seqlens;
  int batch, heads, heads_per_kv, total_tokens;
  float scale_log2;  // softmax_scale * log2(e)
  float scale;
  int causal;
  int window;  // -1: no window
  // backward
  const __nv_bfloat16* dO;
  int64_t ld_do;
  const float* dvec;  // [heads, T] rowsum(dO * O)
  float* dq_acc;      // [T, heads * D] fp32, pre-zeroed
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int64_t ld_dk, ld_dv;
};


__global__ void __launch_bounds__(kThreads) attn_fwd_kernel(const Params p);
__global__ void __launch_bounds__(kThreads) attn_bwd_kernel(const Params p);
__global__ void attn_dvec_kernel(const __nv_bfloat16* __restrict__ o, int64_t ldo,
                                 const __nv_bfloat16* __restrict__ dO, int64_t ld_do,
                                 float* __restrict__ dvec, int total, int heads);
__global__ void attn_dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq,
                                       int64_t ld_dq, int total, int width);

}  // namespace attn
}  // namespace rx
