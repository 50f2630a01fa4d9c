// Multiple-negatives ranking (MNR) objective kernels: an fp32 tiled GEMM for
// the cosine-similarity matrix and its two gradient products, and a row
// kernel that turns similarity rows into masked log-sum-exp, weighted
// cross-entropy row losses and the logit gradient in one pass.
//
// The similarity stays in fp32 end to end (the objective is precision
// sensitive and small next to the encoder).
//
// Reference parity: `_direction_row_terms` and the query-balanced reduction in
// src/representax/tasks/retrieval/mnr.py:123-158, 315-379.
#include "common.h"
#include "sm100.cuh"

namespace rx {
namespace mnr {

constexpr int TM = 128, TN = 128, TK = 8;
constexpr int kThreads = 256;

// C[M,N] (+)= alpha * sum_k A(m,k) B(n,k). A is [M,K] (a_mn false) or [K,M];
// B is [N,K] (b_mn false) or [K,N]. 128x128 tile per CTA, 8x8 per thread.
template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads)
    sgemm_kernel(const float* __restrict__ A, int64_t lda, const float* __restrict__ B,
                 int64_t ldb, float* __restrict__ C, int64_t ldc, int M, int N, int K, float alpha,
                 bool accumulate) {
  __shared__ float As[2][TK][TM + 4];
  __shared__ float Bs[2][TK][TN + 4];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  const int tx = tid % 16, ty = tid / 16;

  auto load = [&](int buf, int k0) {
    // 1024 elements per operand tile, 4 per thread.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + i * kThreads;
      if (A_MN) {
        const int kk = idx / TM, mm = idx % TM;
        const int gk = k0 + kk, gm = m0 + mm;
        As[buf][kk][mm] = (gk < K && gm < M) ? A[static_cast<int64_t>(gk) * lda + gm] : 0.f;
      } else {
        const int mm = idx / TK, kk = idx % TK;
        const int gk = k0 + kk, gm = m0 + mm;
        As[buf][kk][mm] = (gk < K && gm < M) ? A[static_cast<int64_t>(gm) * lda + gk] : 0.f;
      }
      if (B_MN) {
        const int kk = idx / TN, nn = idx % TN;
        const int gk = k0 + kk, gn = n0 + nn;
        Bs[buf][kk][nn] = (gk < K && gn < N) ? B[static_cast<int64_t>(gk) * ldb + gn] : 0.f;
      } else {
        const int nn = idx / TK, kk = idx % TK;
        const int gk = k0 + kk, gn = n0 + nn;
        Bs[buf][kk][nn] = (gk < K && gn < N) ? B[static_cast<int64_t>(gn) * ldb + gk] : 0.f;
      }
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  const int ktiles = (K + TK - 1) / TK;
  load(0, 0);
  __syncthreads();
  for (int kt = 0; kt < ktiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < ktiles) load(buf ^ 1, (kt + 1) * TK);
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[buf][kk][ty * 4 + i];
        a[4 + i] = As[buf][kk][64 + ty * 4 + i];
        b[i] = Bs[buf][kk][tx * 4 + i];
        b[4 + i] = Bs[buf][kk][64 + tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (gn >= N) continue;
      float* c = C + static_cast<int64_t>(gm) * ldc + gn;
      const float v = alpha * acc[i][j];
      *c = accumulate ? *c + v : v;
    }
  }
}

// One CTA per row i of `logits` (cosines, unscaled) [R, Cn]:
//   raw = scale * cos, logit = col_valid ? raw : -inf, lse = logsumexp(logit)
//   w   = weight * row_valid * col_valid, rw = sum_j w
//   row_loss = sum_j w (lse - raw) / max(rw, 1), row_active = row_valid & rw > 0
//   grad[i, j] = coef * active * scale * ((rw / max(rw,1)) softmax_j - w_j / max(rw,1))
// `coef` is a device scalar (upstream gradient / number of active rows).
__global__ void __launch_bounds__(256)
    mnr_rows_kernel(const float* __restrict__ logits, const float* __restrict__ weight,
                    const bool* __restrict__ row_valid, const bool* __restrict__ col_valid,
                    float* __restrict__ grad, float* __restrict__ row_loss,
                    float* __restrict__ row_active, int R, int Cn, float scale,
                    const float* __restrict__ coef) {
  __shared__ float red[32];
  __shared__ float bcast;
  const int i = blockIdx.x;
  const float* row = logits + static_cast<int64_t>(i) * Cn;
  const float* wrow = weight + static_cast<int64_t>(i) * Cn;
  const bool rv = row_valid[i];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;

  auto reduce = [&](float v, bool is_max) -> float {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float other = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, other) : v + other;
    }
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
      float r = red[0];
      for (int w = 1; w < nw; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];
      bcast = r;
    }
    __syncthreads();
    const float r = bcast;
    __syncthreads();
    return r;
  };

  float mx = -INFINITY;
  for (int j = threadIdx.x; j < Cn; j += blockDim.x)
    if (col_valid[j]) mx = fmaxf(mx, scale * row[j]);
  mx = reduce(mx, true);
  const float m_use = (mx == -INFINITY) ? 0.f : mx;
  float se = 0.f, rw = 0.f, wl = 0.f;
  for (int j = threadIdx.x; j < Cn; j += blockDim.x) {
    if (!col_valid[j]) continue;
    const float raw = scale * row[j];
    se += expf(raw - m_use);
    const float w = rv ? wrow[j] : 0.f;
    rw += w;
    wl -= w * raw;
  }
  se = reduce(se, false);
  rw = reduce(rw, false);
  wl = reduce(wl, false);
  const float lse = (mx == -INFINITY) ? -INFINITY : m_use + logf(se);
  const float denom = fmaxf(rw, 1.f);
  const bool active = rv && rw > 0.f;
  if (threadIdx.x == 0) {
    row_loss[i] = active ? (rw * lse + wl) / denom : 0.f;
    row_active[i] = active ? 1.f : 0.f;
  }
  if (grad != nullptr) {
    const float c = active ? coef[0] * scale : 0.f;
    float* grow = grad + static_cast<int64_t>(i) * Cn;
    for (int j = threadIdx.x; j < Cn; j += blockDim.x) {
      float gval = 0.f;
      if (active && col_valid[j]) {
        const float raw = scale * row[j];
        const float p = expf(raw - lse);
        gval = c * ((rw / denom) * p - wrow[j] / denom);
      }
      grow[j] = gval;
    }
  }
}

}  // namespace mnr

void sgemm(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, at::Tensor& C,
           double alpha, bool accumulate) {
  check_f32(A, "A");
  check_f32(B, "B");
  check_f32(C, "C");
  RX_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "unit inner stride required");
  const int M = static_cast<int>(C.size(0)), N = static_cast<int>(C.size(1));
  const int K = static_cast<int>(a_mn ? A.size(0) : A.size(1));
  RX_CHECK((a_mn ? A.size(1) : A.size(0)) == M, "A/C mismatch");
  RX_CHECK((b_mn ? B.size(1) : B.size(0)) == N, "B/C mismatch");
  RX_CHECK((b_mn ? B.size(0) : B.size(1)) == K, "A/B reduction mismatch");
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(C.get_device());
  dim3 grid((N + mnr::TN - 1) / mnr::TN, (M + mnr::TM - 1) / mnr::TM);
  auto st = at::cuda::getCurrentCUDAStream().stream();
#define RX_SGEMM(AM, BM_)                                                                          \
  mnr::sgemm_kernel<AM, BM_><<<grid, mnr::kThreads, 0, st>>>(                                     \
      A.data_ptr<float>(), A.stride(0), B.data_ptr<float>(), B.stride(0), C.data_ptr<float>(),    \
      C.stride(0), M, N, K, static_cast<float>(alpha), accumulate)
  if (!a_mn && !b_mn) RX_SGEMM(false, false);
  else if (!a_mn && b_mn) RX_SGEMM(false, true);
  else if (a_mn && !b_mn) RX_SGEMM(true, false);
  else RX_SGEMM(true, true);
#undef RX_SGEMM
  RX_CUDA_CHECK(cudaGetLastError());
}

void mnr_rows(const at::Tensor& logits, const at::Tensor& weight, const at::Tensor& row_valid,
              const at::Tensor& col_valid, at::Tensor& grad, at::Tensor& row_loss,
              at::Tensor& row_active, double scale, const at::Tensor& coef) {
  check_f32(logits, "logits");
  check_f32(weight, "weight");
  RX_CHECK(logits.is_contiguous() && weight.is_contiguous() && grad.is_contiguous(),
           "mnr tensors must be contiguous");
  RX_CHECK(row_valid.scalar_type() == at::kBool && col_valid.scalar_type() == at::kBool,
           "validity masks must be bool");
  const int R = static_cast<int>(logits.size(0)), Cn = static_cast<int>(logits.size(1));
  if (R == 0) return;
  c10::cuda::CUDAGuard guard(logits.get_device());
  mnr::mnr_rows_kernel<<<R, 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      logits.data_ptr<float>(), weight.data_ptr<float>(), row_valid.data_ptr<bool>(),
      col_valid.data_ptr<bool>(), grad.numel() ? grad.data_ptr<float>() : nullptr,
      row_loss.data_ptr<float>(), row_active.data_ptr<float>(), R, Cn, static_cast<float>(scale),
      coef.data_ptr<float>());
  RX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace rx
