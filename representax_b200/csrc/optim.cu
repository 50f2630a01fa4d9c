// Optimizer-step kernels over flat fp32 buffers (all trainable parameters,
// gradients and moments live in one contiguous buffer each):
//   grad_norm_sq   sum of squared gradients (fp64 accumulation across CTAs)
//   finalize_clip  global norm, clip coefficient min(1, max/(norm+1e-6)),
//                  finite gate over loss and norm, device-side step counter
//   adamw_step     clipped AdamW (Optax semantics: eps outside the sqrt,
//                  decoupled weight decay), skipped entirely when the step is
//                  not finite, with the bf16 compute copy refreshed in the
//                  same pass.
// Nothing here synchronises with the host: the gate and the step count stay
// on the device.
//
// Reference parity: global norm, clipping and the finite gate
// (src/representax/train/step.py:36-60, 346-410) around `optax.adamw`.
#include "common.h"
#include "sm100.cuh"

namespace rx {
namespace optim {

// scalars layout (fp32 device tensor):
//   [0] clip coefficient  [1] finite flag  [2] optimizer step count
//   [3] gradient norm     [4] skipped-step count
constexpr int kScalars = 8;

__global__ void grad_norm_sq_kernel(const float* __restrict__ g, int64_t n, double* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 4;
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < n; i += stride) {
    if (i + 3 < n) {
      const float4 v = *reinterpret_cast<const float4*>(g + i);
      s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    } else {
      for (int64_t j = i; j < n; ++j) s += g[j] * g[j];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    atomicAdd(out, t);
  }
}

__global__ void finalize_clip_kernel(const double* __restrict__ norm_sq, float* __restrict__ scalars,
                                     const float* __restrict__ loss, float max_norm,
                                     int step_offset) {
  const double nsq = norm_sq[0];
  const float norm = static_cast<float>(sqrt(nsq));
  const bool finite = isfinite(norm) && isfinite(loss[0]);
  float coef = 1.f;
  if (max_norm > 0.f && finite) coef = fminf(1.f, max_norm / (norm + 1e-6f));
  scalars[0] = coef;
  scalars[1] = finite ? 1.f : 0.f;
  if (finite) scalars[2] += static_cast<float>(step_offset);
  else scalars[4] += 1.f;
  scalars[3] = norm;
}

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g,
                             float* __restrict__ m, float* __restrict__ v,
                             __nv_bfloat16* __restrict__ copy, int64_t n,
                             const float* __restrict__ scalars, float lr, float b1, float b2,
                             float eps, float wd) {
  if (scalars[1] == 0.f) return;  // non-finite step: leave every buffer untouched
  const float coef = scalars[0];
  const float step = scalars[2];
  const float bc1 = 1.f - powf(b1, step);
  const float bc2 = 1.f - powf(b2, step);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float gi = g[i] * coef;
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    const float mhat = mi / bc1;
    const float vhat = vi / bc2;
    const float pi = p[i];
    const float upd = mhat / (sqrtf(vhat) + eps) + wd * pi;
    const float np = pi - lr * upd;
    p[i] = np;
    if (copy != nullptr) copy[i] = __float2bfloat16_rn(np);
  }
}

}  // namespace optim

void grad_norm_sq(const at::Tensor& grad, at::Tensor& out) {
  check_f32(grad, "grad");
  RX_CHECK(out.scalar_type() == at::kDouble && out.is_cuda(), "norm accumulator must be CUDA fp64");
  RX_CHECK(grad.is_contiguous(), "grad must be contiguous");
  c10::cuda::CUDAGuard guard(grad.get_device());
  auto st = at::cuda::getCurrentCUDAStream().stream();
  RX_CUDA_CHECK(cudaMemsetAsync(out.data_ptr(), 0, sizeof(double), st));
  const int64_t n = grad.numel();
  if (n == 0) return;
  const int sms = num_sms(grad.get_device());
  const int blocks = static_cast<int>(std::min<int64_t>((n / 4 + 255) / 256 + 1, 4 * sms));
  optim::grad_norm_sq_kernel<<<blocks, 256, 0, st>>>(grad.data_ptr<float>(), n, out.data_ptr<double>());
  RX_CUDA_CHECK(cudaGetLastError());
}

void finalize_clip(const at::Tensor& norm_sq, at::Tensor& scalars, const at::Tensor& loss,
                   double max_norm, int64_t step_offset) {
  check_f32(scalars, "scalars");
  check_f32(loss, "loss");
  RX_CHECK(scalars.numel() >= optim::kScalars, "scalars must hold 8 values");
  c10::cuda::CUDAGuard guard(scalars.get_device());
  optim::finalize_clip_kernel<<<1, 1, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      norm_sq.data_ptr<double>(), scalars.data_ptr<float>(), loss.data_ptr<float>(),
      static_cast<float>(max_norm), static_cast<int>(step_offset));
  RX_CUDA_CHECK(cudaGetLastError());
}

void adamw_step(const at::Tensor& param, const at::Tensor& grad, at::Tensor& exp_avg,
                at::Tensor& exp_avg_sq, const c10::optional<at::Tensor>& compute_copy,
                const at::Tensor& scalars, double lr, double beta1, double beta2, double eps,
                double weight_decay) {
  check_f32(param, "param");
  check_f32(grad, "grad");
  const int64_t n = param.numel();
  RX_CHECK(grad.numel() == n && exp_avg.numel() == n && exp_avg_sq.numel() == n, "optimizer buffer sizes differ");
  __nv_bfloat16* copy = nullptr;
  if (compute_copy.has_value() && compute_copy->numel() > 0) {
    check_bf16(*compute_copy, "compute_copy");
    RX_CHECK(compute_copy->numel() == n, "compute copy size differs");
    copy = reinterpret_cast<__nv_bfloat16*>(compute_copy->data_ptr());
  }
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(param.get_device());
  const int sms = num_sms(param.get_device());
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 8 * sms));
  optim::adamw_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      const_cast<float*>(param.data_ptr<float>()), grad.data_ptr<float>(), exp_avg.data_ptr<float>(),
      exp_avg_sq.data_ptr<float>(), copy, n, scalars.data_ptr<float>(), static_cast<float>(lr),
      static_cast<float>(beta1), static_cast<float>(beta2), static_cast<float>(eps),
      static_cast<float>(weight_decay));
  RX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace rx
