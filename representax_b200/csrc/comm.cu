// Peer-memory communication for one process per GPU on an NVLink/NVSwitch box.
//
//   * IPC buffers: memory allocated here with cudaMalloc, exported with
//     cudaIpcGetMemHandle, opened by every peer (peer access enabled lazily),
//     so kernels address every rank's buffer with plain loads and stores.
//   * signal_barrier: a one-CTA kernel; thread r stores this rank's epoch into
//     flag[me] of rank r's signal pad (st.release.sys), then waits (bounded by
//     %globaltimer) until every rank's flag in the local pad reaches the epoch
//     (ld.acquire.sys). A wait that runs out records kStatusTimeoutPeer.
//   * peer_sgemm: the fp32 tiled GEMM of the MNR objective with rank-segmented
//     operands: rows of B (or of an MN-major B) come from `seg_ptrs[row / seg]`
//     (fusing the all-gather of candidate embeddings into the GEMM's loads), and
//     rows of C can be written to `out_ptrs[row / seg] + slot * seg * ldc`
//     (fusing the reduce-scatter's send into the GEMM's stores).
//   * slot_reduce: sum of `world` equally shaped slots in fixed rank order
//     (the receive side of the reduce-scatter, deterministic).
//   * sharded AdamW: reduce-scatter of fp32 gradients (peer loads in rank
//     order) + global-norm partial, then clipped AdamW on the owned shard with
//     the updated fp32 master and bf16 compute copy stored into every rank.
//
// Reference parity: the SPMD all-gather / reduce-scatter of candidate
// embeddings (src/representax/tasks/retrieval/mnr.py:140-148) and gradient
// reduction (src/representax/train/sharding.py:441-492) that XLA inserts.
#include <cstring>
#include <vector>

#include "common.h"
#include "sm100.cuh"

namespace rx {
namespace comm {

__device__ __forceinline__ void st_release_sys(int* addr, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* addr) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// pads[r]: rank r's signal pad (int[world]); flag[me] written by rank `me`.
__global__ void signal_barrier_kernel(const int64_t* __restrict__ pads, int me, int world, int epoch,
                                      int* status, uint64_t timeout_ns) {
  const int t = threadIdx.x;
  if (t < world) {
    int* remote = reinterpret_cast<int*>(pads[t]);
    __threadfence_system();
    st_release_sys(remote + me, epoch);
  }
  __syncthreads();
  if (t < world) {
    const int* local = reinterpret_cast<const int*>(pads[me]);
    const uint64_t start = globaltimer_ns();
    while (ld_acquire_sys(local + t) < epoch) {
      if (globaltimer_ns() - start > timeout_ns) {
        report_status(status, kStatusTimeoutPeer);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
}

constexpr int TM = 128, TN = 128, TK = 8;
constexpr int kThreads = 256;

// C[M,N] (+)= alpha * sum_k A(m,k) B(n,k); B rows (n) live in segments of
// `seg_b` rows at seg_ptrs (B_MN false: [N rows, K]) or B is [K, N] with its
// N columns split in segments (B_MN true: each segment a [K, seg_b] block with
// leading dimension ldb). C rows optionally scattered to out_ptrs.
template <bool A_MN, bool B_MN, bool B_SEG_K, bool C_SCATTER>
__global__ void __launch_bounds__(kThreads)
    peer_sgemm_kernel(const float* __restrict__ A, int64_t lda, const int64_t* __restrict__ b_ptrs,
                      int seg_b, int64_t ldb, float* __restrict__ C, int64_t ldc,
                      const int64_t* __restrict__ c_ptrs, int seg_c, int c_slot, int M, int N, int K,
                      float alpha, bool accumulate) {
  __shared__ float As[2][TK][TM + 4];
  __shared__ float Bs[2][TK][TN + 4];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * TM, n0 = blockIdx.x * TN;
  const int tx = tid % 16, ty = tid / 16;

  // B element (n, k). Segments split the n index (B_SEG_K false) or the k
  // index (B_SEG_K true) across the rank pointers.
  auto bval = [&](int gn, int gk) -> float {
    if (B_SEG_K) {
      const float* base = reinterpret_cast<const float*>(b_ptrs[gk / seg_b]);
      const int r = gk % seg_b;
      return B_MN ? base[static_cast<int64_t>(r) * ldb + gn] : base[static_cast<int64_t>(gn) * ldb + r];
    }
    const float* base = reinterpret_cast<const float*>(b_ptrs[gn / seg_b]);
    const int r = gn % seg_b;
    return B_MN ? base[static_cast<int64_t>(gk) * ldb + r] : base[static_cast<int64_t>(r) * ldb + gk];
  };
  auto load = [&](int buf, int k0) {
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
        Bs[buf][kk][nn] = (gk < K && gn < N) ? bval(gn, gk) : 0.f;
      } else {
        const int nn = idx / TK, kk = idx % TK;
        const int gk = k0 + kk, gn = n0 + nn;
        Bs[buf][kk][nn] = (gk < K && gn < N) ? bval(gn, gk) : 0.f;
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
    float* row;
    if (C_SCATTER) {
      float* dst = reinterpret_cast<float*>(c_ptrs[gm / seg_c]);
      row = dst + (static_cast<int64_t>(c_slot) * seg_c + gm % seg_c) * ldc;
    } else {
      row = C + static_cast<int64_t>(gm) * ldc;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (gn >= N) continue;
      const float v = alpha * acc[i][j];
      row[gn] = accumulate ? row[gn] + v : v;
    }
  }
}

// out[i] (+)= sum_r slots[r * n + i], r = 0..world-1 in order.
__global__ void slot_reduce_kernel(const float* __restrict__ slots, int world, int64_t n, float* __restrict__ out,
                                   bool accumulate) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    float s = 0.f;
    for (int r = 0; r < world; ++r) s += slots[r * n + i];
    out[i] = accumulate ? out[i] + s : s;
  }
}

// Sharded optimizer, phase 1: shard[i] = sum_r grad_r[off + i] (peer loads in
// rank order) and norm_sq += sum shard^2.
__global__ void rs_grad_kernel(const int64_t* __restrict__ grad_ptrs, int world, int64_t off, int64_t n,
                               float* __restrict__ shard, double* __restrict__ norm_sq) {
  __shared__ float red[32];
  float s2 = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    float s = 0.f;
    for (int r = 0; r < world; ++r) s += reinterpret_cast<const float*>(grad_ptrs[r])[off + i];
    shard[i] = s;
    s2 += s * s;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s2;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    atomicAdd(norm_sq, t);
  }
}

// Phase 2: clipped AdamW on the owned shard; the new fp32 master and bf16
// compute values are stored into every rank's buffers (fused all-gather).
// master_ptrs[r] / copy_ptrs[r]: rank r's flat master / compute buffers;
// m / v hold only this rank's shard (indexed from 0). With FSDP (world = 1,
// the rank's own shard buffers, dst_off = off) nothing is pushed: the master
// and compute values stay in the owner's shard, which peers gather at use.
__global__ void adamw_shard_kernel(const float* __restrict__ shard_grad, int64_t off, int64_t n,
                                   const int64_t* __restrict__ master_ptrs, const int64_t* __restrict__ copy_ptrs,
                                   int world, int me, float* __restrict__ m, float* __restrict__ v,
                                   const float* __restrict__ scalars, float lr, float b1, float b2, float eps,
                                   float wd, int64_t dst_off) {
  if (scalars[1] == 0.f) return;  // non-finite step: nothing changes anywhere
  const float coef = scalars[0];
  const float step = scalars[2];
  const float bc1 = 1.f - powf(b1, step);
  const float bc2 = 1.f - powf(b2, step);
  const float* local = reinterpret_cast<const float*>(master_ptrs[me]);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int64_t gi = off + i - dst_off;
    const float g = shard_grad[i] * coef;
    const float mi = b1 * m[i] + (1.f - b1) * g;
    const float vi = b2 * v[i] + (1.f - b2) * g * g;
    m[i] = mi;
    v[i] = vi;
    const float p = local[gi];
    const float np = p - lr * ((mi / bc1) / (sqrtf(vi / bc2) + eps) + wd * p);
    const __nv_bfloat16 nb = __float2bfloat16_rn(np);
    for (int r = 0; r < world; ++r) {
      reinterpret_cast<float*>(master_ptrs[r])[gi] = np;
      if (copy_ptrs != nullptr) reinterpret_cast<__nv_bfloat16*>(copy_ptrs[r])[gi] = nb;
    }
  }
}

// FSDP: copy flat element ranges [lo, hi) of a buffer sharded over ranks
// (rank r holds [r * seg, (r + 1) * seg) at src[r]) into this GPU's full copy,
// 16 bytes (8 bf16) at a time from whichever rank owns each piece.
struct ShardSources {
  int64_t ptr[16];
};

__global__ void gather_ranges_kernel(ShardSources src, int64_t seg, const int64_t* __restrict__ ranges,
                                     __nv_bfloat16* __restrict__ dst) {
  const int64_t lo = ranges[2 * blockIdx.y], hi = ranges[2 * blockIdx.y + 1];
  const int64_t pieces = (hi - lo) >> 3;
  for (int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; q < pieces;
       q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = lo + (q << 3);
    const int64_t owner = e / seg;
    *reinterpret_cast<uint4*>(dst + e) =
        *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(src.ptr[owner]) + (e - owner * seg));
  }
}

}  // namespace comm

// --------------------------------------------------------------------- host API
int64_t ipc_malloc(int64_t nbytes, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void* ptr = nullptr;
  RX_CUDA_CHECK(cudaMalloc(&ptr, static_cast<size_t>(nbytes)));
  RX_CUDA_CHECK(cudaMemset(ptr, 0, static_cast<size_t>(nbytes)));
  return reinterpret_cast<int64_t>(ptr);
}

void ipc_free(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  RX_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr)));
}

at::Tensor ipc_handle(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t handle;
  RX_CUDA_CHECK(cudaIpcGetMemHandle(&handle, reinterpret_cast<void*>(ptr)));
  at::Tensor out = at::empty({static_cast<int64_t>(sizeof(handle))}, at::kByte);
  std::memcpy(out.data_ptr(), &handle, sizeof(handle));
  return out;
}

int64_t ipc_open(const at::Tensor& handle_bytes, int64_t device) {
  RX_CHECK(handle_bytes.numel() == static_cast<int64_t>(sizeof(cudaIpcMemHandle_t)), "bad IPC handle");
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t handle;
  std::memcpy(&handle, handle_bytes.cpu().data_ptr(), sizeof(handle));
  void* ptr = nullptr;
  RX_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, handle, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(ptr);
}

void ipc_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  RX_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

at::Tensor wrap_device_pointer(int64_t ptr, int64_t numel, int64_t dtype_code, int64_t device) {
  const auto dtype = dtype_code == 0 ? at::kFloat : (dtype_code == 1 ? at::kBFloat16 : at::kInt);
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, static_cast<c10::DeviceIndex>(device));
  return at::from_blob(reinterpret_cast<void*>(ptr), {numel}, [](void*) {}, opts);
}

void signal_barrier(const at::Tensor& pads, int64_t rank, int64_t world, int64_t epoch, const at::Tensor& status) {
  RX_CHECK(pads.scalar_type() == at::kLong && pads.is_cuda() && pads.numel() == world, "pads must be CUDA int64[world]");
  RX_CHECK(world <= 1024, "world too large");
  c10::cuda::CUDAGuard guard(pads.get_device());
  comm::signal_barrier_kernel<<<1, 32 * ((world + 31) / 32), 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      pads.data_ptr<int64_t>(), static_cast<int>(rank), static_cast<int>(world), static_cast<int>(epoch),
      status_ptr(status), kWaitBudgetNs);
  RX_CUDA_CHECK(cudaGetLastError());
}

void peer_sgemm(const at::Tensor& A, bool a_mn, const at::Tensor& b_ptrs, int64_t seg_b, int64_t ldb, bool b_mn,
                bool b_seg_k, int64_t M, int64_t N, int64_t K, at::Tensor& C, const c10::optional<at::Tensor>& c_ptrs,
                int64_t seg_c, int64_t c_slot, double alpha, bool accumulate) {
  check_f32(A, "A");
  RX_CHECK(b_ptrs.scalar_type() == at::kLong && b_ptrs.is_cuda(), "b_ptrs must be CUDA int64");
  RX_CHECK(A.stride(1) == 1, "A must have unit inner stride");
  if (M == 0 || N == 0) return;
  c10::cuda::CUDAGuard guard(A.get_device());
  dim3 grid((N + comm::TN - 1) / comm::TN, (M + comm::TM - 1) / comm::TM);
  auto st = at::cuda::getCurrentCUDAStream().stream();
  const bool scatter = c_ptrs.has_value();
  const int64_t* cp = scatter ? c_ptrs->data_ptr<int64_t>() : nullptr;
  float* cbase = scatter ? nullptr : C.data_ptr<float>();
  const int64_t ldc = scatter ? N : C.stride(0);
#define RX_PEER(AM, BM_, SK, SC)                                                                      \
  comm::peer_sgemm_kernel<AM, BM_, SK, SC><<<grid, comm::kThreads, 0, st>>>(                             \
      A.data_ptr<float>(), A.stride(0), b_ptrs.data_ptr<int64_t>(), static_cast<int>(seg_b), ldb, cbase, \
      ldc, cp, static_cast<int>(seg_c), static_cast<int>(c_slot), static_cast<int>(M),                \
      static_cast<int>(N), static_cast<int>(K), static_cast<float>(alpha), accumulate)
  // Variants used by the sharded MNR objective:
  //   S = Q D_all^T          A K-major, B rows split over ranks
  //   dQ = G D_all           A K-major, B MN-major with K split over ranks
  //   dD_all = G^T Q -> peers A MN-major, local B MN-major, C rows scattered
  if (!a_mn && !b_mn && !b_seg_k && !scatter) RX_PEER(false, false, false, false);
  else if (!a_mn && b_mn && b_seg_k && !scatter) RX_PEER(false, true, true, false);
  else if (a_mn && b_mn && !b_seg_k && scatter) RX_PEER(true, true, false, true);
  else RX_CHECK(false, "unsupported peer_sgemm variant");
#undef RX_PEER
  RX_CUDA_CHECK(cudaGetLastError());
}

void slot_reduce(const at::Tensor& slots, int64_t world, at::Tensor& out, bool accumulate) {
  check_f32(slots, "slots");
  check_f32(out, "out");
  const int64_t n = out.numel();
  RX_CHECK(slots.numel() >= world * n && out.is_contiguous() && slots.is_contiguous(), "slot shapes");
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(out.get_device());
  const int sms = num_sms(out.get_device());
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 8 * sms));
  comm::slot_reduce_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      slots.data_ptr<float>(), static_cast<int>(world), n, out.data_ptr<float>(), accumulate);
  RX_CUDA_CHECK(cudaGetLastError());
}

void sharded_grad_reduce(const at::Tensor& grad_ptrs, int64_t world, int64_t off, int64_t n, at::Tensor& shard,
                         at::Tensor& norm_sq) {
  RX_CHECK(grad_ptrs.scalar_type() == at::kLong && grad_ptrs.is_cuda(), "grad_ptrs must be CUDA int64");
  check_f32(shard, "shard");
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(shard.get_device());
  const int sms = num_sms(shard.get_device());
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 8 * sms));
  comm::rs_grad_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      grad_ptrs.data_ptr<int64_t>(), static_cast<int>(world), off, n, shard.data_ptr<float>(),
      norm_sq.data_ptr<double>());
  RX_CUDA_CHECK(cudaGetLastError());
}

void sharded_adamw(const at::Tensor& shard_grad, int64_t off, int64_t n, const at::Tensor& master_ptrs,
                   const c10::optional<at::Tensor>& copy_ptrs, int64_t world, int64_t rank, at::Tensor& exp_avg,
                   at::Tensor& exp_avg_sq, const at::Tensor& scalars, double lr, double b1, double b2, double eps,
                   double wd, int64_t dst_offset) {
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(shard_grad.get_device());
  const int sms = num_sms(shard_grad.get_device());
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 8 * sms));
  comm::adamw_shard_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      shard_grad.data_ptr<float>(), off, n, master_ptrs.data_ptr<int64_t>(),
      copy_ptrs.has_value() ? copy_ptrs->data_ptr<int64_t>() : nullptr, static_cast<int>(world),
      static_cast<int>(rank), exp_avg.data_ptr<float>(), exp_avg_sq.data_ptr<float>(), scalars.data_ptr<float>(), static_cast<float>(lr),
      static_cast<float>(b1), static_cast<float>(b2), static_cast<float>(eps), static_cast<float>(wd), dst_offset);
  RX_CUDA_CHECK(cudaGetLastError());
}

void gather_ranges(const std::vector<int64_t>& shard_ptrs, int64_t shard_numel, const at::Tensor& ranges,
                   at::Tensor& dst) {
  check_bf16(dst, "dst");
  RX_CHECK(ranges.is_cuda() && ranges.scalar_type() == at::kLong && ranges.dim() == 2 && ranges.size(1) == 2,
           "ranges must be CUDA int64 [n, 2]");
  RX_CHECK(!shard_ptrs.empty() && shard_ptrs.size() <= 16, "1..16 shards");
  RX_CHECK(shard_numel % 8 == 0 && dst.numel() >= static_cast<int64_t>(shard_ptrs.size()) * shard_numel,
           "shards must be 8-element multiples and dst must cover them");
  if (ranges.size(0) == 0) return;
  comm::ShardSources src{};
  for (size_t r = 0; r < shard_ptrs.size(); ++r) {
    RX_CHECK(shard_ptrs[r] % 16 == 0, "shard pointers must be 16-byte aligned");
    src.ptr[r] = shard_ptrs[r];
  }
  c10::cuda::CUDAGuard guard(dst.get_device());
  dim3 grid(64, static_cast<unsigned>(ranges.size(0)));
  comm::gather_ranges_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream().stream()>>>(
      src, shard_numel, ranges.data_ptr<int64_t>(), reinterpret_cast<__nv_bfloat16*>(dst.data_ptr()));
  RX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace rx
