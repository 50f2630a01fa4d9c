// Allocation-free variant of the packed-attention backward (see rx_noalloc.h).
//
// It launches the same kernels as the regular entry point in attention.cu,
// but takes their two scratch buffers (the fp32 dQ accumulator and the
// rowsum(dO * O) vector) from a static device array compiled into this file,
// so the call performs no cudaMalloc, cudaFree or allocating library call.
#include <mutex>

#include "attention_kernels.cuh"
#include "rx_noalloc.h"

namespace {

// Scratch shared by every call on a device; lives until the process exits.
static __device__ __align__(256) unsigned char g_scratch[RX_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_lock;
void* g_scratch_ptr[kMaxDevices] = {nullptr};
// The CUDA error behind the calling thread's last RX_NOALLOC_CUDA_ERROR.
thread_local cudaError_t g_last_error = cudaSuccess;

int cuda_failed(cudaError_t e) {
  g_last_error = e;
  return RX_NOALLOC_CUDA_ERROR;
}

// Device address of g_scratch on the current device. In host code the name
// g_scratch is only a host-side stand-in, so the address must be looked up
// (once per device, with that device current) before a kernel may use it.
int scratch_address(void** out) {
  int device = 0;
  const cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return cuda_failed(e);
  if (device < 0 || device >= kMaxDevices) return RX_NOALLOC_BAD_ARGUMENT;
  std::lock_guard<std::mutex> guard(g_setup_lock);
  if (g_scratch_ptr[device] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t s = cudaGetSymbolAddress(&ptr, g_scratch);
    if (s != cudaSuccess) return cuda_failed(s);
    if (ptr == nullptr) return cuda_failed(cudaErrorInvalidSymbol);
    g_scratch_ptr[device] = ptr;
  }
  *out = g_scratch_ptr[device];
  return RX_NOALLOC_OK;
}

bool aligned16(const void* p, int64_t ld) {
  return p != nullptr && reinterpret_cast<uintptr_t>(p) % 16 == 0 && ld % 8 == 0;
}

}  // namespace

extern "C" int rx_attention_backward_noalloc(
    const void* dO, int64_t ld_do, const void* q, int64_t ld_q, const void* k, int64_t ld_k,
    const void* v, int64_t ld_v, const void* o, int64_t ld_o, const float* lse,
    const int* cu_seqlens, int batch, int total_tokens, int max_len, int heads, float scale,
    int causal, int window, void* dq, int64_t ld_dq, void* dk, int64_t ld_dk, void* dv,
    int64_t ld_dv, cudaStream_t stream) {
  using namespace rx::attn;
  if (batch < 0 || total_tokens < 0 || max_len < 0 || heads <= 0) return RX_NOALLOC_BAD_ARGUMENT;
  if (batch == 0 || total_tokens == 0 || max_len == 0) return RX_NOALLOC_OK;
  if (lse == nullptr || cu_seqlens == nullptr) return RX_NOALLOC_BAD_ARGUMENT;
  // Operand rows are read with 16-byte copies; gradient rows are written in
  // 4-byte (dK, dV) and 8-byte (dQ) pieces.
  if (!aligned16(q, ld_q) || !aligned16(k, ld_k) || !aligned16(v, ld_v) || !aligned16(dO, ld_do))
    return RX_NOALLOC_BAD_ARGUMENT;
  if (o == nullptr || ld_o % 2 != 0 || reinterpret_cast<uintptr_t>(o) % 4 != 0)
    return RX_NOALLOC_BAD_ARGUMENT;
  if (dq == nullptr || reinterpret_cast<uintptr_t>(dq) % 8 != 0 || ld_dq % 4 != 0)
    return RX_NOALLOC_BAD_ARGUMENT;
  if (dk == nullptr || dv == nullptr || ld_dk % 2 != 0 || ld_dv % 2 != 0 ||
      reinterpret_cast<uintptr_t>(dk) % 4 != 0 || reinterpret_cast<uintptr_t>(dv) % 4 != 0)
    return RX_NOALLOC_BAD_ARGUMENT;

  // Scratch layout: dQ accumulator [T, heads * 64] fp32, then (256-byte
  // aligned) rowsum(dO * O) [heads, T] fp32.
  const uint64_t width = static_cast<uint64_t>(heads) * 64;
  const uint64_t acc_bytes = static_cast<uint64_t>(total_tokens) * width * sizeof(float);
  const uint64_t dvec_offset = (acc_bytes + 255) / 256 * 256;
  const uint64_t dvec_bytes = static_cast<uint64_t>(heads) * total_tokens * sizeof(float);
  if (dvec_offset + dvec_bytes > RX_NOALLOC_SCRATCH_BYTES) return RX_NOALLOC_TOO_LARGE;

  // The scratch address is the current device's; the stream must run there too.
  int current = 0, stream_device = 0;
  cudaError_t e = cudaGetDevice(&current);
  if (e != cudaSuccess) return cuda_failed(e);
  e = cudaStreamGetDevice(stream, &stream_device);
  if (e != cudaSuccess) return cuda_failed(e);
  if (stream_device != current) return RX_NOALLOC_BAD_ARGUMENT;
  void* base = nullptr;
  const int setup = scratch_address(&base);
  if (setup != RX_NOALLOC_OK) return setup;
  float* dq_acc = static_cast<float*>(base);
  float* dvec = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + dvec_offset);

  Params p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.ldq = ld_q;
  p.ldk = ld_k;
  p.ldv = ld_v;
  p.lse = const_cast<float*>(lse);
  p.cu_seqlens = cu_seqlens;
  p.batch = batch;
  p.heads = heads;
  p.heads_per_kv = 1;
  p.total_tokens = total_tokens;
  p.scale = scale;
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  p.causal = causal ? 1 : 0;
  p.window = window;
  p.dO = static_cast<const __nv_bfloat16*>(dO);
  p.ld_do = ld_do;
  p.dvec = dvec;
  p.dq_acc = dq_acc;
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  p.ld_dk = ld_dk;
  p.ld_dv = ld_dv;

  // The previous call's contents are still in the array: clear the
  // accumulator (dvec is fully overwritten by its kernel).
  // Every launch goes through cudaLaunchKernel, whose return value is that
  // launch's own status: errors left by unrelated earlier work are neither
  // reported as this call's nor cleared.
  e = cudaMemsetAsync(dq_acc, 0, acc_bytes, stream);
  if (e != cudaSuccess) return cuda_failed(e);
  {
    const int64_t threads = 256;
    const int64_t warps = static_cast<int64_t>(total_tokens) * heads;
    const __nv_bfloat16* o_arg = static_cast<const __nv_bfloat16*>(o);
    const __nv_bfloat16* do_arg = p.dO;
    int t_arg = total_tokens, h_arg = heads, d_arg = 64;
    void* args[] = {&o_arg, &ld_o, &do_arg, &ld_do, &dvec, &t_arg, &h_arg, &d_arg};
    e = cudaLaunchKernel(reinterpret_cast<const void*>(&attn_dvec_kernel),
                         dim3(static_cast<unsigned>((warps * 32 + threads - 1) / threads)), dim3(threads), args, 0,
                         stream);
    if (e != cudaSuccess) return cuda_failed(e);
  }
  {
    void* args[] = {&p};
    e = cudaLaunchKernel(reinterpret_cast<const void*>(&attn_bwd_kernel<64, false>),
                         dim3((max_len + BN - 1) / BN, heads, batch), dim3(kThreads), args, bwd_smem_bytes<64>(),
                         stream);
    if (e != cudaSuccess) return cuda_failed(e);
  }
  {
    const int64_t n4 = static_cast<int64_t>(total_tokens) * static_cast<int64_t>(width) / 4;
    __nv_bfloat16* dq_arg = static_cast<__nv_bfloat16*>(dq);
    int t_arg = total_tokens, w_arg = static_cast<int>(width);
    void* args[] = {&dq_acc, &dq_arg, &ld_dq, &t_arg, &w_arg};
    e = cudaLaunchKernel(reinterpret_cast<const void*>(&attn_dq_convert_kernel),
                         dim3(static_cast<unsigned>((n4 + 255) / 256)), dim3(256), args, 0, stream);
    if (e != cudaSuccess) return cuda_failed(e);
  }
  return RX_NOALLOC_OK;
}

extern "C" int rx_noalloc_last_cuda_error(void) { return static_cast<int>(g_last_error); }

extern "C" const char* rx_noalloc_error_string(int code) {
  switch (code) {
    case RX_NOALLOC_OK: return "ok";
    case RX_NOALLOC_TOO_LARGE:
      return "problem needs more scratch than the library's static array holds (32 MiB)";
    case RX_NOALLOC_BAD_ARGUMENT:
      return "null pointer, negative size, misaligned tensor, or a stream of another device";
    case RX_NOALLOC_CUDA_ERROR: return "a CUDA call failed";
    default: return "unknown code";
  }
}
