/* Allocation-free attention backward: a C entry point of this library.
 *
 * This entry point has no counterpart in the reference project; it exists
 * for callers that cannot allocate device memory while they run, such as a
 * host program that owns a fixed memory pool and forbids cudaMalloc during a
 * step, or an embedding runtime that never links a device allocator. The
 * regular attention backward needs two scratch buffers (an fp32 dQ
 * accumulator and a per-row dot-product vector) that its caller allocates;
 * here they come from one static device array built into the library
 * instead, so the call itself allocates nothing.
 *
 * Limits and sharing:
 *   - The scratch array holds RX_NOALLOC_SCRATCH_BYTES (32 MiB) on every GPU
 *     that loads the library, from load until the process exits. A call needs
 *     total_tokens * heads * 65 * 4 bytes (256-byte aligned) and is rejected
 *     with RX_NOALLOC_TOO_LARGE beyond that (about 10,700 tokens at 12 heads).
 *   - Every call shares the one array and it keeps the last call's contents;
 *     the call clears the part that must start at zero itself. Calls whose
 *     work overlaps on the GPU (different streams, no ordering between them)
 *     race on the array and produce wrong gradients: order them.
 *   - The first call on each device looks up the array's device address with
 *     that device current; make that first call before any stream capture.
 *   - The array used is the current device's, so `stream` has to belong to
 *     the current device; a stream of another device is rejected with
 *     RX_NOALLOC_BAD_ARGUMENT.
 *   - Head dimension 64, heads == key/value heads, bf16 tensors, packed
 *     sequences delimited by cu_seqlens (int32, on the device).
 */
#ifndef RX_NOALLOC_H_
#define RX_NOALLOC_H_

#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RX_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

enum {
  RX_NOALLOC_OK = 0,
  RX_NOALLOC_TOO_LARGE = 1,    /* the problem needs more scratch than the array holds */
  RX_NOALLOC_BAD_ARGUMENT = 2, /* null pointer, bad size, misaligned tensor, or stream of another device */
  RX_NOALLOC_CUDA_ERROR = 3    /* a CUDA call failed; rx_noalloc_last_cuda_error() gives its cudaError_t */
};

/* dQ, dK, dV of packed multi-head attention given dO, the forward inputs q/k/v,
 * the forward output o and its base-2 log-sum-exp lse ([heads, total_tokens]
 * fp32). Row strides are in elements. Work is enqueued on `stream`; the
 * function returns once it is enqueued. */
int rx_attention_backward_noalloc(const void* dO, int64_t ld_do, const void* q, int64_t ld_q,
                                  const void* k, int64_t ld_k, const void* v, int64_t ld_v,
                                  const void* o, int64_t ld_o, const float* lse,
                                  const int* cu_seqlens, int batch, int total_tokens, int max_len,
                                  int heads, float scale, int causal, int window, void* dq,
                                  int64_t ld_dq, void* dk, int64_t ld_dk, void* dv, int64_t ld_dv,
                                  cudaStream_t stream);

/* Human-readable text of a return code. */
const char* rx_noalloc_error_string(int code);

/* The cudaError_t (as int) of the calling thread's last RX_NOALLOC_CUDA_ERROR.
 * The entry point never calls cudaGetLastError, so errors of other work stay
 * where they were. */
int rx_noalloc_last_cuda_error(void);

#ifdef __cplusplus
}
#endif

#endif /* RX_NOALLOC_H_ */
