// Host-side helpers shared by the extension's translation units: argument
// checks, TMA tensor-map construction through the driver entry point, and the
// per-call wait budget.
#pragma once

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstdint>

#define RX_CHECK(cond, ...) TORCH_CHECK(cond, "representax_b200: ", __VA_ARGS__)

#define RX_CUDA_CHECK(expr)                                                             \
  do {                                                                                  \
    cudaError_t _e = (expr);                                                            \
    TORCH_CHECK(_e == cudaSuccess, "representax_b200 CUDA error: ", cudaGetErrorString(_e), \
                " at ", __FILE__, ":", __LINE__);                                       \
  } while (0)

namespace rx {

// Budget for every bounded device-side wait (nanoseconds). Two seconds is far
// above any legitimate wait in these kernels and short enough that a stuck
// pipeline unwinds well inside a process-group timeout.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

inline void check_cuda(const at::Tensor& t, const char* name) {
  RX_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

inline void check_bf16(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  RX_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bfloat16");
}

inline void check_f32(const at::Tensor& t, const char* name) {
  check_cuda(t, name);
  RX_CHECK(t.scalar_type() == at::kFloat, name, " must be float32");
}

inline int* status_ptr(const at::Tensor& status) {
  RX_CHECK(status.is_cuda() && status.scalar_type() == at::kInt && status.numel() >= 1,
           "status must be a CUDA int32 tensor");
  return status.data_ptr<int>();
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* raw = nullptr;
    cudaDriverEntryPointQueryResult query;
    RX_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &raw, cudaEnableDefault,
                                          &query));
    RX_CHECK(query == cudaDriverEntryPointSuccess && raw != nullptr,
             "cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(raw);
  }
  return fn;
}

// Tensor map over a row-major 2-D bf16 matrix [rows, cols] with leading
// dimension `ld` elements, loaded in boxes of [box_rows, box_cols] with the
// 128-byte swizzle (box_cols * 2 must be 128).
inline CUtensorMap make_tmap_2d_bf16(const void* base, int64_t rows, int64_t cols, int64_t ld,
                                     int box_cols, int box_rows) {
  RX_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  RX_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes (ld % 8 == 0)");
  RX_CHECK(box_cols * 2 == 128, "128-byte swizzle needs 64-element boxes");
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t elem_strides[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                 const_cast<void*>(base), dims, strides, box, elem_strides,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  RX_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", static_cast<int>(r));
  return map;
}

// bf16 map for tile stores: boxes of 32 columns (64 bytes) x 32 rows with
// the 64-byte swizzle (16-byte chunk index XOR (row / 2) % 4).
inline CUtensorMap make_tmap_2d_bf16_store(const void* base, int64_t rows, int64_t cols, int64_t ld) {
  RX_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  RX_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes (ld % 8 == 0)");
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {32u, 32u};
  cuuint32_t elem_strides[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                                 box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                                 CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  RX_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (store) failed with code ", static_cast<int>(r));
  return map;
}

// 2-D tiled map of 8-bit elements with 128-byte rows per box (128 elements)
// and the 128-byte swizzle (the same shared-memory geometry as 64 bf16).
inline CUtensorMap make_tmap_2d_u8(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  RX_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  RX_CHECK(ld % 16 == 0, "8-bit TMA row stride must be a multiple of 16 elements");
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {128u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t elem_strides[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides,
                                 box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  RX_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", static_cast<int>(r));
  return map;
}

inline int num_sms(int device) {
  static int cached[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (cached[device] == 0) {
    int n = 0;
    RX_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
    cached[device] = n;
  }
  return cached[device];
}

}  // namespace rx
