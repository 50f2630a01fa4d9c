// Packed INT4 weights -> bf16 (QLoRA base weights).
//
// Layout: uint8 [N, ceil(K / 2)] with column 2j in the low nibble and 2j + 1
// in the high nibble of byte j, 4-bit two's complement values in [-7, 7], and
// one bf16 scale per output row (passed as its uint16 bit pattern). Each
// thread expands 8 packed bytes (16 weights) into two 16-byte stores.
//
// Reference parity: `_unpack_int4_rows` (src/representax/models/adapters.py:38-79).
#include "common.h"

#include <algorithm>

namespace rx {
namespace int4 {

__device__ __forceinline__ float nib(uint32_t v) { return static_cast<float>(static_cast<int>(v << 28) >> 28); }

__global__ void dequant_kernel(const uint8_t* __restrict__ packed, int64_t ldp, const uint16_t* __restrict__ scale_bits,
                               __nv_bfloat16* __restrict__ out, int64_t ldo, int64_t rows, int64_t cols) {
  const int64_t groups = cols / 16;  // 16 output values per thread
  const int64_t n = rows * groups;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / groups, g = i % groups;
    const uint2 w = *reinterpret_cast<const uint2*>(packed + r * ldp + g * 8);
    const float s = __bfloat162float(__ushort_as_bfloat16(scale_bits[r]));
    uint32_t words[2] = {w.x, w.y};
    uint4 o[2];
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(o);
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const uint32_t byte = (words[b >> 2] >> (8 * (b & 3))) & 0xFFu;
      h[b] = __floats2bfloat162_rn(nib(byte & 0xFu) * s, nib(byte >> 4) * s);
    }
    uint4* dst = reinterpret_cast<uint4*>(out + r * ldo + g * 16);
    dst[0] = o[0];
    dst[1] = o[1];
  }
}

}  // namespace int4

void int4_dequantize(const at::Tensor& packed, const at::Tensor& scale_bits, at::Tensor& out) {
  RX_CHECK(packed.scalar_type() == at::kByte && packed.is_cuda() && packed.dim() == 2 && packed.stride(1) == 1,
           "packed must be a CUDA uint8 matrix");
  check_bf16(out, "out");
  const int64_t rows = out.size(0), cols = out.size(1);
  RX_CHECK(packed.size(0) == rows && packed.size(1) * 2 >= cols, "packed shape does not match");
  RX_CHECK(cols % 16 == 0, "int4 dequantization needs in_features % 16 == 0");
  RX_CHECK(scale_bits.numel() == rows && scale_bits.is_contiguous() && scale_bits.element_size() == 2,
           "scale_bits must hold one 16-bit value per row");
  RX_CHECK(packed.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(packed.data_ptr()) % 8 == 0, "packed alignment");
  RX_CHECK(out.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0, "out alignment");
  if (rows == 0) return;
  const int device = out.get_device();
  c10::cuda::CUDAGuard guard(device);
  const int64_t work = rows * (cols / 16);
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, 8 * num_sms(device))));
  int4::dequant_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream(device).stream()>>>(
      packed.data_ptr<uint8_t>(), packed.stride(0), reinterpret_cast<const uint16_t*>(scale_bits.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), rows, cols);
  RX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace rx
