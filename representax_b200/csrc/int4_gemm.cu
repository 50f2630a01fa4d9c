// INT4-weight GEMMs on tcgen05 with the dequantisation inside the main loop:
// no bf16 copy of a frozen QLoRA base weight ever reaches HBM.
//
//   forward  y  [T, N] = x  [T, K] . Wq^T   (+ bias [N]) (+ residual [T, N])
//   dgrad    dx [T, K] = dy [T, N] . Wq
//
// Wq [N, K] is the packed base weight (uint8 [N, ldp], column 2j in the low
// nibble and 2j + 1 in the high nibble of byte j, 4-bit two's complement) with
// one bf16 scale s[n] per row n. The forward multiplies the integer products by
// s[n] in fp32 in the epilogue (y = s[n] * sum_k x q, no rounding of q * s);
// dgrad contracts over n, so its B tile holds bf16(q[n, k] * s[n]), bit for
// bit the weight the dequantisation kernel writes.
//
// Structure (persistent, one CTA per SM):
//   warp 0     producer: per stage the 128 x 64 bf16 activation tile (TMA,
//              128-byte swizzle) and the packed weight bytes of the B tile (TMA
//              without swizzle into a staging buffer: 256 rows x 32 bytes for
//              the forward, 64 rows x 128 bytes for dgrad), one barrier;
//   warps 6-21 transform: expand the staged nibbles into the bf16 B tile in
//              the tensor core's 128-byte-swizzled layout (K-major rows for the
//              forward; MN-major 64 x 64 blocks for dgrad, where the
//              contraction runs over W's rows), then release the stage to the
//              MMA warp;
//   warp 1     TMEM owner (two 256-column fp32 accumulators) and MMA issuer
//              (M = 128, N = 256, K = 16 per instruction);
//   warps 2-5  epilogue: tcgen05.ld, row scale (forward), bias / residual (the
//              LoRA product), bf16.
// Nibble expansion: u = q + 8 (xor 0x8 per nibble); bytes u are placed under a
// 0x43 high byte, making the bf16 value 128 + u exactly; subtracting 136 gives
// q exactly (and one bf16 multiply gives bf16(q * s) for dgrad).
// Where this kernel pays: every M tile expands its B tiles again, so the
// expansion costs as much issue time as the MMAs; with many tokens a one-pass
// dequantisation plus the CTA-pair bf16 GEMM is faster (the host dispatch in
// models/adapters.py picks by token count), with few tokens the GEMM is bound
// by reading the weight and the packed 4-bit read wins.
// Every wait is bounded by %globaltimer and reports to the status word.
//
// Reference parity: `_unpack_int4_rows` and the quantized LoRA linear
// (src/representax/models/adapters.py:38-79, :158-182).
#include <algorithm>

#include "common.h"
#include "sm100.cuh"

namespace rx {
namespace w4 {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int kTileA = BM * BK * 2;  // 16 KB
constexpr int kTileB = BN * BK * 2;  // 32 KB
constexpr int kStaging = BN * BK / 2;  // 8 KB of packed nibbles
constexpr int kStage = kTileA + kTileB + kStaging;  // 56 KB
constexpr int kEpiWarps = 4, kXformWarps = 16;
constexpr int kXformThreads = 32 * kXformWarps;
constexpr int kThreads = 32 * (2 + kEpiWarps + kXformWarps);
constexpr size_t kSmem = 1024 + STAGES * kStage + 256;
constexpr int kTmemCols = 2 * BN;

struct Params {
  int M, N, K;  // output [M, N], contraction K
  int m_tiles, n_tiles, k_blocks, num_units;
  const uint16_t* scale;  // bf16 bits, one per weight row
  int w_rows;             // weight rows (the forward's N, dgrad's K)
  __nv_bfloat16* C;
  int64_t ldc;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;
  int64_t ldr;
  int* status;
  uint64_t timeout_ns;
};

__device__ __forceinline__ void xform_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kXformThreads) : "memory");
}
// Barrier of the transform warps that also returns whether any of them passed `flag`.
__device__ __forceinline__ bool xform_sync_any(bool flag) {
  uint32_t any;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, 1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(any)
      : "r"(static_cast<uint32_t>(flag)), "n"(kXformThreads)
      : "memory");
  return any != 0;
}

// 8 packed nibbles -> 8 bf16 values q (exact), times s2 when SCALED (16 bytes).
template <bool SCALED>
__device__ __forceinline__ uint4 expand8(uint32_t w, __nv_bfloat162 s2) {
  w ^= 0x88888888u;
  const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
  const uint32_t t0 = __byte_perm(lo, hi, 0x5140), t1 = __byte_perm(lo, hi, 0x7362);
  uint32_t o[4] = {__byte_perm(t0, 0x43u, 0x4140), __byte_perm(t0, 0x43u, 0x4342), __byte_perm(t1, 0x43u, 0x4140),
                   __byte_perm(t1, 0x43u, 0x4342)};
  const __nv_bfloat162 off = __floats2bfloat162_rn(136.f, 136.f);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&o[j]);
    v = __hsub2(v, off);
    if constexpr (SCALED) v = __hmul2(v, s2);
    o[j] = *reinterpret_cast<uint32_t*>(&v);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

template <bool DGRAD>
__global__ void __launch_bounds__(kThreads, 1)
    w4_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* raw = reinterpret_cast<uint64_t*>(base + STAGES * kStage);
  uint64_t* full = raw + STAGES;
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&raw[s], 1);
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 32 * kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_map(&tmA);
      tma_prefetch_map(&tmW);
      int stage = 0;
      uint32_t phase = 0, issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
        const int mt = u % p.m_tiles, nt = u / p.m_tiles;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (*abort_flag || !mbar_wait(&empty[stage], phase ^ 1, p.timeout_ns)) {
            report_status(p.status, kStatusTimeoutProducer);
            *abort_flag = 1;
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&raw[stage], kTileA + kStaging);
          uint8_t* st = base + stage * kStage;
          tma_load_2d(st, &tmA, &raw[stage], kb * BK, mt * BM);
          if constexpr (DGRAD)  // weight rows kb*64.. (contraction), bytes of columns nt*256..
            tma_load_2d(st + kTileA + kTileB, &tmW, &raw[stage], nt * (BN / 2), kb * BK);
          else  // weight rows nt*256.. (outputs), bytes of columns kb*64..
            tma_load_2d(st + kTileA + kTileB, &tmW, &raw[stage], kb * (BK / 2), nt * BN);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s)
        if (((issued_mask >> s) & 1u) && !mbar_wait(&raw[s], (issued_parity >> s) & 1u, p.timeout_ns))
          report_status(p.status, kStatusTimeoutDrain);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN, false, DGRAD);
      int stage = 0, local = 0;
      uint32_t phase = 0;
      bool ok = true, issued_any = false;
      for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (*abort_flag || !mbar_wait(&tempty[acc], acc_phase ^ 1, p.timeout_ns)) {
          report_status(p.status, kStatusTimeoutMma);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (*abort_flag || !mbar_wait(&full[stage], phase, p.timeout_ns)) {
            report_status(p.status, kStatusTimeoutMma);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(base + stage * kStage), b = a + kTileA;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t da = smem_desc_sw128(a + kk * 32, 16, 1024);
            const uint64_t db = DGRAD ? smem_desc_sw128(b + kk * 2048, 8192, 1024) : smem_desc_sw128(b + kk * 32, 16, 1024);
            umma_f16_ss(d_tmem, da, db, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
      }
      if (issued_any) {
        umma_commit(drain);
        if (!mbar_wait(drain, 0, p.timeout_ns)) report_status(p.status, kStatusTimeoutDrain);
      }
    }
  } else if (warp < 2 + kEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    int local = 0;
    for (int u = blockIdx.x; u < p.num_units; u += gridDim.x, ++local) {
      const int mt = u % p.m_tiles, nt = u / p.m_tiles;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      bool ok = (*abort_flag == 0) && mbar_wait(&tfull[acc], acc_phase, p.timeout_ns);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) report_status(p.status, kStatusTimeoutEpilogue);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int m = mt * BM + quad * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(t_row + c * 32, r);
        tmem_ld_wait();
        const int nb = nt * BN + c * 32;
        if (m >= p.M || nb >= p.N) continue;
        __nv_bfloat16* row = p.C + static_cast<int64_t>(m) * p.ldc + nb;
        const __nv_bfloat16* res = p.residual ? p.residual + static_cast<int64_t>(m) * p.ldr + nb : nullptr;
        if (nb + 32 <= p.N) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(r[8 * q + j]);
            if constexpr (!DGRAD) {  // forward: weight row scale of output column n
              const uint4 sw = *reinterpret_cast<const uint4*>(p.scale + nb + 8 * q);
              const __nv_bfloat162* s2 = reinterpret_cast<const __nv_bfloat162*>(&sw);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 f = __bfloat1622float2(s2[j]);
                v[2 * j] *= f.x;
                v[2 * j + 1] *= f.y;
              }
            }
            if (p.bias) {
              const uint4 bw = *reinterpret_cast<const uint4*>(p.bias + nb + 8 * q);
              const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&bw);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 f = __bfloat1622float2(b2[j]);
                v[2 * j] += f.x;
                v[2 * j + 1] += f.y;
              }
            }
            if (res) {
              const uint4 rw = *reinterpret_cast<const uint4*>(res + 8 * q);
              const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rw);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 f = __bfloat1622float2(r2[j]);
                v[2 * j] += f.x;
                v[2 * j + 1] += f.y;
              }
            }
            uint4 o;
            __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
            for (int j = 0; j < 4; ++j) o2[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
            *reinterpret_cast<uint4*>(row + 8 * q) = o;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {  // static indices keep r[] in registers
            if (nb + i >= p.N) continue;
            float v = __uint_as_float(r[i]);
            if constexpr (!DGRAD) v *= __bfloat162float(__ushort_as_bfloat16(p.scale[nb + i]));
            if (p.bias) v += __bfloat162float(p.bias[nb + i]);
            if (res) v += __bfloat162float(res[i]);
            row[i] = __float2bfloat16_rn(v);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  } else {
    // ------------------------------------------------------------ transform
    const int t = threadIdx.x - 32 * (2 + kEpiWarps);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < p.num_units; u += gridDim.x) {
      const int nt = u / p.m_tiles;
      for (int kb = 0; kb < p.k_blocks; ++kb) {
        const bool stop = *abort_flag != 0;
        const bool got = !stop && mbar_wait(&raw[stage], phase, p.timeout_ns);
        if (!stop && !got) report_status(p.status, kStatusTimeoutProducer);
        // one decision for all transform threads, so their named barriers stay matched
        if (xform_sync_any(!got)) {
          *abort_flag = 1;
          ok = false;
          break;
        }
        uint8_t* st = base + stage * kStage;
        const uint8_t* packed = st + kTileA + kTileB;
        uint8_t* btile = st + kTileA;
#pragma unroll
        for (int i = 0; i < 2048 / kXformThreads; ++i) {
          const int job = t + i * kXformThreads;  // 2048 jobs of 8 weights
          if constexpr (DGRAD) {
            // row kr of the contraction block (weight row), 8 columns c8 of 256
            const int kr = job >> 5, c = job & 31;
            const int wrow = kb * BK + kr;
            const float s = wrow < p.w_rows ? __bfloat162float(__ushort_as_bfloat16(p.scale[wrow])) : 0.f;
            const uint32_t w = *reinterpret_cast<const uint32_t*>(packed + kr * 128 + c * 4);
            const int blk = c >> 3, cc = c & 7;
            *reinterpret_cast<uint4*>(btile + blk * 8192 + kr * 128 + ((cc ^ (kr & 7)) << 4)) =
                expand8<true>(w, __floats2bfloat162_rn(s, s));
          } else {
            // weight row r of the tile, 8 contraction values c of 64; the row
            // scale is applied to the fp32 accumulator in the epilogue
            const int r = job >> 3, c = job & 7;
            const uint32_t w = *reinterpret_cast<const uint32_t*>(packed + r * 32 + c * 4);
            *reinterpret_cast<uint4*>(btile + r * 128 + ((c ^ (r & 7)) << 4)) =
                expand8<false>(w, __nv_bfloat162());
          }
        }
        fence_proxy_async_smem();
        xform_sync();
        if (t == 0) mbar_arrive(&full[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

}  // namespace w4

// Packed uint8 map without swizzle: boxes of box_cols bytes x box_rows rows.
static CUtensorMap make_tmap_packed(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_cols,
                                    int box_rows) {
  RX_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0 && ld % 16 == 0, "packed weight rows must be 16-byte aligned");
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t elem_strides[2] = {1, 1};
  CUresult r = encode_tiled_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                                 elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  RX_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (packed int4) failed with code ", static_cast<int>(r));
  return map;
}

// dgrad == false: out [T, N] = x [T, K] . Wq^T (+ bias) (+ residual);
// dgrad == true:  out [T, K] = x [T, N] . Wq (x is the output gradient).
// packed: uint8 [N, ldp >= K / 2]; scale_bits: 16-bit [N].
void int4_gemm(const at::Tensor& x, const at::Tensor& packed, const at::Tensor& scale_bits, int64_t in_features,
               at::Tensor& out, const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
               bool dgrad, const at::Tensor& status) {
  check_bf16(x, "x");
  check_bf16(out, "out");
  RX_CHECK(packed.is_cuda() && packed.scalar_type() == at::kByte && packed.dim() == 2 && packed.stride(1) == 1,
           "packed must be a CUDA uint8 matrix");
  const int64_t N = packed.size(0), K = in_features;
  RX_CHECK(K % 32 == 0 && packed.size(1) * 2 >= K, "in_features must be a multiple of 32 covered by packed");
  RX_CHECK(scale_bits.is_cuda() && scale_bits.numel() == N && scale_bits.is_contiguous() &&
               scale_bits.element_size() == 2 && reinterpret_cast<uintptr_t>(scale_bits.data_ptr()) % 16 == 0,
           "scale_bits must hold one 16-bit value per weight row, 16-byte aligned");
  const int64_t T = x.size(0);
  const int64_t Kc = dgrad ? N : K, Nout = dgrad ? K : N;
  RX_CHECK(x.dim() == 2 && x.size(1) == Kc && x.stride(1) == 1, "x has the wrong shape");
  RX_CHECK(out.dim() == 2 && out.size(0) == T && out.size(1) == Nout && out.stride(1) == 1 && out.stride(0) % 8 == 0 &&
               reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
           "out must be [T, out_features] with 16-byte aligned rows");
  RX_CHECK(!dgrad || (!bias.has_value() && !residual.has_value()), "dgrad takes no bias / residual");
  if (bias.has_value()) {
    check_bf16(*bias, "bias");
    RX_CHECK(bias->numel() == Nout && bias->is_contiguous() && Nout % 8 == 0 &&
                 reinterpret_cast<uintptr_t>(bias->data_ptr()) % 16 == 0,
             "bias must be a 16-byte aligned contiguous [N], N % 8 == 0");
  }
  if (residual.has_value()) {
    check_bf16(*residual, "residual");
    RX_CHECK(residual->size(0) == T && residual->size(1) == Nout && residual->stride(1) == 1 &&
                 residual->stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(residual->data_ptr()) % 16 == 0,
             "residual must be [T, N] with 16-byte aligned rows");
  }
  if (T == 0 || Nout == 0) return;
  c10::cuda::CUDAGuard guard(x.get_device());
  w4::Params p{};
  p.M = static_cast<int>(T);
  p.N = static_cast<int>(Nout);
  p.K = static_cast<int>(Kc);
  p.m_tiles = static_cast<int>((T + w4::BM - 1) / w4::BM);
  p.n_tiles = static_cast<int>((Nout + w4::BN - 1) / w4::BN);
  p.k_blocks = static_cast<int>((Kc + w4::BK - 1) / w4::BK);
  p.num_units = p.m_tiles * p.n_tiles;
  p.scale = reinterpret_cast<const uint16_t*>(scale_bits.data_ptr());
  p.w_rows = static_cast<int>(N);
  p.C = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldc = out.stride(0);
  p.bias = bias.has_value() ? reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr()) : nullptr;
  p.residual = residual.has_value() ? reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr()) : nullptr;
  p.ldr = residual.has_value() ? residual->stride(0) : 0;
  p.status = status_ptr(status);
  p.timeout_ns = kWaitBudgetNs;
  const CUtensorMap ta = make_tmap_2d_bf16(x.data_ptr(), T, Kc, x.stride(0), 64, w4::BM);
  // packed columns in bytes: K / 2 (only the first in_features / 2 bytes of a row are read)
  const CUtensorMap tw = dgrad ? make_tmap_packed(packed.data_ptr(), N, K / 2, packed.stride(0), w4::BN / 2, w4::BK)
                               : make_tmap_packed(packed.data_ptr(), N, K / 2, packed.stride(0), w4::BK / 2, w4::BN);
  const int dev = x.get_device();
  auto kern = dgrad ? w4::w4_gemm_kernel<true> : w4::w4_gemm_kernel<false>;
  static bool configured[2][64] = {};
  if (dev < 0 || dev >= 64 || !configured[dgrad][dev]) {
    RX_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(w4::kSmem)));
    if (dev >= 0 && dev < 64) configured[dgrad][dev] = true;
  }
  const int grid = std::max(1, std::min(p.num_units, num_sms(dev)));
  kern<<<grid, w4::kThreads, w4::kSmem, at::cuda::getCurrentCUDAStream().stream()>>>(ta, tw, p);
  RX_CUDA_CHECK(cudaGetLastError());
}

}  // namespace rx
