// Host entry of the tcgen05 GEMM: argument checks, tile/split planning,
// TMA tensor maps, variant dispatch. The kernel itself is in gemm_kernel.cuh.
#include "gemm_kernel.cuh"

#include <algorithm>
#include <vector>

namespace rx {
void colsum_accumulate(const at::Tensor& x, at::Tensor& out);

// C = epilogue(alpha * A . B^T). Shapes: A is [M, K] (a_mn false) or [K, M]
// (a_mn true); B is [N, K] (b_mn false) or [K, N] (b_mn true); C is [M, N].
// `split_k` > 1 is allowed only with the atomic fp32 output mode; 0 picks a
// split automatically when the output has too few tiles to fill the GPU.
namespace {

struct GatherArgs {
  const std::vector<int64_t>* src;
  int64_t seg, off;
  at::Tensor ready;
};

void gemm_impl(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool a_mn, bool b_mn,
               int64_t epi, int64_t out_mode, double alpha,
               const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& aux_in,
               const c10::optional<at::Tensor>& aux_out,
               const c10::optional<at::Tensor>& residual, const at::Tensor& status,
               int64_t split_k, int64_t variant, int64_t drop_seed, int64_t drop_stream, double drop_p,
               const c10::optional<at::Tensor>& colsum, const GatherArgs* gather) {
  using namespace gemm;
  check_bf16(A, "A");
  check_bf16(B, "B");
  RX_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm operands must be matrices");
  RX_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1,
           "gemm operands must have unit inner stride");
  const int64_t M = C.size(0), N = C.size(1);
  const int64_t K = a_mn ? A.size(0) : A.size(1);
  RX_CHECK((a_mn ? A.size(1) : A.size(0)) == M, "A does not match C rows");
  RX_CHECK((b_mn ? B.size(1) : B.size(0)) == N, "B does not match C columns");
  RX_CHECK((b_mn ? B.size(0) : B.size(1)) == K, "A and B reduction sizes differ");
  RX_CHECK(M > 0 && N > 0 && K > 0, "empty gemm");
  RX_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm too large");
  if (out_mode == OUT_BF16) {
    check_bf16(C, "C");
    RX_CHECK(C.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0,
             "bf16 C must be 16-byte aligned with ldc % 8 == 0");
  } else {
    check_f32(C, "C");
    RX_CHECK(C.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(C.data_ptr()) % 16 == 0,
             "fp32 C must be 16-byte aligned with ldc % 4 == 0");
  }
  Params p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.C = C.data_ptr();
  p.ldc = C.stride(0);
  p.alpha = static_cast<float>(alpha);
  p.status = status_ptr(status);
  p.timeout_ns = kWaitBudgetNs;
  auto vec_ok = [](const at::Tensor& t) {
    return t.stride(1) == 1 && (t.dim() == 1 || t.stride(0) % 8 == 0) &&
           reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0;
  };
  if (epi & EPI_BIAS) {
    RX_CHECK(bias.has_value(), "bias epilogue needs a bias");
    check_bf16(*bias, "bias");
    RX_CHECK(bias->numel() == N && bias->is_contiguous() &&
                 reinterpret_cast<uintptr_t>(bias->data_ptr()) % 16 == 0,
             "bias must be a contiguous aligned [N] vector");
    p.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  if (epi & EPI_DGELU) {
    RX_CHECK(aux_in.has_value(), "GELU-backward epilogue needs the pre-activation");
    check_bf16(*aux_in, "aux_in");
    RX_CHECK(aux_in->size(0) == M && aux_in->size(1) == N && vec_ok(*aux_in), "bad aux_in");
    p.aux_in = reinterpret_cast<const __nv_bfloat16*>(aux_in->data_ptr());
    p.ld_aux_in = aux_in->stride(0);
  }
  if (epi & EPI_GELU) {
    RX_CHECK(aux_out.has_value(), "GELU epilogue needs a pre-activation output");
    check_bf16(*aux_out, "aux_out");
    RX_CHECK(aux_out->size(0) == M && aux_out->size(1) == N && vec_ok(*aux_out), "bad aux_out");
    p.aux_out = reinterpret_cast<__nv_bfloat16*>(aux_out->data_ptr());
    p.ld_aux_out = aux_out->stride(0);
  }
  if (epi & EPI_RESID) {
    RX_CHECK(residual.has_value(), "residual epilogue needs a residual");
    check_bf16(*residual, "residual");
    RX_CHECK(residual->size(0) == M && residual->size(1) == N && vec_ok(*residual),
             "bad residual");
    p.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    p.ld_res = residual->stride(0);
  }
  if (epi & EPI_DROP) {
    RX_CHECK(drop_p > 0.0 && drop_p < 1.0, "dropout probability must be in (0, 1)");
    p.drop = make_dropout_site(drop_seed, drop_stream, drop_p);
  }
  // variant: 1 = one CTA per 128x256 tile, 2 = CTA pair per 256x256 tile,
  // 0 = pair whenever there are at least 256 rows (with or without a fused gather).
  const bool pair = variant == 2 || (variant == 0 && M >= 256);
  if (gather != nullptr) {
    RX_CHECK(!a_mn && !b_mn, "the fused weight gather is a forward (K-major) GEMM");
    const int64_t world = static_cast<int64_t>(gather->src->size());
    RX_CHECK(world >= 1 && world <= kMaxGatherRanks, "gather: 1..", kMaxGatherRanks, " owners");
    RX_CHECK(B.is_contiguous() && K % 8 == 0 && gather->off % 8 == 0 && gather->seg % 8 == 0,
             "gather: contiguous [N, K] weight, K and flat offsets multiples of 8 elements");
    RX_CHECK(gather->off + N * K <= world * gather->seg, "gather: weight range beyond the shards");
    const int64_t chunks = (N + kGatherRows - 1) / kGatherRows;
    RX_CHECK(gather->ready.is_cuda() && gather->ready.scalar_type() == at::kInt && gather->ready.numel() >= chunks,
             "gather: ready must be CUDA int32 with one entry per ", kGatherRows, " weight rows");
    for (int64_t r = 0; r < world; ++r) {
      RX_CHECK(gather->src->at(r) % 16 == 0, "gather: shard pointers must be 16-byte aligned");
      p.g_src[r] = gather->src->at(r);
    }
    p.gather = 1;
    p.g_world = static_cast<int>(world);
    p.g_seg = gather->seg;
    p.g_off = gather->off;
    p.g_dst = reinterpret_cast<__nv_bfloat16*>(B.data_ptr());
    p.g_ready = gather->ready.data_ptr<int>();
    RX_CUDA_CHECK(cudaMemsetAsync(p.g_ready, 0, sizeof(int) * chunks,
                                  at::cuda::getCurrentCUDAStream(C.get_device()).stream()));
  }
  bool colsum_after = false;
  if (epi & EPI_COLSUM) {
    RX_CHECK(colsum.has_value() && colsum->numel() == N, "the column-sum epilogue needs an fp32 [N] accumulator");
    check_f32(*colsum, "colsum");
    p.colsum = colsum->data_ptr<float>();
    if (!pair) {  // only the tile-store epilogue sums columns; reduce afterwards instead
      epi &= ~EPI_COLSUM;
      colsum_after = true;
    }
  }
  constexpr int BN = 256;
  const int tile_m = pair ? 2 * BM : BM;
  p.m_tiles = static_cast<int>((M + tile_m - 1) / tile_m);
  p.n_tiles = static_cast<int>((N + BN - 1) / BN);
  p.kb_total = static_cast<int>((K + BK - 1) / BK);
  const int device = C.get_device();
  const int sms = num_sms(device);
  const int workers = pair ? sms / 2 : sms;
  int splits = 1;
  const int tiles = p.m_tiles * p.n_tiles;
  if (split_k == 0 && out_mode == OUT_F32_ATOMIC && tiles < workers) {
    // Wave-aware split: among splits that leave >= 4 k-blocks each, take the
    // one whose work units fill the persistent grid best (units / (waves *
    // workers)), preferring fewer splits on ties (less atomic traffic).
    double best = -1.0;
    const int max_splits = std::max(1, std::min(16, p.kb_total / 4));
    for (int s = 1; s <= max_splits; ++s) {
      const int units = tiles * s;
      const int waves = (units + workers - 1) / workers;
      const double eff = static_cast<double>(units) / (static_cast<double>(waves) * workers);
      if (eff > best + 1e-3) {
        best = eff;
        splits = s;
      }
    }
  } else if (split_k > 1) {
    RX_CHECK(out_mode == OUT_F32_ATOMIC, "split-K needs the atomic fp32 output mode");
    splits = static_cast<int>(std::min<int64_t>(split_k, p.kb_total));
  }
  p.kb_per_split = (p.kb_total + splits - 1) / splits;
  p.splits = (p.kb_total + p.kb_per_split - 1) / p.kb_per_split;
  p.num_units = tiles * p.splits;
  LaunchFn fn = nullptr;
  const int e = static_cast<int>(epi), o = static_cast<int>(out_mode);
  if (!a_mn && !b_mn) fn = pair ? pick_forward_pair(e, o) : pick_forward(e, o);
  else if (!a_mn && b_mn) fn = pair ? pick_dgrad_pair(e, o) : pick_dgrad(e, o);
  else if (a_mn && b_mn) fn = pair ? pick_wgrad_pair(e, o) : pick_wgrad(e, o);
  RX_CHECK(fn != nullptr, "unsupported gemm variant a_mn=", a_mn, " b_mn=", b_mn, " epi=", epi,
           " out=", out_mode);
  // A: K-major boxes [128 rows x 64 k]; MN-major boxes [64 k rows x 64 m].
  // B: K-major boxes [BN rows x 64 k] (half of the pair tile per CTA);
  //    MN-major boxes [64 k rows x 64 n].
  CUtensorMap ta = a_mn ? make_tmap_2d_bf16(A.data_ptr(), K, M, A.stride(0), 64, 64)
                        : make_tmap_2d_bf16(A.data_ptr(), M, K, A.stride(0), 64, BM);
  CUtensorMap tb = b_mn ? make_tmap_2d_bf16(B.data_ptr(), K, N, B.stride(0), 64, 64)
                        : make_tmap_2d_bf16(B.data_ptr(), N, K, B.stride(0), 64, pair ? BN / 2 : BN);
  const int grid = pair ? 2 * std::min(p.num_units, workers) : std::min(p.num_units, sms);
  c10::cuda::CUDAGuard guard(device);
  fn(ta, tb, p, grid, at::cuda::getCurrentCUDAStream(device).stream(), device);
  if (colsum_after) {
    at::Tensor out = *colsum;
    colsum_accumulate(C, out);
  }
}

}  // namespace

void gemm_tcgen05(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool a_mn, bool b_mn,
                  int64_t epi, int64_t out_mode, double alpha,
                  const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& aux_in,
                  const c10::optional<at::Tensor>& aux_out,
                  const c10::optional<at::Tensor>& residual, const at::Tensor& status,
                  int64_t split_k, int64_t variant, int64_t drop_seed, int64_t drop_stream, double drop_p,
                  const c10::optional<at::Tensor>& colsum) {
  gemm_impl(A, B, C, a_mn, b_mn, epi, out_mode, alpha, bias, aux_in, aux_out, residual, status, split_k, variant,
            drop_seed, drop_stream, drop_p, colsum, nullptr);
}

// Forward GEMM whose weight B is first assembled (inside the kernel) from its
// owners' shards: `B` is this GPU's full-copy view of the weight, `shard_ptrs`
// the bf16 shard base of every rank, `shard_numel` the flat elements per
// shard and `flat_offset` the weight's first flat element.
void gemm_gather(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, int64_t epi, int64_t out_mode,
                 double alpha, const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& aux_out,
                 const c10::optional<at::Tensor>& residual, const at::Tensor& status, int64_t drop_seed,
                 int64_t drop_stream, double drop_p, const std::vector<int64_t>& shard_ptrs, int64_t shard_numel,
                 int64_t flat_offset, const at::Tensor& ready, int64_t variant) {
  GatherArgs g{&shard_ptrs, shard_numel, flat_offset, ready};
  gemm_impl(A, B, C, false, false, epi, out_mode, alpha, bias, c10::nullopt, aux_out, residual, status, 0, variant,
            drop_seed, drop_stream, drop_p, c10::nullopt, &g);
}

}  // namespace rx
