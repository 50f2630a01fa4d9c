// Python bindings of the sm_100a extension `representax_b200._C`.
#include <torch/extension.h>

namespace rx {
void rope_forward(const at::Tensor& x, at::Tensor& y, const at::Tensor& pos, const c10::optional<at::Tensor>& axis_of,
                  const at::Tensor& inv_freq, int64_t heads, const c10::optional<at::Tensor>& norm_w, double eps);
void rope_backward(const at::Tensor& dy, at::Tensor& dx, const c10::optional<at::Tensor>& x, const at::Tensor& pos,
                   const c10::optional<at::Tensor>& axis_of, const at::Tensor& inv_freq, int64_t heads,
                   const c10::optional<at::Tensor>& norm_w, double eps, const c10::optional<at::Tensor>& dw);
void activation_forward(const at::Tensor& z, at::Tensor& y, int64_t act, bool gated);
void activation_backward(const at::Tensor& dy, const at::Tensor& z, at::Tensor& dz, int64_t act, bool gated);
void fp8_scale(const at::Tensor& x, at::Tensor& scale, at::Tensor& amax_scratch, bool e5m2);
void fp8_quantize(const at::Tensor& x, const at::Tensor& scale, at::Tensor& out, bool e5m2, bool transpose);
void gemm_fp8(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, int64_t a_fmt, int64_t b_fmt,
              int64_t epi, int64_t out_mode, double alpha, const at::Tensor& scales,
              const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
              const at::Tensor& status);
void int4_dequantize(const at::Tensor& packed, const at::Tensor& scale_bits, at::Tensor& out);
void int4_gemm(const at::Tensor& x, const at::Tensor& packed, const at::Tensor& scale_bits, int64_t in_features,
               at::Tensor& out, const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
               bool dgrad, const at::Tensor& status);
void dropout_apply(const at::Tensor& x, at::Tensor& y, int64_t seed, int64_t stream, double p,
                   const c10::optional<at::Tensor>& colsum);
void gemm_tcgen05(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, bool a_mn, bool b_mn,
                  int64_t epi, int64_t out_mode, double alpha,
                  const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& aux_in,
                  const c10::optional<at::Tensor>& aux_out,
                  const c10::optional<at::Tensor>& residual, const at::Tensor& status,
                  int64_t split_k, int64_t variant, int64_t drop_seed, int64_t drop_stream, double drop_p,
                  const c10::optional<at::Tensor>& colsum);
void norm_forward(const at::Tensor& x, const at::Tensor& gamma, const c10::optional<at::Tensor>& beta,
                  at::Tensor& y, const c10::optional<at::Tensor>& mean, at::Tensor& rstd,
                  double eps, bool rms);
void norm_backward(const at::Tensor& dy, const at::Tensor& x, const c10::optional<at::Tensor>& mean,
                   const at::Tensor& rstd, const at::Tensor& gamma, at::Tensor& dx,
                   const c10::optional<at::Tensor>& dgamma, const c10::optional<at::Tensor>& dbeta,
                   const c10::optional<at::Tensor>& dbias_prev, bool rms);
void embed_ln_forward(const at::Tensor& ids, const at::Tensor& pos_ids,
                      const c10::optional<at::Tensor>& type_ids, const at::Tensor& word,
                      const at::Tensor& pos, const at::Tensor& type, const at::Tensor& gamma,
                      const at::Tensor& beta, at::Tensor& y, at::Tensor& mean, at::Tensor& rstd,
                      double eps);
void embed_ln_backward(const at::Tensor& dy, const at::Tensor& ids, const at::Tensor& pos_ids,
                       const c10::optional<at::Tensor>& type_ids, const at::Tensor& word,
                       const at::Tensor& pos, const at::Tensor& type, const at::Tensor& gamma,
                       const at::Tensor& mean, const at::Tensor& rstd, at::Tensor& word_grad,
                       at::Tensor& pos_grad, at::Tensor& type_grad, at::Tensor& dgamma,
                       at::Tensor& dbeta, int64_t pad_id);
void attention_forward(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o,
                       at::Tensor& lse, const at::Tensor& cu_seqlens, int64_t max_len,
                       int64_t heads, int64_t kv_heads, double scale, bool causal, int64_t window,
                       int64_t drop_seed, int64_t drop_stream, double drop_p,
                       const c10::optional<at::Tensor>& rel_lut);
void attention_backward(const at::Tensor& dO, const at::Tensor& q, const at::Tensor& k,
                        const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse,
                        at::Tensor& dq, at::Tensor& dk, at::Tensor& dv, at::Tensor& dq_acc,
                        at::Tensor& dvec, const at::Tensor& cu_seqlens, int64_t max_len,
                        int64_t heads, int64_t kv_heads, double scale, bool causal,
                        int64_t window, int64_t drop_seed, int64_t drop_stream, double drop_p,
                        const c10::optional<at::Tensor>& rel_lut, const c10::optional<at::Tensor>& drel);
void attention_backward_bias(const at::Tensor& dO, const at::Tensor& q, const at::Tensor& k,
                             const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse,
                             at::Tensor& dq, at::Tensor& dk, at::Tensor& dv, at::Tensor& dq_acc,
                             at::Tensor& dvec, const at::Tensor& cu_seqlens, int64_t max_len,
                             int64_t heads, int64_t kv_heads, double scale, bool causal,
                             int64_t window, int64_t drop_seed, int64_t drop_stream, double drop_p,
                             const c10::optional<at::Tensor>& rel_lut, const c10::optional<at::Tensor>& drel,
                             const c10::optional<at::Tensor>& dbias_qkv);
void pool_forward(const at::Tensor& h, const at::Tensor& cu_seqlens, at::Tensor& out,
                  at::Tensor& norm, int64_t mode, bool normalize);
void pool_backward(const at::Tensor& dout, const at::Tensor& out, const at::Tensor& norm,
                   const at::Tensor& cu_seqlens, at::Tensor& dh, int64_t mode, bool normalize);
void colsum_accumulate(const at::Tensor& x, at::Tensor& out);
void sgemm(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, at::Tensor& C,
           double alpha, bool accumulate);
void mnr_rows(const at::Tensor& logits, const at::Tensor& positive_weight,
              const at::Tensor& row_valid, const at::Tensor& col_valid, at::Tensor& grad,
              at::Tensor& row_loss, at::Tensor& row_active, double scale,
              const at::Tensor& coef);
void adamw_step(const at::Tensor& param, const at::Tensor& grad, at::Tensor& exp_avg,
                at::Tensor& exp_avg_sq, const c10::optional<at::Tensor>& compute_copy,
                const at::Tensor& scalars, double lr, double beta1, double beta2, double eps,
                double weight_decay);
void grad_norm_sq(const at::Tensor& grad, at::Tensor& out);
void finalize_clip(const at::Tensor& norm_sq, at::Tensor& scalars, const at::Tensor& loss,
                   double max_norm, int64_t step_offset);
void cast_bf16(const at::Tensor& src, at::Tensor& dst);
int64_t ipc_malloc(int64_t nbytes, int64_t device);
void ipc_free(int64_t ptr, int64_t device);
at::Tensor ipc_handle(int64_t ptr, int64_t device);
int64_t ipc_open(const at::Tensor& handle_bytes, int64_t device);
void ipc_close(int64_t ptr, int64_t device);
at::Tensor wrap_device_pointer(int64_t ptr, int64_t numel, int64_t dtype_code, int64_t device);
void signal_barrier(const at::Tensor& pads, int64_t rank, int64_t world, int64_t epoch, const at::Tensor& status);
void peer_sgemm(const at::Tensor& A, bool a_mn, const at::Tensor& b_ptrs, int64_t seg_b, int64_t ldb, bool b_mn,
                bool b_seg_k, int64_t M, int64_t N, int64_t K, at::Tensor& C, const c10::optional<at::Tensor>& c_ptrs,
                int64_t seg_c, int64_t c_slot, double alpha, bool accumulate);
void slot_reduce(const at::Tensor& slots, int64_t world, at::Tensor& out, bool accumulate);
void mnr_split(const at::Tensor& src, at::Tensor& hi, at::Tensor& lo);
void gemm_gather(const at::Tensor& A, const at::Tensor& B, at::Tensor& C, int64_t epi, int64_t out_mode,
                 double alpha, const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& aux_out,
                 const c10::optional<at::Tensor>& residual, const at::Tensor& status, int64_t drop_seed,
                 int64_t drop_stream, double drop_p, const std::vector<int64_t>& shard_ptrs, int64_t shard_numel,
                 int64_t flat_offset, const at::Tensor& ready, int64_t variant);
void gather_ranges(const std::vector<int64_t>& shard_ptrs, int64_t shard_numel, const at::Tensor& ranges,
                   at::Tensor& dst);
void mnr_tc_scores(const at::Tensor& rows, const std::vector<int64_t>& src_ptrs, int64_t src_rows, int64_t rank,
                   at::Tensor& a_hi, at::Tensor& a_lo, at::Tensor& b_hi, at::Tensor& b_lo, at::Tensor& ready,
                   at::Tensor& scores, double alpha, const at::Tensor& status);
void mnr_tc_gemm(const at::Tensor& a_hi, const at::Tensor& a_lo, bool a_mn, const at::Tensor& b_hi,
                 const at::Tensor& b_lo, bool b_mn, int64_t M, int64_t N, int64_t K,
                 const c10::optional<at::Tensor>& out, const std::vector<int64_t>& route_ptrs, int64_t route_seg,
                 int64_t route_off, int64_t ldc, double alpha, bool accumulate, const at::Tensor& status);
void mnr_tc_argmax(const at::Tensor& a_hi, const at::Tensor& a_lo, const at::Tensor& b_hi, const at::Tensor& b_lo,
                   at::Tensor& best, const c10::optional<at::Tensor>& valid, int64_t exclude_off,
                   const at::Tensor& status);
void mx_quantize(const at::Tensor& x, const c10::optional<at::Tensor>& q, const c10::optional<at::Tensor>& sf,
                 const c10::optional<at::Tensor>& qt, const c10::optional<at::Tensor>& sft, bool e5m2);
void mx_gemm(const at::Tensor& a, const at::Tensor& sfa, int64_t a_fmt, const at::Tensor& b, const at::Tensor& sfb,
             int64_t b_fmt, int64_t K, at::Tensor& out, int64_t out_mode, const c10::optional<at::Tensor>& bias,
             const c10::optional<at::Tensor>& residual, const at::Tensor& status);
void sharded_grad_reduce(const at::Tensor& grad_ptrs, int64_t world, int64_t off, int64_t n, at::Tensor& shard,
                         at::Tensor& norm_sq);
void sharded_adamw(const at::Tensor& shard_grad, int64_t off, int64_t n, const at::Tensor& master_ptrs,
                   const c10::optional<at::Tensor>& copy_ptrs, int64_t world, int64_t rank, at::Tensor& exp_avg,
                   at::Tensor& exp_avg_sq, const at::Tensor& scalars, double lr, double b1, double b2, double eps,
                   double wd, int64_t dst_offset);
}  // namespace rx

namespace rx {
namespace attn {
bool tc_attention_enabled();
void set_tc_attention_enabled(bool on);
void register_tc_status(int device, int* status);
bool ws_backward_enabled();
void set_ws_backward_enabled(bool on);
bool ws_forward_enabled();
void set_ws_forward_enabled(bool on);
}  // namespace attn
}  // namespace rx

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "representax_b200 sm_100a kernels";
  m.def("gemm", &rx::gemm_tcgen05, "tcgen05 GEMM with fused epilogue");
  m.def("norm_forward", &rx::norm_forward);
  m.def("norm_backward", &rx::norm_backward);
  m.def("embed_ln_forward", &rx::embed_ln_forward);
  m.def("embed_ln_backward", &rx::embed_ln_backward);
  m.def("attention_forward", &rx::attention_forward);
  m.def("attention_backward", &rx::attention_backward);
  m.def("attention_backward_bias", &rx::attention_backward_bias,
        "attention backward that also adds the column sums of dq | dk | dv into a QKV bias gradient");
  m.def("set_attention_tcgen05", &rx::attn::set_tc_attention_enabled,
        "route eligible attention calls (no dropout, no relative bias) to the tcgen05 kernels");
  m.def("attention_tcgen05_enabled", &rx::attn::tc_attention_enabled);
  m.def("set_attention_backward_ws", &rx::attn::set_ws_backward_enabled,
        "use the warp-specialised persistent tcgen05 backward for head dim 64 (default on)");
  m.def("attention_backward_ws_enabled", &rx::attn::ws_backward_enabled);
  m.def("set_attention_forward_ws", &rx::attn::set_ws_forward_enabled,
        "use the warp-specialised persistent tcgen05 forward for head dim 64");
  m.def("attention_forward_ws_enabled", &rx::attn::ws_forward_enabled);
  m.def("register_status_word", [](const at::Tensor& status) {
    TORCH_CHECK(status.is_cuda() && status.scalar_type() == at::kInt, "status must be CUDA int32");
    rx::attn::register_tc_status(status.get_device(), status.data_ptr<int>());
  }, "status word that kernels without a status argument report bounded-wait failures to");
  m.def("pool_forward", &rx::pool_forward);
  m.def("pool_backward", &rx::pool_backward);
  m.def("colsum_accumulate", &rx::colsum_accumulate);
  m.def("sgemm", &rx::sgemm);
  m.def("mnr_rows", &rx::mnr_rows);
  m.def("adamw_step", &rx::adamw_step);
  m.def("grad_norm_sq", &rx::grad_norm_sq);
  m.def("finalize_clip", &rx::finalize_clip);
  m.def("cast_bf16", &rx::cast_bf16);
  m.def("ipc_malloc", &rx::ipc_malloc);
  m.def("ipc_free", &rx::ipc_free);
  m.def("ipc_handle", &rx::ipc_handle);
  m.def("ipc_open", &rx::ipc_open);
  m.def("ipc_close", &rx::ipc_close);
  m.def("wrap_device_pointer", &rx::wrap_device_pointer);
  m.def("signal_barrier", &rx::signal_barrier);
  m.def("peer_sgemm", &rx::peer_sgemm);
  m.def("slot_reduce", &rx::slot_reduce);
  m.def("mnr_split", &rx::mnr_split, "fp32 -> (hi, lo) bf16 split");
  m.def("gemm_gather", &rx::gemm_gather, "forward tcgen05 GEMM with the FSDP weight gather fused in");
  m.def("gather_ranges", &rx::gather_ranges, "copy flat [lo, hi) ranges of a sharded bf16 buffer into a full copy");
  m.def("mnr_tc_scores", &rx::mnr_tc_scores, "tcgen05 MNR scores with the candidate all-gather fused in");
  m.def("mnr_tc_gemm", &rx::mnr_tc_gemm, "tcgen05 split-bf16 GEMM, local or row-routed (peer) output");
  m.def("int4_gemm", &rx::int4_gemm, "tcgen05 GEMM with the packed INT4 weight expanded in the main loop");
  m.def("mx_quantize", &rx::mx_quantize, "MXFP8 quantiser: row-wise and / or transposed 8-bit data + UE8M0 scales");
  m.def("mx_gemm", &rx::mx_gemm, "tcgen05 block-scaled MXFP8 GEMM (kind::mxf8f6f4.block_scale)");
  m.def("mnr_tc_argmax", &rx::mnr_tc_argmax, "tcgen05 split-bf16 scores reduced to each row's hardest candidate");
  m.def("sharded_grad_reduce", &rx::sharded_grad_reduce);
  m.def("sharded_adamw", &rx::sharded_adamw);
  m.def("int4_dequantize", &rx::int4_dequantize);
  m.def("dropout_apply", &rx::dropout_apply);
  m.def("fp8_scale", &rx::fp8_scale);
  m.def("fp8_quantize", &rx::fp8_quantize);
  m.def("gemm_fp8", &rx::gemm_fp8);
  m.def("rope_forward", &rx::rope_forward);
  m.def("rope_backward", &rx::rope_backward);
  m.def("activation_forward", &rx::activation_forward);
  m.def("activation_backward", &rx::activation_backward);
}
