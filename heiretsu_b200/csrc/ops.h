// Declarations of every host entry point exported by the extension.
#pragma once
#include <torch/extension.h>

namespace hb {
int64_t read_and_clear_status(int64_t device);

void gemm(const at::Tensor& a, const at::Tensor& b, at::Tensor& c, int64_t N, int64_t epi, bool a_mn, bool b_mn,
          const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& aux,
          const c10::optional<at::Tensor>& resid, int64_t block_n, const std::vector<uint64_t>& ag_src,
          const c10::optional<at::Tensor>& ag_flags, int64_t ag_rank, int64_t ag_rows,
          const std::vector<uint64_t>& rs_dst, int64_t rs_rank, int64_t rs_rows, int64_t grp_mode,
          const c10::optional<at::Tensor>& grp_off, int64_t grp_n, int64_t grp_b_off, int64_t grp_c_off,
          const c10::optional<at::Tensor>& drop_seed, int64_t drop_site, double drop_p, int64_t drop_row0,
          const std::vector<uint64_t>& cmb_dst, const c10::optional<at::Tensor>& cmb_inv,
          const c10::optional<at::Tensor>& cmb_w, int64_t cmb_k, int64_t cmb_n);

void layernorm_fwd(const at::Tensor& x, const at::Tensor& w, const at::Tensor& b, at::Tensor& y, at::Tensor& mean,
                   at::Tensor& rstd, double eps);
int64_t layernorm_bwd_scratch_rows(int64_t M);
void layernorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& mean, const at::Tensor& rstd,
                   const at::Tensor& w, const at::Tensor& dres_in, at::Tensor& dres, at::Tensor& dres16,
                   at::Tensor& scratch, at::Tensor& dgamma, at::Tensor& dbeta, int64_t dy_srcs);
void resid_sum_ln(const at::Tensor& x, const at::Tensor& parts, int64_t nsrc, const at::Tensor& bias,
                  at::Tensor& x_new, const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& b,
                  const c10::optional<at::Tensor>& y, const c10::optional<at::Tensor>& mean,
                  const c10::optional<at::Tensor>& rstd, double eps);
void colsum_bf16(const at::Tensor& x, at::Tensor& out);
void cross_entropy_fwd(const at::Tensor& logits, int64_t V, const at::Tensor& targets, int64_t ignore_index,
                       at::Tensor& lse, at::Tensor& loss_rows, at::Tensor& loss_mean);
void cross_entropy_bwd(at::Tensor& logits, int64_t V, const at::Tensor& targets, int64_t ignore_index,
                       const at::Tensor& lse, const c10::optional<at::Tensor>& scale, double scale_mul);
void cross_entropy_fused(at::Tensor& logits, int64_t V, const at::Tensor& targets, int64_t ignore_index,
                         at::Tensor& lse, at::Tensor& loss_rows, at::Tensor& loss_mean, const at::Tensor& scale);
void cross_entropy_rescale(at::Tensor& g, const at::Tensor& actual, const at::Tensor& expected);
void embedding_fwd(const at::Tensor& idx, const at::Tensor& wte, const at::Tensor& wpe, at::Tensor& out);
void embedding_bwd(const at::Tensor& idx, const at::Tensor& dx, const c10::optional<at::Tensor>& dwte,
                   const c10::optional<at::Tensor>& dwpe);
int64_t sumsq_scratch_size();
void sumsq(const at::Tensor& x, at::Tensor& scratch, double weight, at::Tensor& out, bool accumulate);
void clip_coef(const at::Tensor& norm2, double max_norm, at::Tensor& coef, const c10::optional<at::Tensor>& norm,
               const c10::optional<at::Tensor>& loss_scale);
void loss_scale_update(const at::Tensor& coef, at::Tensor& state, double growth, double backoff, int64_t interval);
void adamw_step(at::Tensor& p, const at::Tensor& grad, at::Tensor& m, at::Tensor& v,
                const c10::optional<at::Tensor>& p16, const at::Tensor& hyper, const c10::optional<at::Tensor>& coef);
void f32_to_bf16(const at::Tensor& x, at::Tensor& y);
void attention_set_trace(const c10::optional<at::Tensor>& trace);
void attention_fwd(const at::Tensor& qkv, int64_t B, int64_t T, int64_t nh, at::Tensor& out, at::Tensor& lse,
                   const c10::optional<at::Tensor>& drop_seed, int64_t drop_site, double drop_p, int64_t h0,
                   int64_t nh_total, int64_t head_dim);
void dropout_bf16(const at::Tensor& g, at::Tensor& out, const at::Tensor& seed, int64_t site, double p,
                  int64_t row0);
void attention_bwd(const at::Tensor& qkv, const at::Tensor& out, const at::Tensor& dout, const at::Tensor& lse,
                   int64_t B, int64_t T, int64_t nh, at::Tensor& dvec, at::Tensor& dq_acc, at::Tensor& dqkv,
                   const c10::optional<at::Tensor>& drop_seed, int64_t drop_site, double drop_p, int64_t h0,
                   int64_t nh_total, int64_t head_dim);
uint64_t raw_malloc(int64_t bytes);
void raw_free(uint64_t ptr);
at::Tensor tensor_from_ptr(uint64_t ptr, int64_t numel, at::ScalarType dtype, int64_t device);
pybind11::bytes ipc_handle_py(uint64_t ptr);
uint64_t ipc_open_py(pybind11::bytes handle);
void ipc_close(uint64_t ptr);
void dp_allreduce(const std::vector<uint64_t>& data, const std::vector<uint64_t>& signal, int64_t rank, int64_t n,
                  double scale, const at::Tensor& counter, int64_t threads, int64_t blocks);
void group_barrier(const std::vector<uint64_t>& data, const std::vector<uint64_t>& signal, int64_t rank,
                   const at::Tensor& counter);
void peer_sum(const std::vector<uint64_t>& data, const std::vector<uint64_t>& signal, int64_t rank,
              const c10::optional<at::Tensor>& addend, const at::Tensor& dst, int64_t n, const at::Tensor& counter);
void moe_route(const at::Tensor& x, const at::Tensor& wg, int64_t K, double coef, at::Tensor& probs, at::Tensor& topi,
               at::Tensor& topw, at::Tensor& counts, at::Tensor& probsum, at::Tensor& off, at::Tensor& aux,
               at::Tensor& pos);
void moe_gather(const at::Tensor& x, const at::Tensor& pos, int64_t K, at::Tensor& xp, const at::Tensor& off,
                int64_t e0, int64_t e1, const c10::optional<at::Tensor>& inv);
void moe_slots_reduce(const at::Tensor& x, const at::Tensor& slots, int64_t K, at::Tensor& out);
void moe_combine(const at::Tensor& yp, const at::Tensor& pos, const at::Tensor& topw,
                 const c10::optional<at::Tensor>& resid, at::Tensor& out, const at::Tensor& off, int64_t e0,
                 int64_t e1);
void moe_combine_bwd(const at::Tensor& dy, const at::Tensor& yp, const at::Tensor& pos, const at::Tensor& topw,
                     at::Tensor& dyp, at::Tensor& dw, const at::Tensor& off, int64_t e0, int64_t e1);
void moe_unpermute(const at::Tensor& dxp, const at::Tensor& pos, int64_t K, at::Tensor& dx, const at::Tensor& off,
                   int64_t e0, int64_t e1);
void moe_local_offsets(const at::Tensor& off, int64_t e0, int64_t n, at::Tensor& out);
void moe_router_bwd(const at::Tensor& probs, const at::Tensor& topi, const at::Tensor& topw, const at::Tensor& dw,
                    const at::Tensor& daux, const at::Tensor& counts, double coef, const at::Tensor& wg,
                    at::Tensor& dlogits, at::Tensor& dx);
}  // namespace hb
