// Torch-facing entry points of the non-GEMM kernels: argument validation,
// stream selection, then a call into the raw launchers in the .cu files.
#include <ATen/cuda/CUDAContext.h>
#include <cmath>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include <initializer_list>

#include "host_utils.h"
#include "dropout_args.h"
#include "ops.h"

namespace hb {

// launchers (norm.cu, loss.cu, embed_optim.cu, attention.cu)
void ln_fwd_launch(const float*, const float*, const float*, __nv_bfloat16*, float*, float*, int, int, float, bool,
                   cudaStream_t);
int ln_bwd_num_ctas(int M, int device);
void ln_bwd_launch(const float*, const float*, const float*, const float*, const float*, const float*, float*,
                   __nv_bfloat16*, float*, int, float*, float*, int, int, int, long, bool, cudaStream_t);
void resid_sum_ln_launch(const float*, const __nv_bfloat16*, int, long, const float*, float*, const float*,
                         const float*, __nv_bfloat16*, float*, float*, int, int, float, bool, cudaStream_t);
void colsum_bf16_launch(const __nv_bfloat16*, long, int, int, float*, bool, cudaStream_t);
void ce_fwd_launch(const __nv_bfloat16*, long, int, int, const int64_t*, int, float*, float*, float*, float*, bool,
                   int*, cudaStream_t);
void ce_bwd_launch(__nv_bfloat16*, long, int, int, int, const int64_t*, int, const float*, const float*, float, bool,
                   cudaStream_t);
void ce_fused_launch(__nv_bfloat16*, long, int, int, int, const int64_t*, int, float*, float*, float*, const float*,
                     bool, int*, cudaStream_t);
void ce_rescale_launch(__nv_bfloat16*, long, int, int, const float*, const float*, bool, cudaStream_t);
void embed_fwd_launch(const int64_t*, const float*, const float*, float*, int, int, int, int, int*, cudaStream_t);
void embed_bwd_launch(const int64_t*, const float*, float*, float*, int, int, int, int, cudaStream_t);
int sumsq_num_parts(int device);
void sumsq_launch(const float*, long, float*, int, float, float*, bool, cudaStream_t);
void clip_coef_launch(const float*, float, float*, float*, const float*, cudaStream_t);
void loss_scale_update_launch(const float*, float*, float, float, int, cudaStream_t);
void adamw_launch(float*, const float*, float*, float*, __nv_bfloat16*, long, const void*, const float*, bool,
                  cudaStream_t);
void f32_to_bf16_launch(const float*, __nv_bfloat16*, long, bool, cudaStream_t);
// (16-bit tensors travel as __nv_bfloat16 pointers; the bool before the stream
// says whether they hold fp16.)
void attn_fwd_launch(const __nv_bfloat16*, long, __nv_bfloat16*, long, float*, int, int, int, int, float,
                     const DropoutArgs&, int, int, int*, bool, cudaStream_t);
void attn_bwd_launch(const __nv_bfloat16*, long, const __nv_bfloat16*, long, const __nv_bfloat16*, long,
                     const float*, float*, float*, __nv_bfloat16*, long, int, int, int, int, float,
                     const DropoutArgs&, int, int, int*, bool, cudaStream_t);
void attn_fwd_d128_launch(const __nv_bfloat16*, long, __nv_bfloat16*, long, float*, int, int, int, int, float,
                          const DropoutArgs&, int, int, int*, bool, cudaStream_t);
void attn_bwd_d128_launch(const __nv_bfloat16*, long, const __nv_bfloat16*, long, const __nv_bfloat16*, long,
                          const float*, float*, float*, __nv_bfloat16*, long, int, int, int, int, float,
                          const DropoutArgs&, int, int, int*, bool, cudaStream_t);
void attn_pad_heads(const __nv_bfloat16*, long, __nv_bfloat16*, long, long, int, int, int, cudaStream_t);
void attn_unpad_heads(const __nv_bfloat16*, long, __nv_bfloat16*, long, long, int, int, int, cudaStream_t);
void dropout_bf16_launch(const float*, __nv_bfloat16*, long, int, const DropoutArgs&, bool, cudaStream_t);

// Dropout site arguments from a device seed tensor (int32 scalar) and a rate p (0 = off).
static DropoutArgs make_dropout(const c10::optional<at::Tensor>& seed, int64_t site, double p, int64_t row0) {
  DropoutArgs d{nullptr, 0, 0, 1.f, 0};
  if (p <= 0.0) return d;
  TORCH_CHECK(p < 1.0 && seed && seed->defined() && seed->is_cuda() && seed->scalar_type() == at::kInt &&
                  seed->numel() >= 1,
              "dropout needs 0 < p < 1 and an int32 device seed");
  d.seed = reinterpret_cast<const uint32_t*>(seed->data_ptr<int>());
  d.site = static_cast<uint32_t>(site);
  d.thresh = static_cast<uint32_t>(std::lround(p * 65536.0));
  d.scale = static_cast<float>(1.0 / (1.0 - p));
  d.row0 = static_cast<long>(row0);
  if (d.thresh == 0) d.seed = nullptr;
  return d;
}

#define CHECK_CUDA(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_DT(t, dt) TORCH_CHECK((t).scalar_type() == (dt), #t " has the wrong dtype")
#define CHECK_CONTIG(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")
#define CHECK_ROWS(t) TORCH_CHECK((t).dim() == 2 && (t).stride(1) == 1, #t " must be 2-D with contiguous rows")
// Output and operand buffers are written / read up to the sizes the launch
// derives from its main input: each must hold at least that many elements.
#define CHECK_HOLDS(t, n) TORCH_CHECK((t).numel() >= (int64_t)(n), #t " holds fewer than " #n " elements")
#define CHECK_F32_HOLDS(t, n) \
  do {                        \
    CHECK_DT(t, at::kFloat);  \
    CHECK_CONTIG(t);          \
    CHECK_HOLDS(t, n);        \
  } while (0)

// Data pointer of a bf16 or fp16 tensor as the kernels' 16-bit element pointer
// (kernels take the format as a flag: is_f16).
static __nv_bfloat16* raw16(const at::Tensor& t) {
  TORCH_CHECK(t.scalar_type() == at::kBFloat16 || t.scalar_type() == at::kHalf, "expected a bf16 or fp16 tensor");
  return reinterpret_cast<__nv_bfloat16*>(t.data_ptr());
}
static bool is_f16(const at::Tensor& t) { return t.scalar_type() == at::kHalf; }

static cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }
template <typename T>
static T* ptr(const at::Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}

void layernorm_fwd(const at::Tensor& x, const at::Tensor& w, const at::Tensor& b, at::Tensor& y, at::Tensor& mean,
                   at::Tensor& rstd, double eps) {
  CHECK_CUDA(x);
  CHECK_DT(x, at::kFloat);
  CHECK_CONTIG(x);
  CHECK_DT(w, at::kFloat);
  CHECK_DT(b, at::kFloat);
  CHECK_CONTIG(y);
  c10::cuda::CUDAGuard g(x.device());
  const int H = x.size(-1);
  const int M = x.numel() / H;
  CHECK_F32_HOLDS(w, H);
  CHECK_F32_HOLDS(b, H);
  CHECK_HOLDS(y, (int64_t)M * H);
  CHECK_F32_HOLDS(mean, M);
  CHECK_F32_HOLDS(rstd, M);
  ln_fwd_launch(ptr<float>(x), ptr<float>(w), ptr<float>(b), raw16(y), ptr<float>(mean), ptr<float>(rstd), M, H,
                static_cast<float>(eps), is_f16(y), stream());
}

int64_t layernorm_bwd_scratch_rows(int64_t M) { return ln_bwd_num_ctas(static_cast<int>(M), current_device()); }

void layernorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& mean, const at::Tensor& rstd,
                   const at::Tensor& w, const at::Tensor& dres_in, at::Tensor& dres, at::Tensor& dres16,
                   at::Tensor& scratch, at::Tensor& dgamma, at::Tensor& dbeta, int64_t dy_srcs) {
  CHECK_CUDA(dy);
  CHECK_DT(dy, at::kFloat);
  CHECK_CONTIG(dy);
  CHECK_DT(x, at::kFloat);
  CHECK_CONTIG(x);
  CHECK_DT(dres, at::kFloat);
  CHECK_CONTIG(dres);
  CHECK_DT(dres_in, at::kFloat);
  CHECK_CONTIG(dres_in);
  CHECK_CONTIG(dres16);
  CHECK_DT(scratch, at::kFloat);
  c10::cuda::CUDAGuard g(x.device());
  const int H = x.size(-1);
  const int M = x.numel() / H;
  const int ctas = ln_bwd_num_ctas(M, x.get_device());
  TORCH_CHECK(scratch.numel() >= (int64_t)ctas * 2 * H, "layernorm_bwd: scratch too small");
  CHECK_F32_HOLDS(mean, M);
  CHECK_F32_HOLDS(rstd, M);
  CHECK_F32_HOLDS(w, H);
  CHECK_HOLDS(dres_in, (int64_t)M * H);
  CHECK_HOLDS(dres, (int64_t)M * H);
  CHECK_HOLDS(dres16, (int64_t)M * H);
  CHECK_F32_HOLDS(dgamma, H);
  CHECK_F32_HOLDS(dbeta, H);
  TORCH_CHECK(dy_srcs >= 1 && dy.numel() >= dy_srcs * (int64_t)M * H, "layernorm_bwd: dy holds dy_srcs slots of [M, H]");
  ln_bwd_launch(ptr<float>(dy), ptr<float>(x), ptr<float>(mean), ptr<float>(rstd), ptr<float>(w),
                ptr<float>(dres_in), ptr<float>(dres), raw16(dres16), ptr<float>(scratch), ctas, ptr<float>(dgamma),
                ptr<float>(dbeta), M, H, static_cast<int>(dy_srcs), (long)M * H, is_f16(dres16), stream());
}

void resid_sum_ln(const at::Tensor& x, const at::Tensor& parts, int64_t nsrc, const at::Tensor& bias,
                  at::Tensor& x_new, const c10::optional<at::Tensor>& w, const c10::optional<at::Tensor>& b,
                  const c10::optional<at::Tensor>& y, const c10::optional<at::Tensor>& mean,
                  const c10::optional<at::Tensor>& rstd, double eps) {
  CHECK_CUDA(x);
  CHECK_DT(x, at::kFloat);
  CHECK_CONTIG(x);
  CHECK_DT(x_new, at::kFloat);
  const int H = x.size(-1);
  const int M = x.numel() / H;
  TORCH_CHECK(parts.numel() >= nsrc * (int64_t)M * H, "resid_sum_ln: parts holds nsrc slots of [M, H]");
  CHECK_F32_HOLDS(bias, H);
  CHECK_CONTIG(x_new);
  CHECK_HOLDS(x_new, (int64_t)M * H);
  const bool ln = w && w->defined();
  if (ln) {
    TORCH_CHECK(b && b->defined() && y && y->defined() && mean && mean->defined() && rstd && rstd->defined(),
                "resid_sum_ln: with w, also b, y, mean and rstd");
    CHECK_F32_HOLDS((*w), H);
    CHECK_F32_HOLDS((*b), H);
    CHECK_CONTIG((*y));
    CHECK_HOLDS((*y), (int64_t)M * H);
    CHECK_F32_HOLDS((*mean), M);
    CHECK_F32_HOLDS((*rstd), M);
  }
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(!ln || y->scalar_type() == parts.scalar_type(), "resid_sum_ln: y and parts share one 16-bit format");
  resid_sum_ln_launch(ptr<float>(x), raw16(parts), static_cast<int>(nsrc), (long)M * H, ptr<float>(bias),
                      ptr<float>(x_new), ln ? ptr<float>(*w) : nullptr, ln ? ptr<float>(*b) : nullptr,
                      ln ? raw16(*y) : nullptr, ln ? ptr<float>(*mean) : nullptr, ln ? ptr<float>(*rstd) : nullptr, M,
                      H, static_cast<float>(eps), is_f16(parts), stream());
}

void colsum_bf16(const at::Tensor& x, at::Tensor& out) {
  CHECK_CUDA(x);
  CHECK_ROWS(x);
  CHECK_DT(out, at::kFloat);
  TORCH_CHECK(x.size(1) % 2 == 0 && x.stride(0) % 2 == 0, "colsum_bf16: even column count required");
  CHECK_CONTIG(out);
  CHECK_HOLDS(out, x.size(1));
  c10::cuda::CUDAGuard g(x.device());
  colsum_bf16_launch(raw16(x), x.stride(0), x.size(0), x.size(1), ptr<float>(out), is_f16(x), stream());
}

// The cross-entropy kernels read and write logit rows in 16-byte pieces: the row
// stride must be a multiple of 8 elements and the base 16-byte aligned, and
// 1 <= V <= the row width.
static void check_ce_logits(const at::Tensor& logits, int64_t V) {
  CHECK_CUDA(logits);
  CHECK_ROWS(logits);
  raw16(logits);
  TORCH_CHECK(logits.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0,
              "cross-entropy: logit rows must start on 16-byte boundaries (row stride a multiple of 8)");
  TORCH_CHECK(V >= 1 && V <= logits.size(1), "cross-entropy: V must be in [1, row width]");
}
static void check_ce_targets(const at::Tensor& targets, int64_t M) {
  CHECK_DT(targets, at::kLong);
  CHECK_CONTIG(targets);
  CHECK_HOLDS(targets, M);
}

void cross_entropy_fwd(const at::Tensor& logits, int64_t V, const at::Tensor& targets, int64_t ignore_index,
                       at::Tensor& lse, at::Tensor& loss_rows, at::Tensor& loss_mean) {
  check_ce_logits(logits, V);
  const int64_t M = logits.size(0);
  check_ce_targets(targets, M);
  CHECK_F32_HOLDS(lse, M);
  CHECK_F32_HOLDS(loss_rows, M);
  CHECK_F32_HOLDS(loss_mean, 1);
  c10::cuda::CUDAGuard g(logits.device());
  ce_fwd_launch(raw16(logits), logits.stride(0), logits.size(0), V, ptr<int64_t>(targets), ignore_index,
                ptr<float>(lse), ptr<float>(loss_rows), ptr<float>(loss_mean), nullptr, is_f16(logits),
                device_status_ptr(logits.get_device()), stream());
}

void cross_entropy_bwd(at::Tensor& logits, int64_t V, const at::Tensor& targets, int64_t ignore_index,
                       const at::Tensor& lse, const c10::optional<at::Tensor>& scale, double scale_mul) {
  check_ce_logits(logits, V);
  const int64_t M = logits.size(0);
  check_ce_targets(targets, M);
  CHECK_F32_HOLDS(lse, M);
  if (scale && scale->defined()) CHECK_F32_HOLDS((*scale), 1);
  c10::cuda::CUDAGuard g(logits.device());
  const float* sp = (scale && scale->defined()) ? ptr<float>(*scale) : nullptr;
  ce_bwd_launch(raw16(logits), logits.stride(0), logits.size(0), V, logits.size(1), ptr<int64_t>(targets),
                ignore_index, ptr<float>(lse), sp, static_cast<float>(scale_mul), is_f16(logits), stream());
}

void cross_entropy_fused(at::Tensor& logits, int64_t V, const at::Tensor& targets, int64_t ignore_index,
                         at::Tensor& lse, at::Tensor& loss_rows, at::Tensor& loss_mean, const at::Tensor& scale) {
  check_ce_logits(logits, V);
  const int64_t M = logits.size(0);
  check_ce_targets(targets, M);
  CHECK_F32_HOLDS(lse, M);
  CHECK_F32_HOLDS(loss_rows, M);
  CHECK_F32_HOLDS(loss_mean, 1);
  CHECK_F32_HOLDS(scale, 1);
  c10::cuda::CUDAGuard g(logits.device());
  ce_fused_launch(raw16(logits), logits.stride(0), logits.size(0), V, logits.size(1), ptr<int64_t>(targets),
                  ignore_index, ptr<float>(lse), ptr<float>(loss_rows), ptr<float>(loss_mean), ptr<float>(scale),
                  is_f16(logits), device_status_ptr(logits.get_device()), stream());
}

void cross_entropy_rescale(at::Tensor& g, const at::Tensor& actual, const at::Tensor& expected) {
  CHECK_CUDA(g);
  CHECK_ROWS(g);
  CHECK_F32_HOLDS(actual, 1);
  CHECK_F32_HOLDS(expected, 1);
  raw16(g);
  TORCH_CHECK(g.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(g.data_ptr()) % 16 == 0,
              "cross_entropy_rescale: rows must start on 16-byte boundaries");
  c10::cuda::CUDAGuard gd(g.device());
  ce_rescale_launch(raw16(g), g.stride(0), g.size(0), g.size(1), ptr<float>(actual), ptr<float>(expected), is_f16(g),
                    stream());
}

void embedding_fwd(const at::Tensor& idx, const at::Tensor& wte, const at::Tensor& wpe, at::Tensor& out) {
  CHECK_CUDA(idx);
  CHECK_DT(idx, at::kLong);
  CHECK_CONTIG(idx);
  CHECK_DT(wte, at::kFloat);
  CHECK_CONTIG(wte);
  CHECK_DT(wpe, at::kFloat);
  CHECK_CONTIG(wpe);
  CHECK_CONTIG(out);
  TORCH_CHECK(idx.dim() == 2 && wte.dim() == 2 && wpe.dim() == 2 && wpe.size(1) == wte.size(1),
              "embedding_fwd: idx [B, T], wte [V, H], wpe [P, H]");
  TORCH_CHECK(idx.size(1) <= wpe.size(0), "embedding_fwd: sequence longer than the position table");
  CHECK_HOLDS(out, idx.numel() * wte.size(1));
  c10::cuda::CUDAGuard g(idx.device());
  embed_fwd_launch(ptr<int64_t>(idx), ptr<float>(wte), ptr<float>(wpe), ptr<float>(out), idx.size(0), idx.size(1),
                   wte.size(1), static_cast<int>(wte.size(0)), device_status_ptr(idx.get_device()), stream());
}

void embedding_bwd(const at::Tensor& idx, const at::Tensor& dx, const c10::optional<at::Tensor>& dwte,
                   const c10::optional<at::Tensor>& dwpe) {
  CHECK_CUDA(dx);
  CHECK_DT(dx, at::kFloat);
  CHECK_CONTIG(dx);
  CHECK_DT(idx, at::kLong);
  CHECK_CONTIG(idx);
  TORCH_CHECK(idx.dim() == 2, "embedding_bwd: idx [B, T]");
  const int H = dx.size(-1);
  CHECK_HOLDS(dx, idx.numel() * H);
  const bool tok = dwte && dwte->defined(), pos = dwpe && dwpe->defined();
  if (tok) {
    CHECK_CONTIG((*dwte));
    TORCH_CHECK(dwte->scalar_type() == at::kFloat && dwte->dim() == 2 && dwte->size(1) == H, "embedding_bwd: dwte [V, H]");
  }
  if (pos) {
    CHECK_CONTIG((*dwpe));
    TORCH_CHECK(dwpe->scalar_type() == at::kFloat && dwpe->dim() == 2 && dwpe->size(1) == H &&
                    dwpe->size(0) >= idx.size(1),
                "embedding_bwd: dwpe [P >= T, H]");
  }
  c10::cuda::CUDAGuard g(dx.device());
  embed_bwd_launch(ptr<int64_t>(idx), ptr<float>(dx), tok ? ptr<float>(*dwte) : nullptr,
                   pos ? ptr<float>(*dwpe) : nullptr, idx.size(0), idx.size(1), H,
                   tok ? static_cast<int>(dwte->size(0)) : 0, stream());
}

int64_t sumsq_scratch_size() { return sumsq_num_parts(current_device()); }

void sumsq(const at::Tensor& x, at::Tensor& scratch, double weight, at::Tensor& out, bool accumulate) {
  CHECK_CUDA(x);
  CHECK_DT(x, at::kFloat);
  CHECK_CONTIG(x);
  c10::cuda::CUDAGuard g(x.device());
  const int parts = sumsq_num_parts(x.get_device());
  TORCH_CHECK(scratch.numel() >= parts, "sumsq: scratch too small");
  CHECK_DT(scratch, at::kFloat);
  CHECK_F32_HOLDS(out, 1);
  sumsq_launch(ptr<float>(x), x.numel(), ptr<float>(scratch), parts, static_cast<float>(weight), ptr<float>(out),
               accumulate, stream());
}

void clip_coef(const at::Tensor& norm2, double max_norm, at::Tensor& coef, const c10::optional<at::Tensor>& norm,
               const c10::optional<at::Tensor>& loss_scale) {
  CHECK_CUDA(norm2);
  CHECK_F32_HOLDS(norm2, 1);
  CHECK_F32_HOLDS(coef, 1);
  if (norm && norm->defined()) CHECK_F32_HOLDS((*norm), 1);
  if (loss_scale && loss_scale->defined()) CHECK_F32_HOLDS((*loss_scale), 1);
  c10::cuda::CUDAGuard g(norm2.device());
  clip_coef_launch(ptr<float>(norm2), static_cast<float>(max_norm), ptr<float>(coef),
                   (norm && norm->defined()) ? ptr<float>(*norm) : nullptr,
                   (loss_scale && loss_scale->defined()) ? ptr<float>(*loss_scale) : nullptr, stream());
}

// state = {scale, finite steps in a row} (fp32 device tensor), updated after a step
// whose coefficient (NaN = skipped) is `coef`.
void loss_scale_update(const at::Tensor& coef, at::Tensor& state, double growth, double backoff, int64_t interval) {
  TORCH_CHECK(state.is_cuda() && state.scalar_type() == at::kFloat && state.numel() >= 2, "loss_scale_update: state");
  c10::cuda::CUDAGuard g(state.device());
  loss_scale_update_launch(ptr<float>(coef), ptr<float>(state), static_cast<float>(growth),
                           static_cast<float>(backoff), static_cast<int>(interval), stream());
}

void adamw_step(at::Tensor& p, const at::Tensor& grad, at::Tensor& m, at::Tensor& v,
                const c10::optional<at::Tensor>& p16, const at::Tensor& hyper, const c10::optional<at::Tensor>& coef) {
  CHECK_CUDA(p);
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&p, &grad, &m, &v}) {
    TORCH_CHECK(t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == p.numel(),
                "adamw_step: p, grad, m, v must be contiguous fp32 of equal size");
  }
  TORCH_CHECK(hyper.scalar_type() == at::kFloat && hyper.numel() >= 8 && hyper.is_cuda(), "adamw_step: hyper");
  c10::cuda::CUDAGuard g(p.device());
  __nv_bfloat16* p16p = nullptr;
  bool f16 = false;
  if (p16 && p16->defined()) {
    TORCH_CHECK(p16->numel() == p.numel() && p16->is_contiguous(), "p16");
    p16p = raw16(*p16);
    f16 = is_f16(*p16);
  }
  adamw_launch(ptr<float>(p), ptr<float>(grad), ptr<float>(m), ptr<float>(v), p16p, p.numel(), hyper.data_ptr(),
               (coef && coef->defined()) ? ptr<float>(*coef) : nullptr, f16, stream());
}

void f32_to_bf16(const at::Tensor& x, at::Tensor& y) {
  CHECK_CUDA(x);
  CHECK_DT(x, at::kFloat);
  CHECK_CONTIG(x);
  CHECK_CONTIG(y);
  TORCH_CHECK(x.numel() == y.numel(), "f32_to_bf16: size mismatch");
  c10::cuda::CUDAGuard g(x.device());
  f32_to_bf16_launch(ptr<float>(x), raw16(y), x.numel(), is_f16(y), stream());
}

void attn_set_trace(uint64_t* trace, long rows);

// Phase timestamps of the following attention launches go to `trace`
// (int64, 80 per CTA, on the device; a launch with more CTAs than the buffer has
// rows of 80 is not traced); None turns tracing off.
void attention_set_trace(const c10::optional<at::Tensor>& trace) {
  if (trace && trace->defined()) {
    TORCH_CHECK(trace->is_cuda() && trace->scalar_type() == at::kLong && trace->is_contiguous(),
                "attention_set_trace: int64 contiguous CUDA tensor");
    attn_set_trace(reinterpret_cast<uint64_t*>(trace->data_ptr()), static_cast<long>(trace->numel() / 80));
  } else {
    attn_set_trace(nullptr, 0);
  }
}

// Head widths: 64 and 128 run their own kernels; 16 and 32 run the 64-wide
// kernels on zero-padded copies of the heads (see attention_d128.cu).
static void check_head_dim(int64_t dh) {
  TORCH_CHECK(dh == 16 || dh == 32 || dh == 64 || dh == 128, "attention: head_dim must be 16, 32, 64 or 128, got ",
              dh);
}

void attention_fwd(const at::Tensor& qkv, int64_t B, int64_t T, int64_t nh, at::Tensor& out, at::Tensor& lse,
                   const c10::optional<at::Tensor>& drop_seed, int64_t drop_site, double drop_p, int64_t h0,
                   int64_t nh_total, int64_t head_dim) {
  CHECK_CUDA(qkv);
  TORCH_CHECK(qkv.scalar_type() == at::kBFloat16 || qkv.scalar_type() == at::kHalf, "attention_fwd: bf16 or fp16 qkv");
  CHECK_ROWS(qkv);
  CHECK_DT(out, qkv.scalar_type());
  CHECK_ROWS(out);
  check_head_dim(head_dim);
  const bool f16 = qkv.scalar_type() == at::kHalf;
  TORCH_CHECK(qkv.size(0) == B * T && qkv.size(1) == 3 * nh * head_dim,
              "attention_fwd: qkv must be [B*T, 3*nh*head_dim]");
  TORCH_CHECK(out.size(0) == B * T && out.size(1) >= nh * head_dim, "attention_fwd: out must be [B*T, nh*head_dim]");
  TORCH_CHECK(qkv.stride(0) % 8 == 0 && out.stride(0) % 8 == 0, "attention_fwd: row strides must be 16B multiples");
  const int64_t Tpad = (T + 127) / 128 * 128;
  TORCH_CHECK(lse.numel() >= B * nh * Tpad && lse.scalar_type() == at::kFloat, "attention_fwd: lse [B, nh, Tpad]");
  c10::cuda::CUDAGuard g(qkv.device());
  TORCH_CHECK(drop_p <= 0.0 || T % 2 == 0, "attention dropout pairs keys (T must be even)");
  const DropoutArgs d = make_dropout(drop_seed, drop_site, drop_p, 0);
  const float scale = 1.f / std::sqrt(static_cast<float>(head_dim));
  const int nht = static_cast<int>(nh_total > 0 ? nh_total : nh);
  int* status = device_status_ptr(qkv.get_device());
  if (head_dim == 128) {
    attn_fwd_d128_launch(raw16(qkv), qkv.stride(0), raw16(out), out.stride(0), ptr<float>(lse), B, T, nh, Tpad, scale,
                         d, static_cast<int>(h0), nht, status, f16, stream());
    return;
  }
  if (head_dim == 64) {
    attn_fwd_launch(raw16(qkv), qkv.stride(0), raw16(out), out.stride(0), ptr<float>(lse), B, T, nh, Tpad, scale, d,
                    static_cast<int>(h0), nht, status, f16, stream());
    return;
  }
  const long rows = B * T;
  auto opts = qkv.options();
  at::Tensor qkv_p = at::empty({rows, 3 * nh * 64}, opts), out_p = at::empty({rows, nh * 64}, opts);
  attn_pad_heads(raw16(qkv), qkv.stride(0), raw16(qkv_p), qkv_p.stride(0), rows, 3, nh, head_dim, stream());
  attn_fwd_launch(raw16(qkv_p), qkv_p.stride(0), raw16(out_p), out_p.stride(0), ptr<float>(lse), B, T, nh, Tpad, scale,
                  d, static_cast<int>(h0), nht, status, f16, stream());
  attn_unpad_heads(raw16(out_p), out_p.stride(0), raw16(out), out.stride(0), rows, 1, nh, head_dim, stream());
}

void attention_bwd(const at::Tensor& qkv, const at::Tensor& out, const at::Tensor& dout, const at::Tensor& lse,
                   int64_t B, int64_t T, int64_t nh, at::Tensor& dvec, at::Tensor& dq_acc, at::Tensor& dqkv,
                   const c10::optional<at::Tensor>& drop_seed, int64_t drop_site, double drop_p, int64_t h0,
                   int64_t nh_total, int64_t head_dim) {
  CHECK_CUDA(qkv);
  const bool f16 = qkv.scalar_type() == at::kHalf;
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&qkv, &out, &dout, &dqkv}) {
    TORCH_CHECK(t->scalar_type() == (f16 ? at::kHalf : at::kBFloat16) && t->dim() == 2 && t->stride(1) == 1 &&
                    t->stride(0) % 8 == 0,
                "attention_bwd: 2-D tensors of one 16-bit format with 16B-aligned rows expected");
  }
  check_head_dim(head_dim);
  TORCH_CHECK(qkv.size(1) == 3 * nh * head_dim && dqkv.size(1) >= 3 * nh * head_dim,
              "attention_bwd: qkv / dqkv must be [B*T, 3*nh*head_dim]");
  const int64_t Tpad = (T + 127) / 128 * 128;
  const int64_t dh_k = head_dim < 64 ? 64 : head_dim;  // width the kernels run at
  TORCH_CHECK(dvec.numel() >= B * nh * Tpad && lse.numel() >= B * nh * Tpad, "attention_bwd: lse/dvec size");
  TORCH_CHECK(dq_acc.numel() >= B * T * nh * dh_k && dq_acc.scalar_type() == at::kFloat, "attention_bwd: dq_acc");
  c10::cuda::CUDAGuard g(qkv.device());
  const DropoutArgs d = make_dropout(drop_seed, drop_site, drop_p, 0);
  const float scale = 1.f / std::sqrt(static_cast<float>(head_dim));
  const int nht = static_cast<int>(nh_total > 0 ? nh_total : nh);
  int* status = device_status_ptr(qkv.get_device());
  if (head_dim >= 64) {
    auto launch = head_dim == 128 ? attn_bwd_d128_launch : attn_bwd_launch;
    launch(raw16(qkv), qkv.stride(0), raw16(out), out.stride(0), raw16(dout), dout.stride(0), ptr<float>(lse),
           ptr<float>(dvec), ptr<float>(dq_acc), raw16(dqkv), dqkv.stride(0), B, T, nh, Tpad, scale, d,
           static_cast<int>(h0), nht, status, f16, stream());
    return;
  }
  const long rows = B * T;
  auto opts = qkv.options();
  at::Tensor qkv_p = at::empty({rows, 3 * nh * 64}, opts), out_p = at::empty({rows, nh * 64}, opts);
  at::Tensor dout_p = at::empty({rows, nh * 64}, opts), dqkv_p = at::empty({rows, 3 * nh * 64}, opts);
  attn_pad_heads(raw16(qkv), qkv.stride(0), raw16(qkv_p), qkv_p.stride(0), rows, 3, nh, head_dim, stream());
  attn_pad_heads(raw16(out), out.stride(0), raw16(out_p), out_p.stride(0), rows, 1, nh, head_dim, stream());
  attn_pad_heads(raw16(dout), dout.stride(0), raw16(dout_p), dout_p.stride(0), rows, 1, nh, head_dim, stream());
  attn_bwd_launch(raw16(qkv_p), qkv_p.stride(0), raw16(out_p), out_p.stride(0), raw16(dout_p), dout_p.stride(0),
                  ptr<float>(lse), ptr<float>(dvec), ptr<float>(dq_acc), raw16(dqkv_p), dqkv_p.stride(0), B, T, nh, Tpad,
                  scale, d, static_cast<int>(h0), nht, status, f16, stream());
  attn_unpad_heads(raw16(dqkv_p), dqkv_p.stride(0), raw16(dqkv), dqkv.stride(0), rows, 3, nh, head_dim, stream());
}

// out (bf16) = g * mask for a residual dropout site: the gradient reaching
// the sub-layer's output projection (element (row0 + row) * H + col).
void dropout_bf16(const at::Tensor& g, at::Tensor& out, const at::Tensor& seed, int64_t site, double p,
                  int64_t row0) {
  CHECK_CUDA(g);
  TORCH_CHECK(g.scalar_type() == at::kFloat && g.is_contiguous() && g.dim() == 2, "dropout_bf16: g fp32 [M, H]");
  TORCH_CHECK((out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kHalf) && out.is_contiguous() &&
                  out.sizes() == g.sizes(),
              "dropout_bf16: out 16-bit (bf16 or fp16) like g");
  TORCH_CHECK(g.size(1) % 4 == 0, "dropout_bf16: H % 4 == 0");
  const DropoutArgs d = make_dropout(seed, site, p, row0);
  TORCH_CHECK(d.seed != nullptr, "dropout_bf16: p must be > 0");
  c10::cuda::CUDAGuard guard(g.device());
  dropout_bf16_launch(ptr<float>(g), raw16(out), g.size(0), static_cast<int>(g.size(1)), d, is_f16(out), stream());
}

}  // namespace hb
