// Torch-facing entry points of the mixture-of-experts kernels (moe.cu).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <torch/extension.h>

#include "host_utils.h"
#include "ops.h"

namespace hb {

void moe_route_launch(const __nv_bfloat16*, const float*, int, int, int, int, float, float*, int*, float*, int*, float*,
                      int*, float*, int*, bool, cudaStream_t);
void moe_gather_launch(const __nv_bfloat16*, const int*, int, int, int, __nv_bfloat16*, const int*, int, int, int,
                       int*, int*, cudaStream_t);
void moe_slots_reduce_launch(const float*, const __nv_bfloat16*, int, int, int, float*, bool, cudaStream_t);
void moe_combine_launch(const __nv_bfloat16*, const int*, const float*, const float*, int, int, int, float*,
                        const int*, int, int, int, int*, bool, cudaStream_t);
void moe_combine_bwd_launch(const float*, const __nv_bfloat16*, const int*, const float*, int, int, int,
                            __nv_bfloat16*, float*, const int*, int, int, int, int*, bool, cudaStream_t);
void moe_unpermute_launch(const float*, const int*, int, int, int, float*, const int*, int, int, int, int*,
                          cudaStream_t);
void moe_local_offsets_launch(const int*, int, int, int*, cudaStream_t);
void moe_router_bwd_launch(const float*, const int*, const float*, const float*, const float*, const int*, float, int,
                           int, int, int, const float*, __nv_bfloat16*, long, float*, bool, cudaStream_t);

template <typename T>
static T* P(const at::Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}
static cudaStream_t S() { return at::cuda::getCurrentCUDAStream(); }

static void check_i32(const at::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kInt && t.is_contiguous(), what, ": int32 contiguous CUDA tensor");
}
static void check_f32(const at::Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.is_contiguous(), what, ": fp32 contiguous CUDA tensor");
}

void moe_route(const at::Tensor& x, const at::Tensor& wg, int64_t K, double coef, at::Tensor& probs, at::Tensor& topi,
               at::Tensor& topw, at::Tensor& counts, at::Tensor& probsum, at::Tensor& off, at::Tensor& aux,
               at::Tensor& pos) {
  TORCH_CHECK(x.is_cuda() && (x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kHalf) && x.is_contiguous(),
              "moe_route: x bf16 or fp16 [N, H]");
  check_f32(wg, "moe_route: gate weight [E, H]");
  check_f32(probs, "moe_route: probs");
  check_i32(topi, "moe_route: topi");
  check_i32(counts, "moe_route: counts");
  check_i32(off, "moe_route: off");
  check_i32(pos, "moe_route: pos");
  c10::cuda::CUDAGuard g(x.device());
  const int N = x.size(0), H = x.size(1), E = wg.size(0);
  check_f32(topw, "moe_route: topw");
  check_f32(probsum, "moe_route: probsum");
  check_f32(aux, "moe_route: aux");
  TORCH_CHECK(K >= 1 && K <= E, "moe_route: top-k must be in [1, E]");
  TORCH_CHECK(wg.size(1) == H && probs.numel() >= (int64_t)N * E && topi.numel() >= N * K && off.numel() >= E + 1 &&
                  pos.numel() >= N * K && topw.numel() >= N * K && counts.numel() >= E && probsum.numel() >= E &&
                  aux.numel() >= 1,
              "moe_route: shape mismatch");
  moe_route_launch(P<__nv_bfloat16>(x), P<float>(wg), N, H, E, K, static_cast<float>(coef), P<float>(probs),
                   P<int>(topi), P<float>(topw), P<int>(counts), P<float>(probsum), P<int>(off), P<float>(aux),
                   P<int>(pos), x.scalar_type() == at::kHalf, S());
}

// Expert window [e0, e1): only rows of padded expert segments e0 .. e1-1 take
// part (this rank's experts under expert parallelism; e0 = 0, e1 = E
// otherwise). Rows are addressed relative to the window's first row off[e0].
static void check_window(const at::Tensor& off, int64_t e0, int64_t e1) {
  check_i32(off, "moe: expert offsets");
  TORCH_CHECK(0 <= e0 && e0 < e1 && e1 < off.numel(), "moe: expert window out of range");
}

void moe_gather(const at::Tensor& x, const at::Tensor& pos, int64_t K, at::Tensor& xp, const at::Tensor& off,
                int64_t e0, int64_t e1, const c10::optional<at::Tensor>& inv) {
  TORCH_CHECK((x.scalar_type() == at::kBFloat16 || x.scalar_type() == at::kHalf) &&
                  xp.scalar_type() == x.scalar_type() && x.size(1) == xp.size(1),
              "moe_gather: 16-bit [N, H] -> [R, H] of one format");
  check_window(off, e0, e1);
  c10::cuda::CUDAGuard g(x.device());
  int* inv_p = nullptr;
  if (inv && inv->defined()) {
    check_i32(*inv, "moe_gather: inv");
    TORCH_CHECK(inv->numel() >= xp.size(0), "moe_gather: inv needs one entry per permuted row");
    inv_p = P<int>(*inv);
  }
  moe_gather_launch(P<__nv_bfloat16>(x), P<int>(pos), x.size(0), K, x.size(1), P<__nv_bfloat16>(xp), P<int>(off),
                    e0, e1, xp.size(0), device_status_ptr(x.get_device()), inv_p, S());
}

// out = x + sum_k slots[k] (fp32 [N, H] out and x; 16-bit slots [K, N, H]).
void moe_slots_reduce(const at::Tensor& x, const at::Tensor& slots, int64_t K, at::Tensor& out) {
  check_f32(x, "moe_slots_reduce: x");
  check_f32(out, "moe_slots_reduce: out");
  TORCH_CHECK((slots.scalar_type() == at::kBFloat16 || slots.scalar_type() == at::kHalf) && slots.is_contiguous() &&
                  slots.numel() >= K * x.numel(),
              "moe_slots_reduce: slots 16-bit [K, N, H]");
  c10::cuda::CUDAGuard g(x.device());
  moe_slots_reduce_launch(P<float>(x), P<__nv_bfloat16>(slots), x.size(0), K, x.size(1), P<float>(out),
                          slots.scalar_type() == at::kHalf, S());
}

void moe_combine(const at::Tensor& yp, const at::Tensor& pos, const at::Tensor& topw,
                 const c10::optional<at::Tensor>& resid, at::Tensor& out, const at::Tensor& off, int64_t e0,
                 int64_t e1) {
  check_f32(out, "moe_combine: out");
  const float* r = nullptr;
  if (resid && resid->defined()) {
    check_f32(*resid, "moe_combine: resid");
    TORCH_CHECK(resid->sizes() == out.sizes(), "moe_combine: resid / out shapes");
    r = P<float>(*resid);
  }
  check_window(off, e0, e1);
  check_i32(pos, "moe_combine: pos");
  check_f32(topw, "moe_combine: topw");
  TORCH_CHECK(out.dim() == 2 && topw.dim() == 2 && topw.size(0) >= out.size(0), "moe_combine: out [N, H], topw [N, K]");
  TORCH_CHECK((yp.scalar_type() == at::kBFloat16 || yp.scalar_type() == at::kHalf) && yp.is_contiguous() &&
                  yp.dim() == 2 && yp.size(1) == out.size(1),
              "moe_combine: yp 16-bit [R, H]");
  TORCH_CHECK(pos.numel() >= out.size(0) * topw.size(1), "moe_combine: pos holds N * K rows");
  c10::cuda::CUDAGuard g(yp.device());
  const int N = out.size(0), H = out.size(1), K = topw.size(1);
  moe_combine_launch(P<__nv_bfloat16>(yp), P<int>(pos), P<float>(topw), r, N, K, H, P<float>(out), P<int>(off), e0,
                     e1, yp.size(0), device_status_ptr(yp.get_device()), yp.scalar_type() == at::kHalf, S());
}

void moe_combine_bwd(const at::Tensor& dy, const at::Tensor& yp, const at::Tensor& pos, const at::Tensor& topw,
                     at::Tensor& dyp, at::Tensor& dw, const at::Tensor& off, int64_t e0, int64_t e1) {
  check_f32(dy, "moe_combine_bwd: dy");
  check_window(off, e0, e1);
  check_i32(pos, "moe_combine_bwd: pos");
  check_f32(topw, "moe_combine_bwd: topw");
  check_f32(dw, "moe_combine_bwd: dw");
  TORCH_CHECK(dy.dim() == 2 && topw.dim() == 2 && topw.size(0) >= dy.size(0), "moe_combine_bwd: dy [N, H], topw [N, K]");
  TORCH_CHECK((yp.scalar_type() == at::kBFloat16 || yp.scalar_type() == at::kHalf) && yp.is_contiguous() &&
                  yp.dim() == 2 && yp.size(1) == dy.size(1) && dyp.scalar_type() == yp.scalar_type() &&
                  dyp.is_contiguous() && dyp.numel() >= yp.numel(),
              "moe_combine_bwd: yp and dyp 16-bit [R, H] of one format");
  TORCH_CHECK(pos.numel() >= dy.size(0) * topw.size(1) && dw.numel() >= dy.size(0) * topw.size(1),
              "moe_combine_bwd: pos and dw hold N * K entries");
  c10::cuda::CUDAGuard g(dy.device());
  const int N = dy.size(0), H = dy.size(1), K = topw.size(1);
  moe_combine_bwd_launch(P<float>(dy), P<__nv_bfloat16>(yp), P<int>(pos), P<float>(topw), N, K, H,
                         P<__nv_bfloat16>(dyp), P<float>(dw), P<int>(off), e0, e1, yp.size(0),
                         device_status_ptr(dy.get_device()), yp.scalar_type() == at::kHalf, S());
}

void moe_unpermute(const at::Tensor& dxp, const at::Tensor& pos, int64_t K, at::Tensor& dx, const at::Tensor& off,
                   int64_t e0, int64_t e1) {
  check_f32(dxp, "moe_unpermute: dxp");
  check_f32(dx, "moe_unpermute: dx");
  check_window(off, e0, e1);
  check_i32(pos, "moe_unpermute: pos");
  TORCH_CHECK(dx.dim() == 2 && dxp.dim() == 2 && dxp.size(1) == dx.size(1) && pos.numel() >= dx.size(0) * K,
              "moe_unpermute: dxp [R, H], dx [N, H], pos N * K");
  c10::cuda::CUDAGuard g(dx.device());
  moe_unpermute_launch(P<float>(dxp), P<int>(pos), dx.size(0), K, dx.size(1), P<float>(dx), P<int>(off), e0, e1,
                       dxp.size(0), device_status_ptr(dx.get_device()), S());
}

void moe_local_offsets(const at::Tensor& off, int64_t e0, int64_t n, at::Tensor& out) {
  check_window(off, e0, e0 + n);
  check_i32(out, "moe_local_offsets: out");
  TORCH_CHECK(out.numel() >= n + 1, "moe_local_offsets: out too small");
  c10::cuda::CUDAGuard g(off.device());
  moe_local_offsets_launch(P<int>(off), e0, n, P<int>(out), S());
}

void moe_router_bwd(const at::Tensor& probs, const at::Tensor& topi, const at::Tensor& topw, const at::Tensor& dw,
                    const at::Tensor& daux, const at::Tensor& counts, double coef, const at::Tensor& wg,
                    at::Tensor& dlogits, at::Tensor& dx) {
  check_f32(dx, "moe_router_bwd: dx");
  check_f32(probs, "moe_router_bwd: probs");
  check_i32(topi, "moe_router_bwd: topi");
  check_f32(topw, "moe_router_bwd: topw");
  check_f32(dw, "moe_router_bwd: dw");
  check_f32(daux, "moe_router_bwd: daux");
  check_i32(counts, "moe_router_bwd: counts");
  check_f32(wg, "moe_router_bwd: gate weight");
  TORCH_CHECK(probs.dim() == 2 && topi.dim() == 2 && wg.dim() == 2 && wg.size(0) == probs.size(1),
              "moe_router_bwd: probs [N, E], topi [N, K], gate weight [E, H]");
  {
    const int64_t n = probs.size(0), e = probs.size(1), k = topi.size(1), h = wg.size(1);
    TORCH_CHECK(topi.size(0) >= n && topw.numel() >= n * k && dw.numel() >= n * k && daux.numel() >= 1 &&
                    counts.numel() >= e && dx.numel() >= n * h,
                "moe_router_bwd: sizes");
    TORCH_CHECK((dlogits.scalar_type() == at::kBFloat16 || dlogits.scalar_type() == at::kHalf) && dlogits.dim() == 2 &&
                    dlogits.stride(1) == 1 && dlogits.size(0) >= n && dlogits.size(1) >= e,
                "moe_router_bwd: dlogits 16-bit [N, >= E]");
  }
  c10::cuda::CUDAGuard g(probs.device());
  const int N = probs.size(0), E = probs.size(1), K = topi.size(1), H = wg.size(1);
  moe_router_bwd_launch(P<float>(probs), P<int>(topi), P<float>(topw), P<float>(dw), P<float>(daux), P<int>(counts),
                        static_cast<float>(coef), N, H, E, K, P<float>(wg), P<__nv_bfloat16>(dlogits),
                        dlogits.stride(0), P<float>(dx), dlogits.scalar_type() == at::kHalf, S());
}

}  // namespace hb
