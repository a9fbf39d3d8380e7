// Token + position embedding (forward gather, backward scatter-add) and the
// fused AdamW / gradient-norm kernels over flat parameter buffers.
//
// Replaces wte(idx) + wpe(pos) (reference gpt_model.py:274-275,
// pipeline.py:111-122), torch.optim.AdamW (train.py:346-351) and
// clip_grad_norm_ (train.py:446).
#include <cuda_bf16.h>

#include "common.cuh"
#include "host_utils.h"

namespace hb {

// out fp32 [B*T, H] = wte[idx] + wpe[t]. One warp per token row, float4.
// A token id outside [0, V) names no row of wte (nn.Embedding rejects it): its
// output row becomes NaN (so the loss and the step's gradient norm are NaN and
// the optimizer skips the step) and the status word records the bad argument.
__global__ void embed_fwd_kernel(const int64_t* __restrict__ idx, const float* __restrict__ wte,
                                 const float* __restrict__ wpe, float* __restrict__ out, int M, int T, int H, int V,
                                 int* status) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const long tok = idx[row];
  const int t = row % T;
  float4* o = reinterpret_cast<float4*>(out + (long)row * H);
  if (tok < 0 || tok >= V) {
    if (lane == 0) record_error(status, kBadArg, 410);
    for (int j = lane; j < H / 4; j += 32) o[j] = make_float4(NAN, NAN, NAN, NAN);
    return;
  }
  const float4* a = reinterpret_cast<const float4*>(wte + tok * H);
  const float4* p = reinterpret_cast<const float4*>(wpe + (long)t * H);
  for (int j = lane; j < H / 4; j += 32) {
    const float4 x = a[j], y = p[j];
    o[j] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
  }
}

// dwte[idx[m]] += dx[m] (vector atomics; rows repeat across the batch). Token ids
// outside [0, V) (reported by the forward) add nothing.
__global__ void embed_bwd_tok_kernel(const int64_t* __restrict__ idx, const float* __restrict__ dx,
                                     float* __restrict__ dwte, int M, int H, int V) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const long tok = idx[row];
  if (tok < 0 || tok >= V) return;
  const float4* g = reinterpret_cast<const float4*>(dx + (long)row * H);
  float4* d = reinterpret_cast<float4*>(dwte + tok * H);
  for (int j = lane; j < H / 4; j += 32) atomicAdd(d + j, g[j]);
}

// dwpe[t, c] += sum_b dx[b, t, c]: one thread per (t, c), fixed order over b.
__global__ void embed_bwd_pos_kernel(const float* __restrict__ dx, float* __restrict__ dwpe, int B, int T, int H) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)T * H) return;
  float s = 0.f;
  for (int b = 0; b < B; ++b) s += dx[(long)b * T * H + i];
  dwpe[i] += s;
}

void embed_fwd_launch(const int64_t* idx, const float* wte, const float* wpe, float* out, int B, int T, int H, int V,
                      int* status, cudaStream_t s) {
  if (H % 4) throw std::runtime_error("embedding: H must be a multiple of 4");
  const int M = B * T;
  embed_fwd_kernel<<<(M * 32 + 255) / 256, 256, 0, s>>>(idx, wte, wpe, out, M, T, H, V, status);
  HB_CUDA_CHECK(cudaGetLastError());
}

void embed_bwd_launch(const int64_t* idx, const float* dx, float* dwte, float* dwpe, int B, int T, int H, int V,
                      cudaStream_t s) {
  if (H % 4) throw std::runtime_error("embedding: H must be a multiple of 4");
  const int M = B * T;
  if (dwte) {
    embed_bwd_tok_kernel<<<(M * 32 + 255) / 256, 256, 0, s>>>(idx, dx, dwte, M, H, V);
    HB_CUDA_CHECK(cudaGetLastError());
  }
  if (dwpe) {
    const long n = (long)T * H;
    embed_bwd_pos_kernel<<<(n + 255) / 256, 256, 0, s>>>(dx, dwpe, B, T, H);
    HB_CUDA_CHECK(cudaGetLastError());
  }
}

// ----------------------------------------------------------------------------
// Gradient norm: partial sums of squares (deterministic two-pass).
// ----------------------------------------------------------------------------
constexpr int SQ_THREADS = 512;

__global__ void __launch_bounds__(SQ_THREADS) sumsq_partial_kernel(const float* __restrict__ x, long n,
                                                                   float* __restrict__ part) {
  __shared__ float sh[SQ_THREADS / 32];
  float s = 0.f;
  const long n4 = n >> 2;
  const float4* x4 = reinterpret_cast<const float4*>(x);
  for (long i = (long)blockIdx.x * SQ_THREADS + threadIdx.x; i < n4; i += (long)gridDim.x * SQ_THREADS) {
    const float4 v = x4[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (long i = n4 * 4 + (long)blockIdx.x * SQ_THREADS + threadIdx.x; i < n; i += (long)gridDim.x * SQ_THREADS) {
    s += x[i] * x[i];
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = (threadIdx.x < SQ_THREADS / 32) ? sh[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) part[blockIdx.x] = v;
  }
}

__global__ void sumsq_final_kernel(const float* __restrict__ part, int nparts, float weight, float* out,
                                   int accumulate) {
  __shared__ float sh[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += part[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = (threadIdx.x < (int)(blockDim.x / 32)) ? sh[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) out[0] = (accumulate ? out[0] : 0.f) + weight * v;
  }
}

int sumsq_num_parts(int device) { return 2 * num_sms(device); }

void sumsq_launch(const float* x, long n, float* part, int nparts, float weight, float* out, bool accumulate,
                  cudaStream_t s) {
  sumsq_partial_kernel<<<nparts, SQ_THREADS, 0, s>>>(x, n, part);
  HB_CUDA_CHECK(cudaGetLastError());
  sumsq_final_kernel<<<1, 1024, 0, s>>>(part, nparts, weight, out, accumulate ? 1 : 0);
  HB_CUDA_CHECK(cudaGetLastError());
}

// coef[0] = min(1, max_norm / (sqrt(norm2) + 1e-6)) (torch clip_grad_norm_ semantics);
// with a non-finite norm the step is skipped by AdamW (coef = NaN sentinel).
// With a loss scale S (fp16, `lscale` != nullptr) the gradients hold S * g:
// the norm is unscaled first (the order of GradScaler.unscale_ then
// clip_grad_norm_), and 1/S is folded into the coefficient AdamW applies.
__global__ void clip_coef_kernel(const float* norm2, float max_norm, float* coef, float* norm_out,
                                 const float* lscale) {
  const float inv_s = lscale ? 1.f / lscale[0] : 1.f;
  const float nrm = sqrtf(norm2[0]) * inv_s;
  if (norm_out) norm_out[0] = nrm;
  float c = 1.f;
  if (max_norm > 0.f) c = fminf(1.f, max_norm / (nrm + 1e-6f));
  coef[0] = isfinite(nrm) ? c * inv_s : NAN;
}

void clip_coef_launch(const float* norm2, float max_norm, float* coef, float* norm_out, const float* lscale,
                      cudaStream_t s) {
  clip_coef_kernel<<<1, 1, 0, s>>>(norm2, max_norm, coef, norm_out, lscale);
  HB_CUDA_CHECK(cudaGetLastError());
}

// Dynamic loss scale (fp16), torch.cuda.amp.GradScaler's rule kept on the
// device: state = {scale, steps since the last non-finite step}. After a
// skipped step (coef NaN) the scale is multiplied by `backoff` and the count
// restarts; after `interval` finite steps in a row it is multiplied by `growth`.
__global__ void loss_scale_update_kernel(const float* coef, float* state, float growth, float backoff,
                                         int interval) {
  if (isnan(coef[0])) {
    state[0] *= backoff;
    state[1] = 0.f;
  } else {
    state[1] += 1.f;
    if (state[1] >= static_cast<float>(interval)) {
      state[0] *= growth;
      state[1] = 0.f;
    }
  }
}

void loss_scale_update_launch(const float* coef, float* state, float growth, float backoff, int interval,
                              cudaStream_t s) {
  loss_scale_update_kernel<<<1, 1, 0, s>>>(coef, state, growth, backoff, interval);
  HB_CUDA_CHECK(cudaGetLastError());
}

// ----------------------------------------------------------------------------
// AdamW (torch.optim.AdamW semantics, decoupled weight decay on every element)
//   g = grad * gscale * coef        (gscale: 1/loss_scale for fp16, coef: clip)
//   p *= 1 - lr*wd;  m = b1 m + (1-b1) g;  v = b2 v + (1-b2) g^2
//   p -= (lr / bc1) * m / (sqrt(v) / sqrt(bc2) + eps)
// and the bf16 shadow copy used by the GEMMs is refreshed in the same pass.
// A NaN `coef` (non-finite gradients) skips the update entirely.
// Hyper-parameters live in device memory so a captured graph can replay steps.
// ----------------------------------------------------------------------------
struct AdamHyper {
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, gscale;
};

template <bool F16>
__global__ void __launch_bounds__(256) adamw_kernel(float* __restrict__ p, const float* __restrict__ g,
                                                    float* __restrict__ m, float* __restrict__ v,
                                                    __nv_bfloat16* __restrict__ p16, long n,
                                                    const AdamHyper* __restrict__ hp,
                                                    const float* __restrict__ coef_ptr) {
  const float coef = coef_ptr ? coef_ptr[0] : 1.f;
  if (isnan(coef)) return;
  const AdamHyper h = *hp;
  const float gs = h.gscale * coef;
  const float decay = 1.f - h.lr * h.wd;
  const float step = h.lr / h.bc1;
  const long n4 = n >> 2;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    float4 pp = reinterpret_cast<float4*>(p)[i];
    const float4 gg = reinterpret_cast<const float4*>(g)[i];
    float4 mm = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pa = &pp.x;
    const float* ga = &gg.x;
    float* ma = &mm.x;
    float* va = &vv.x;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float gq = ga[q] * gs;
      ma[q] = h.beta1 * ma[q] + (1.f - h.beta1) * gq;
      va[q] = h.beta2 * va[q] + (1.f - h.beta2) * gq * gq;
      pa[q] = pa[q] * decay - step * ma[q] / (sqrtf(va[q]) / h.bc2_sqrt + h.eps);
    }
    reinterpret_cast<float4*>(p)[i] = pp;
    reinterpret_cast<float4*>(m)[i] = mm;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (p16) {
      reinterpret_cast<uint2*>(p16)[i] = make_uint2(pack16<F16>(pp.x, pp.y), pack16<F16>(pp.z, pp.w));
    }
  }
  for (long i = n4 * 4 + (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float gq = g[i] * gs;
    m[i] = h.beta1 * m[i] + (1.f - h.beta1) * gq;
    v[i] = h.beta2 * v[i] + (1.f - h.beta2) * gq * gq;
    p[i] = p[i] * decay - step * m[i] / (sqrtf(v[i]) / h.bc2_sqrt + h.eps);
    if (p16) reinterpret_cast<uint16_t*>(p16)[i] = from_f32<F16>(p[i]);
  }
}

void adamw_launch(float* p, const float* g, float* m, float* v, __nv_bfloat16* p16, long n, const void* hyper,
                  const float* coef, bool f16, cudaStream_t s) {
  if (n == 0) return;
  const int grid = 4 * num_sms(current_device());
  (f16 ? adamw_kernel<true> : adamw_kernel<false>)<<<grid, 256, 0, s>>>(
      p, g, m, v, p16, n, reinterpret_cast<const AdamHyper*>(hyper), coef);
  HB_CUDA_CHECK(cudaGetLastError());
}

// Plain fp32 -> 16-bit copy (refresh of the GEMM weight shadow after a load).
template <bool F16>
__global__ void f32_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, long n) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    reinterpret_cast<uint16_t*>(y)[i] = from_f32<F16>(x[i]);
}

void f32_to_bf16_launch(const float* x, __nv_bfloat16* y, long n, bool f16, cudaStream_t s) {
  if (n == 0) return;
  (f16 ? f32_to_bf16_kernel<true> : f32_to_bf16_kernel<false>)<<<4 * num_sms(current_device()), 256, 0, s>>>(x, y, n);
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
