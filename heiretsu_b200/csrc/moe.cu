// Mixture-of-experts kernels: router, device-side permutation, combine.
//
// Replaces the reference's MoE data path (moe.py:34-405): nn.Linear gate +
// softmax + topk + renormalise, the load-balancing aux loss, the repeat /
// argsort / gather permutations and the Python loop over experts. Nothing
// here synchronises with the host: per-expert counts, padded segment offsets
// and row positions all stay on the device, and the grouped expert GEMMs
// (gemm_kernel.cuh, grp_mode) read the offsets directly.
//
// Layout: the N*K (token, choice) slots are grouped by expert into the
// permuted matrix; expert e owns rows [off[e], off[e+1]), its segment padded
// to a multiple of 128 rows (padding rows are zero), so every GEMM tile and
// every weight-gradient k-block belongs to exactly one expert.
#include <cuda_bf16.h>

#include "common.cuh"
#include "host_utils.h"

namespace hb {

constexpr int kMaxExperts = 64;
constexpr int kMaxTopK = 8;
constexpr int kPad = 128;

// One warp per token: logits = x . Wg^T (fp32), softmax, top-k, renormalise.
template <bool F16>
__global__ void moe_router_fwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ wg, int N,
                                      int H, int E, int K, float* __restrict__ probs, int* __restrict__ topi,
                                      float* __restrict__ topw, int* __restrict__ counts,
                                      float* __restrict__ probsum) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= N) return;
  float logit[kMaxExperts];
  const __nv_bfloat16* xr = x + (long)t * H;
  for (int e = 0; e < E; ++e) logit[e] = 0.f;
  for (int j = lane * 2; j < H; j += 64) {
    const uint32_t v = *reinterpret_cast<const uint32_t*>(xr + j);
    const float a = lo16<F16>(v), b = hi16<F16>(v);
    for (int e = 0; e < E; ++e) logit[e] += a * wg[(long)e * H + j] + b * wg[(long)e * H + j + 1];
  }
  float mx = -INFINITY;
  for (int e = 0; e < E; ++e) {
    logit[e] = warp_sum(logit[e]);
    mx = fmaxf(mx, logit[e]);
  }
  float s = 0.f;
  for (int e = 0; e < E; ++e) {
    logit[e] = __expf(logit[e] - mx);
    s += logit[e];
  }
  const float inv = 1.f / s;
  for (int e = 0; e < E; ++e) logit[e] *= inv;  // probabilities
  for (int e = lane; e < E; e += 32) probs[(long)t * E + e] = logit[e];
  // top-k (largest first, lowest index on ties)
  if (lane == 0) {
    unsigned long long taken = 0ull;
    float wsum = 0.f;
    float w[kMaxTopK];
    int id[kMaxTopK];
    for (int k = 0; k < K; ++k) {
      int best = -1;
      float bv = -1.f;
      for (int e = 0; e < E; ++e) {
        if (!((taken >> e) & 1ull) && logit[e] > bv) {
          bv = logit[e];
          best = e;
        }
      }
      taken |= 1ull << best;
      id[k] = best;
      w[k] = bv;
      wsum += bv;
    }
    for (int k = 0; k < K; ++k) {
      topi[(long)t * K + k] = id[k];
      topw[(long)t * K + k] = w[k] / wsum;
      atomicAdd(counts + id[k], 1);
    }
  }
  for (int e = lane; e < E; e += 32) atomicAdd(probsum + e, logit[e]);
}

// off[e] = first row of expert e's segment (segments padded to kPad rows);
// aux = coef * E * sum_e (count_e / (N*K)) * (probsum_e / N).
__global__ void moe_offsets_kernel(const int* __restrict__ counts, const float* __restrict__ probsum, int E, int N,
                                   int K, float coef, int* __restrict__ off, float* __restrict__ aux) {
  if (threadIdx.x == 0) {
    int acc = 0;
    float a = 0.f;
    for (int e = 0; e < E; ++e) {
      off[e] = acc;
      acc += (counts[e] + kPad - 1) / kPad * kPad;
      a += (static_cast<float>(counts[e]) / (N * K)) * (probsum[e] / N);
    }
    off[E] = acc;
    aux[0] = coef * E * a;
  }
}

// Row position of every (token, choice) slot: one block per expert, stable
// (token-major) order inside the expert via a block-wide running prefix.
__global__ void __launch_bounds__(1024) moe_positions_kernel(const int* __restrict__ topi, int NK,
                                                             const int* __restrict__ off, int* __restrict__ pos) {
  __shared__ int warp_tot[32];
  __shared__ int base_sh;
  const int e = blockIdx.x;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (threadIdx.x == 0) base_sh = off[e];
  __syncthreads();
  for (int c0 = 0; c0 < NK; c0 += 1024) {
    const int i = c0 + threadIdx.x;
    const int hit = (i < NK && topi[i] == e) ? 1 : 0;
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    const int in_warp = __popc(m & ((1u << lane) - 1u));
    if (lane == 0) warp_tot[w] = __popc(m);
    __syncthreads();
    int before = 0, total = 0;
    for (int q = 0; q < 32; ++q) {
      const int v = warp_tot[q];
      if (q < w) before += v;
      total += v;
    }
    if (hit) pos[i] = base_sh + before + in_warp;
    __syncthreads();
    if (threadIdx.x == 0) base_sh += total;
    __syncthreads();
  }
}

// Gather rows into the permuted matrix: one warp per slot. With `inv`, also
// records which routing slot (t * K + k) each window row holds (rows left at
// -1 are segment padding); the expert-parallel combine epilogue reads it.
__global__ void moe_gather_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ pos, int NK, int K,
                                  int H, __nv_bfloat16* __restrict__ xp, const int* __restrict__ off, int e0, int e1,
                                  int cap, int* status, int* __restrict__ inv) {
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= NK) return;
  const int lo = off[e0], r = pos[i];
  if (r < lo || r >= off[e1]) return;  // routed to an expert outside this rank's window
  if (!HB_DCHECK(r - lo < cap, status, 300)) return;
  if (inv != nullptr && lane == 0) inv[r - lo] = i;
  const uint4* src = reinterpret_cast<const uint4*>(x + (long)(i / K) * H);
  uint4* dst = reinterpret_cast<uint4*>(xp + (long)(r - lo) * H);
  for (int j = lane; j < H / 8; j += 32) dst[j] = src[j];
}
// out[t] = resid[t] + sum_k round16(w_tk * y_tk) over the experts of this window,
// k ascending. The terms are rounded to 16 bits exactly as the expert-parallel
// combine's slot rows are (and summed in the same order), so the combined
// output does not depend on the EP degree.
template <bool F16>
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ yp, const int* __restrict__ pos,
                                   const float* __restrict__ topw, const float* __restrict__ resid, int N, int K,
                                   int H, float* __restrict__ out, const int* __restrict__ off, int e0, int e1,
                                   int cap, int* status) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= N) return;
  const int lo = off[e0], hi = off[e1];
  for (int j = lane * 4; j < H; j += 128) {
    float4 acc = resid ? *reinterpret_cast<const float4*>(resid + (long)t * H + j) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < K; ++k) {
      const int r = pos[t * K + k];
      if (r < lo || r >= hi) continue;
      if (!HB_DCHECK(r - lo < cap, status, 301)) continue;
      const float wk = topw[(long)t * K + k];
      const uint2 raw = *reinterpret_cast<const uint2*>(yp + (long)(r - lo) * H + j);
      // each weighted term rounded to 16 bits, as the EP combine's slots hold it
      acc.x += round16<F16>(wk * lo16<F16>(raw.x));
      acc.y += round16<F16>(wk * hi16<F16>(raw.x));
      acc.z += round16<F16>(wk * lo16<F16>(raw.y));
      acc.w += round16<F16>(wk * hi16<F16>(raw.y));
    }
    *reinterpret_cast<float4*>(out + (long)t * H + j) = acc;
  }
}
template <bool F16>
__global__ void moe_combine_bwd_kernel(const float* __restrict__ dy, const __nv_bfloat16* __restrict__ yp,
                                       const int* __restrict__ pos, const float* __restrict__ topw, int N, int K,
                                       int H, __nv_bfloat16* __restrict__ dyp, float* __restrict__ dw,
                                       const int* __restrict__ off, int e0, int e1, int cap, int* status) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= N) return;
  const int lo = off[e0], hi = off[e1];
  for (int k = 0; k < K; ++k) {
    const int r = pos[t * K + k];
    if (r < lo || r >= hi || !HB_DCHECK(r - lo < cap, status, 302)) {  // another rank's expert:
      if (lane == 0) dw[(long)t * K + k] = 0.f;                           // its gradient comes from there
      continue;
    }
    const float wk = topw[(long)t * K + k];
    const long row = r - lo;
    float dot = 0.f;
    for (int j = lane * 4; j < H; j += 128) {
      const float4 g = *reinterpret_cast<const float4*>(dy + (long)t * H + j);
      const uint2 raw = *reinterpret_cast<const uint2*>(yp + row * H + j);
      dot += g.x * lo16<F16>(raw.x) + g.y * hi16<F16>(raw.x) + g.z * lo16<F16>(raw.y) + g.w * hi16<F16>(raw.y);
      *reinterpret_cast<uint2*>(dyp + row * H + j) =
          make_uint2(pack16<F16>(wk * g.x, wk * g.y), pack16<F16>(wk * g.z, wk * g.w));
    }
    dot = warp_sum(dot);
    if (lane == 0) dw[(long)t * K + k] = dot;
  }
}
__global__ void moe_unpermute_kernel(const float* __restrict__ dxp, const int* __restrict__ pos, int N, int K, int H,
                                     float* __restrict__ dx, const int* __restrict__ off, int e0, int e1, int cap,
                                     int* status) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= N) return;
  const int lo = off[e0], hi = off[e1];
  for (int j = lane * 4; j < H; j += 128) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < K; ++k) {
      const int r = pos[t * K + k];
      if (r < lo || r >= hi || !HB_DCHECK(r - lo < cap, status, 303)) continue;
      const float4 v = *reinterpret_cast<const float4*>(dxp + (long)(r - lo) * H + j);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    *reinterpret_cast<float4*>(dx + (long)t * H + j) = acc;
  }
}

// Expert-parallel combine, second half: out[t] = x[t] + sum_k slots[k][t]
// (16-bit slots filled by every EP rank's combine epilogue, then a barrier).
// Every rank adds the same values in the same order, so all replicas hold
// identical results. One warp per token, 4 columns per lane per step.
template <bool F16>
__global__ void moe_slots_reduce_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ slots, int N,
                                        int K, int H, float* __restrict__ out) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= N) return;
  for (int j = lane * 4; j < H; j += 128) {
    float4 acc = *reinterpret_cast<const float4*>(x + (long)t * H + j);
    for (int k = 0; k < K; ++k) {
      const uint2 raw = *reinterpret_cast<const uint2*>(slots + ((long)k * N + t) * H + j);
      acc.x += lo16<F16>(raw.x);
      acc.y += hi16<F16>(raw.x);
      acc.z += lo16<F16>(raw.y);
      acc.w += hi16<F16>(raw.y);
    }
    *reinterpret_cast<float4*>(out + (long)t * H + j) = acc;
  }
}

// Offsets of the window's experts relative to its first row: out[i] = off[e0 + i] - off[e0], i = 0 .. n.
__global__ void moe_local_offsets_kernel(const int* __restrict__ off, int e0, int n, int* __restrict__ out) {
  const int i = threadIdx.x;
  if (i <= n) out[i] = off[e0 + i] - off[e0];
}

// Router backward, one warp per token. Upstream: dw (gradient of the
// renormalised top-k weights) and daux (gradient of the aux loss). Produces
// dlogits (16-bit [N, E], for the gate weight gradient GEMM) and adds
// dlogits . Wg to dx (fp32).
template <bool F16>
__global__ void moe_router_bwd_kernel(const float* __restrict__ probs, const int* __restrict__ topi,
                                      const float* __restrict__ topw, const float* __restrict__ dw,
                                      const float* __restrict__ daux, const int* __restrict__ counts, float coef,
                                      int N, int H, int E, int K, const float* __restrict__ wg,
                                      __nv_bfloat16* __restrict__ dlogits, long ld_dl, float* __restrict__ dx) {
  const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= N) return;
  float p[kMaxExperts], dp[kMaxExperts];
  for (int e = 0; e < E; ++e) {
    p[e] = probs[(long)t * E + e];
    // aux = coef * E * sum_e f_e * mean_t p_{t,e}, with f_e = count_e / (N*K) held constant
    dp[e] = daux[0] * coef * E * (static_cast<float>(counts[e]) / (N * K)) / N;
  }
  // w_k = p_{i_k} / S with S = sum_j p_{i_j}: dL/dp_{i_k} += (dw_k - sum_j dw_j w_j) / S
  float S = 0.f, dot = 0.f;
  for (int k = 0; k < K; ++k) {
    S += p[topi[(long)t * K + k]];
    dot += dw[(long)t * K + k] * topw[(long)t * K + k];
  }
  for (int k = 0; k < K; ++k) dp[topi[(long)t * K + k]] += (dw[(long)t * K + k] - dot) / S;
  // softmax: dlogit_e = p_e * (dp_e - sum_j p_j dp_j)
  float pdp = 0.f;
  for (int e = 0; e < E; ++e) pdp += p[e] * dp[e];
  float dl[kMaxExperts];
  for (int e = 0; e < E; ++e) dl[e] = p[e] * (dp[e] - pdp);
  for (int e = lane; e < E; e += 32) reinterpret_cast<uint16_t*>(dlogits)[(long)t * ld_dl + e] = from_f32<F16>(dl[e]);
  for (int j = lane; j < H; j += 32) {
    float acc = 0.f;
    for (int e = 0; e < E; ++e) acc += dl[e] * wg[(long)e * H + j];
    dx[(long)t * H + j] += acc;
  }
}

// ---------------------------------------------------------------------------
void moe_route_launch(const __nv_bfloat16* x, const float* wg, int N, int H, int E, int K, float coef, float* probs,
                      int* topi, float* topw, int* counts, float* probsum, int* off, float* aux, int* pos, bool f16,
                      cudaStream_t s) {
  if (E > kMaxExperts || K > kMaxTopK || K > E || H % 8) throw std::runtime_error("moe: unsupported E / K / H");
  HB_CUDA_CHECK(cudaMemsetAsync(counts, 0, sizeof(int) * E, s));
  HB_CUDA_CHECK(cudaMemsetAsync(probsum, 0, sizeof(float) * E, s));
  (f16 ? moe_router_fwd_kernel<true> : moe_router_fwd_kernel<false>)<<<(N * 32 + 255) / 256, 256, 0, s>>>(
      x, wg, N, H, E, K, probs, topi, topw, counts, probsum);
  HB_CUDA_CHECK(cudaGetLastError());
  moe_offsets_kernel<<<1, 32, 0, s>>>(counts, probsum, E, N, K, coef, off, aux);
  HB_CUDA_CHECK(cudaGetLastError());
  moe_positions_kernel<<<E, 1024, 0, s>>>(topi, N * K, off, pos);
  HB_CUDA_CHECK(cudaGetLastError());
}

void moe_gather_launch(const __nv_bfloat16* x, const int* pos, int N, int K, int H, __nv_bfloat16* xp,
                       const int* off, int e0, int e1, int cap, int* status, int* inv, cudaStream_t s) {
  if (inv != nullptr) HB_CUDA_CHECK(cudaMemsetAsync(inv, 0xFF, sizeof(int) * cap, s));  // -1: padding rows
  moe_gather_kernel<<<(N * K * 32 + 255) / 256, 256, 0, s>>>(x, pos, N * K, K, H, xp, off, e0, e1, cap, status, inv);
  HB_CUDA_CHECK(cudaGetLastError());
}

void moe_combine_launch(const __nv_bfloat16* yp, const int* pos, const float* topw, const float* resid, int N, int K,
                        int H, float* out, const int* off, int e0, int e1, int cap, int* status, bool f16,
                        cudaStream_t s) {
  (f16 ? moe_combine_kernel<true> : moe_combine_kernel<false>)<<<(N * 32 + 255) / 256, 256, 0, s>>>(
      yp, pos, topw, resid, N, K, H, out, off, e0, e1, cap, status);
  HB_CUDA_CHECK(cudaGetLastError());
}

void moe_combine_bwd_launch(const float* dy, const __nv_bfloat16* yp, const int* pos, const float* topw, int N,
                            int K, int H, __nv_bfloat16* dyp, float* dw, const int* off, int e0, int e1, int cap,
                            int* status, bool f16, cudaStream_t s) {
  (f16 ? moe_combine_bwd_kernel<true> : moe_combine_bwd_kernel<false>)<<<(N * 32 + 255) / 256, 256, 0, s>>>(
      dy, yp, pos, topw, N, K, H, dyp, dw, off, e0, e1, cap, status);
  HB_CUDA_CHECK(cudaGetLastError());
}

void moe_unpermute_launch(const float* dxp, const int* pos, int N, int K, int H, float* dx, const int* off, int e0,
                          int e1, int cap, int* status, cudaStream_t s) {
  moe_unpermute_kernel<<<(N * 32 + 255) / 256, 256, 0, s>>>(dxp, pos, N, K, H, dx, off, e0, e1, cap, status);
  HB_CUDA_CHECK(cudaGetLastError());
}

void moe_slots_reduce_launch(const float* x, const __nv_bfloat16* slots, int N, int K, int H, float* out, bool f16,
                             cudaStream_t s) {
  if (H % 4) throw std::runtime_error("moe_slots_reduce: H must be a multiple of 4");
  (f16 ? moe_slots_reduce_kernel<true> : moe_slots_reduce_kernel<false>)<<<(N * 32 + 255) / 256, 256, 0, s>>>(
      x, slots, N, K, H, out);
  HB_CUDA_CHECK(cudaGetLastError());
}

void moe_local_offsets_launch(const int* off, int e0, int n, int* out, cudaStream_t s) {
  if (n + 1 > 1024) throw std::runtime_error("moe_local_offsets: too many experts");
  moe_local_offsets_kernel<<<1, 1024, 0, s>>>(off, e0, n, out);
  HB_CUDA_CHECK(cudaGetLastError());
}

void moe_router_bwd_launch(const float* probs, const int* topi, const float* topw, const float* dw, const float* daux,
                           const int* counts, float coef, int N, int H, int E, int K, const float* wg,
                           __nv_bfloat16* dlogits, long ld_dl, float* dx, bool f16, cudaStream_t s) {
  (f16 ? moe_router_bwd_kernel<true> : moe_router_bwd_kernel<false>)<<<(N * 32 + 255) / 256, 256, 0, s>>>(
      probs, topi, topw, dw, daux, counts, coef, N, H, E, K, wg, dlogits, ld_dl, dx);
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
