// Softmax cross-entropy over the vocabulary and the MoE aux-loss reduction.
//
// Replaces F.cross_entropy on materialised fp32 logits (reference
// gpt_model.py:284-287, pipeline.py:139-142). The logits stay in 16 bits (bf16
// or fp16, written by the lm_head GEMM, row stride Vp >= V, a multiple of 8):
//   forward   per row: lse = log sum_j exp(l_j) over j < V; loss = lse - l_t
//   backward  in place: l_j <- (softmax_j - [j == t]) * scale (0 for j >= V)
// Targets equal to `ignore_index` contribute no loss and a zero gradient row.
// By default one kernel does both (ce_fused_kernel: the gradient is written
// while the row is still in L2).
#include <cuda_bf16.h>

#include "common.cuh"
#include "host_utils.h"

namespace hb {

template <int THREADS>
__device__ __forceinline__ float block_reduce_max(float v, float* sh) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < THREADS / 32) ? sh[l] : -INFINITY;
    v = warp_max(v);
    if (l == 0) sh[0] = v;
  }
  __syncthreads();
  v = sh[0];
  __syncthreads();
  return v;
}

template <int THREADS>
__device__ __forceinline__ float block_reduce_sum(float v, float* sh) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < THREADS / 32) ? sh[l] : 0.f;
    v = warp_sum(v);
    if (l == 0) sh[0] = v;
  }
  __syncthreads();
  v = sh[0];
  __syncthreads();
  return v;
}

constexpr int CE_THREADS = 512;

// One CTA per row. Online (max, sum-exp) per thread over 8-element chunks.
template <bool F16>
__global__ void __launch_bounds__(CE_THREADS) ce_fwd_kernel(const __nv_bfloat16* __restrict__ logits, long ld, int V,
                                                            const int64_t* __restrict__ targets, int ignore_index,
                                                            float* __restrict__ lse_out,
                                                            float* __restrict__ loss_rows, int* status) {
  __shared__ float sh[32];
  const long row = blockIdx.x;
  const __nv_bfloat16* lr = logits + row * ld;
  float m = -INFINITY, s = 0.f;
  const int nchunk = V >> 3;  // full 8-wide chunks
  for (int c = threadIdx.x; c < nchunk; c += CE_THREADS) {
    const uint4 raw = *reinterpret_cast<const uint4*>(lr + c * 8);
    const uint16_t* e = reinterpret_cast<const uint16_t*>(&raw);
    float v[8];
    float cm = -INFINITY;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      v[q] = to_f32<F16>(e[q]);
      cm = fmaxf(cm, v[q]);
    }
    const float nm = fmaxf(m, cm);
    float acc = s * __expf(m - nm);
#pragma unroll
    for (int q = 0; q < 8; ++q) acc += __expf(v[q] - nm);
    m = nm;
    s = acc;
  }
  for (int j = nchunk * 8 + threadIdx.x; j < V; j += CE_THREADS) {
    const float v = to_f32<F16>(reinterpret_cast<const uint16_t*>(lr)[j]);
    const float nm = fmaxf(m, v);
    s = s * __expf(m - nm) + __expf(v - nm);
    m = nm;
  }
  const float gm = block_reduce_max<CE_THREADS>(m, sh);
  const float gs = block_reduce_sum<CE_THREADS>((m == -INFINITY) ? 0.f : s * __expf(m - gm), sh);
  if (threadIdx.x == 0) {
    const float lse = gm + __logf(gs);
    lse_out[row] = lse;
    const int64_t t = targets[row];
    if (t == ignore_index) {
      loss_rows[row] = 0.f;
    } else if (t < 0 || t >= V) {  // no such class (F.cross_entropy rejects it): NaN row, status set
      record_error(status, kBadArg, 400);
      loss_rows[row] = NAN;
    } else {
      loss_rows[row] = lse - to_f32<F16>(reinterpret_cast<const uint16_t*>(lr)[t]);
    }
  }
}

// In-place gradient: l_j <- (exp(l_j - lse) - [j == t]) * scale; j in [V, Vp) -> 0.
template <bool F16>
__global__ void __launch_bounds__(CE_THREADS) ce_bwd_kernel(__nv_bfloat16* __restrict__ logits, long ld, int V,
                                                            int Vp, const int64_t* __restrict__ targets,
                                                            int ignore_index, const float* __restrict__ lse_in,
                                                            const float* __restrict__ scale_ptr, float scale_mul) {
  const long row = blockIdx.x;
  __nv_bfloat16* lr = logits + row * ld;
  const int64_t t = targets[row];
  // an out-of-range target (already reported by the forward) poisons its row's gradient
  const float scale = (t == ignore_index) ? 0.f
                      : (t < 0 || t >= V) ? NAN
                                          : scale_mul * (scale_ptr ? *scale_ptr : 1.f);
  const float lse = lse_in[row];
  const int nchunk = Vp >> 3;
  for (int c = threadIdx.x; c < nchunk; c += CE_THREADS) {
    uint4 raw = *reinterpret_cast<const uint4*>(lr + c * 8);
    const uint16_t* e = reinterpret_cast<const uint16_t*>(&raw);
    float g[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int j = c * 8 + q;
      g[q] = (j < V) ? (__expf(to_f32<F16>(e[q]) - lse) - (j == t ? 1.f : 0.f)) * scale : 0.f;
    }
    *reinterpret_cast<uint4*>(lr + c * 8) =
        make_uint4(pack16<F16>(g[0], g[1]), pack16<F16>(g[2], g[3]), pack16<F16>(g[4], g[5]), pack16<F16>(g[6], g[7]));
  }
}

// Forward and gradient in one pass per row (the model's default; HB_CE_FUSED=0
// on the host side selects the two-kernel pair): the log-sum-exp pass reads the row from DRAM, and the gradient
// pass that follows in the same CTA re-reads it while it is still in L2
// (a 50304-wide bf16 row is 100 KB; the CTAs in flight hold a few tens of MB),
// so the logits cross DRAM once each way instead of read twice and written
// once. The gradient is scaled by *scale_ptr, which the caller computes before
// the launch (the expected upstream gradient over the number of counted rows);
// ce_rescale_kernel corrects it in backward when the actual upstream gradient
// differs. The target logit is read before the row is overwritten.
template <bool F16>
__global__ void __launch_bounds__(CE_THREADS) ce_fused_kernel(__nv_bfloat16* __restrict__ logits, long ld, int V,
                                                              int Vp, const int64_t* __restrict__ targets,
                                                              int ignore_index, float* __restrict__ lse_out,
                                                              float* __restrict__ loss_rows,
                                                              const float* __restrict__ scale_ptr, int* status) {
  __shared__ float sh[32];
  const long row = blockIdx.x;
  __nv_bfloat16* lr = logits + row * ld;
  const int64_t t = targets[row];
  const bool counted = (t != ignore_index);
  // A target outside [0, V) is no class (F.cross_entropy rejects it): its row's
  // loss and gradient become NaN (so the step is skipped) and the status is set.
  const bool bad = counted && (t < 0 || t >= V);
  if (bad && threadIdx.x == 0) record_error(status, kBadArg, 401);
  const float target_logit =
      (threadIdx.x == 0 && counted && !bad) ? to_f32<F16>(reinterpret_cast<const uint16_t*>(lr)[t]) : 0.f;
  float m = -INFINITY, s = 0.f;
  const int nchunk = V >> 3;
  for (int c = threadIdx.x; c < nchunk; c += CE_THREADS) {
    const uint4 raw = *reinterpret_cast<const uint4*>(lr + c * 8);
    const uint16_t* e = reinterpret_cast<const uint16_t*>(&raw);
    float v[8];
    float cm = -INFINITY;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      v[q] = to_f32<F16>(e[q]);
      cm = fmaxf(cm, v[q]);
    }
    const float nm = fmaxf(m, cm);
    float acc = s * __expf(m - nm);
#pragma unroll
    for (int q = 0; q < 8; ++q) acc += __expf(v[q] - nm);
    m = nm;
    s = acc;
  }
  for (int j = nchunk * 8 + threadIdx.x; j < V; j += CE_THREADS) {
    const float v = to_f32<F16>(reinterpret_cast<const uint16_t*>(lr)[j]);
    const float nm = fmaxf(m, v);
    s = s * __expf(m - nm) + __expf(v - nm);
    m = nm;
  }
  // block reductions end with a barrier: every thread has finished reading the
  // row (and thread 0 its target logit) before any gradient is written below
  const float gm = block_reduce_max<CE_THREADS>(m, sh);
  const float gs = block_reduce_sum<CE_THREADS>((m == -INFINITY) ? 0.f : s * __expf(m - gm), sh);
  const float lse = gm + __logf(gs);
  if (threadIdx.x == 0) {
    lse_out[row] = lse;
    loss_rows[row] = bad ? NAN : (counted ? lse - target_logit : 0.f);
  }
  const float scale = bad ? NAN : (counted ? *scale_ptr : 0.f);
  const int nchunk_p = Vp >> 3;
  for (int c = threadIdx.x; c < nchunk_p; c += CE_THREADS) {
    uint4 raw = *reinterpret_cast<const uint4*>(lr + c * 8);
    const uint16_t* e = reinterpret_cast<const uint16_t*>(&raw);
    float g[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int j = c * 8 + q;
      g[q] = (j < V) ? (__expf(to_f32<F16>(e[q]) - lse) - (j == t ? 1.f : 0.f)) * scale : 0.f;
    }
    *reinterpret_cast<uint4*>(lr + c * 8) =
        make_uint4(pack16<F16>(g[0], g[1]), pack16<F16>(g[2], g[3]), pack16<F16>(g[4], g[5]), pack16<F16>(g[6], g[7]));
  }
}

// g *= actual / expected over [M, Vp] bf16 (row stride ld); every CTA returns at
// once when the two device scalars are equal (the usual case).
template <bool F16>
__global__ void __launch_bounds__(256) ce_rescale_kernel(__nv_bfloat16* __restrict__ g, long ld, int M, int Vp,
                                                         const float* __restrict__ actual,
                                                         const float* __restrict__ expected) {
  const float a = *actual, e = *expected;
  if (a == e) return;
  const float r = a / e;
  const long per_row = Vp >> 3;
  const long n = (long)M * per_row;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long row = i / per_row, c = i % per_row;
    uint4* ptr = reinterpret_cast<uint4*>(g + row * ld + c * 8);
    uint4 raw = *ptr;
    const uint16_t* x = reinterpret_cast<const uint16_t*>(&raw);
    float v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = to_f32<F16>(x[q]) * r;
    *ptr = make_uint4(pack16<F16>(v[0], v[1]), pack16<F16>(v[2], v[3]), pack16<F16>(v[4], v[5]), pack16<F16>(v[6], v[7]));
  }
}

// out[0] (+)= mean over rows of loss_rows (rows with ignore_index excluded from the count).
__global__ void __launch_bounds__(1024) mean_loss_kernel(const float* __restrict__ loss_rows,
                                                         const int64_t* __restrict__ targets, int M,
                                                         int ignore_index, float* __restrict__ out,
                                                         float* __restrict__ count_out) {
  __shared__ float sh[32];
  float s = 0.f, n = 0.f;
  for (int i = threadIdx.x; i < M; i += 1024) {
    s += loss_rows[i];
    n += (targets[i] == ignore_index) ? 0.f : 1.f;
  }
  s = block_reduce_sum<1024>(s, sh);
  n = block_reduce_sum<1024>(n, sh);
  if (threadIdx.x == 0) {
    out[0] = s / fmaxf(n, 1.f);
    if (count_out) count_out[0] = n;
  }
}

void ce_fwd_launch(const __nv_bfloat16* logits, long ld, int M, int V, const int64_t* targets, int ignore_index,
                   float* lse, float* loss_rows, float* loss_mean, float* count, bool f16, int* status,
                   cudaStream_t s) {
  if (ld % 8 != 0) throw std::runtime_error("cross_entropy: logits row stride must be a multiple of 8");
  if (M == 0) return;
  (f16 ? ce_fwd_kernel<true> : ce_fwd_kernel<false>)<<<M, CE_THREADS, 0, s>>>(logits, ld, V, targets, ignore_index, lse,
                                                                             loss_rows, status);
  HB_CUDA_CHECK(cudaGetLastError());
  mean_loss_kernel<<<1, 1024, 0, s>>>(loss_rows, targets, M, ignore_index, loss_mean, count);
  HB_CUDA_CHECK(cudaGetLastError());
}

void ce_fused_launch(__nv_bfloat16* logits, long ld, int M, int V, int Vp, const int64_t* targets, int ignore_index,
                     float* lse, float* loss_rows, float* loss_mean, const float* scale_ptr, bool f16,
                     int* status, cudaStream_t s) {
  if (ld % 8 != 0 || Vp % 8 != 0) throw std::runtime_error("cross_entropy: Vp and row stride must be multiples of 8");
  if (M == 0) return;
  (f16 ? ce_fused_kernel<true> : ce_fused_kernel<false>)<<<M, CE_THREADS, 0, s>>>(logits, ld, V, Vp, targets,
                                                                                 ignore_index, lse, loss_rows,
                                                                                 scale_ptr, status);
  HB_CUDA_CHECK(cudaGetLastError());
  mean_loss_kernel<<<1, 1024, 0, s>>>(loss_rows, targets, M, ignore_index, loss_mean, nullptr);
  HB_CUDA_CHECK(cudaGetLastError());
}

void ce_rescale_launch(__nv_bfloat16* g, long ld, int M, int Vp, const float* actual, const float* expected,
                       bool f16, cudaStream_t s) {
  if (ld % 8 != 0 || Vp % 8 != 0) throw std::runtime_error("cross_entropy: Vp and row stride must be multiples of 8");
  if (M == 0) return;
  const long n = (long)M * (Vp >> 3);
  const int blocks = (int)std::min<long>((n + 255) / 256, 4L * num_sms(current_device()));
  (f16 ? ce_rescale_kernel<true> : ce_rescale_kernel<false>)<<<blocks, 256, 0, s>>>(g, ld, M, Vp, actual, expected);
  HB_CUDA_CHECK(cudaGetLastError());
}

void ce_bwd_launch(__nv_bfloat16* logits, long ld, int M, int V, int Vp, const int64_t* targets, int ignore_index,
                   const float* lse, const float* scale_ptr, float scale_mul, bool f16, cudaStream_t s) {
  if (ld % 8 != 0 || Vp % 8 != 0) throw std::runtime_error("cross_entropy: Vp and row stride must be multiples of 8");
  if (M == 0) return;
  (f16 ? ce_bwd_kernel<true> : ce_bwd_kernel<false>)<<<M, CE_THREADS, 0, s>>>(logits, ld, V, Vp, targets, ignore_index,
                                                                             lse, scale_ptr, scale_mul);
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb

// ============================================================================
// Allocation-free cross-entropy forward (declared in noalloc.h).
//
// Same kernels as ce_fwd_launch, but the per-row loss scratch lives in a
// file-scope device array instead of a buffer the caller allocates. See
// noalloc.h for who needs this, its limits and its concurrency rules.
// ============================================================================
#include <mutex>

#include "noalloc.h"

namespace {

// Per-row losses of the most recent call (every call overwrites rows [0, M)).
// Held by every GPU that loads the library, until the process exits.
static __device__ __align__(256) float g_ce_noalloc_rows[HB_CE_NOALLOC_MAX_ROWS];

std::mutex g_ce_noalloc_mu;
float* g_ce_noalloc_ptr[64] = {};

// Device address of the scratch array for the current device; resolved once
// per device (the host-side name of the array is only a stand-in).
int ce_noalloc_scratch(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HB_NOALLOC_ERR_CUDA;
  std::lock_guard<std::mutex> lk(g_ce_noalloc_mu);
  if (g_ce_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress((void**)&p, g_ce_noalloc_rows) != cudaSuccess || p == nullptr) return HB_NOALLOC_ERR_CUDA;
    g_ce_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_ce_noalloc_ptr[dev];
  return HB_NOALLOC_OK;
}

}  // namespace

extern "C" int hb_cross_entropy_fwd_noalloc(const void* logits, long ld, int M, int V, const int64_t* targets,
                                            int ignore_index, float* lse, float* loss_mean, cudaStream_t stream) {
  if (logits == nullptr || targets == nullptr || lse == nullptr || loss_mean == nullptr) return HB_NOALLOC_ERR_ARG;
  if (M < 0 || V <= 0 || ld < V || ld % 8 != 0) return HB_NOALLOC_ERR_ARG;
  // Rows are read with 16-byte vector loads: the first row must start 16-byte aligned.
  if (reinterpret_cast<uintptr_t>(logits) % 16 != 0) return HB_NOALLOC_ERR_ARG;
  if (M > HB_CE_NOALLOC_MAX_ROWS) return HB_NOALLOC_ERR_TOO_LARGE;
  if (M == 0) return HB_NOALLOC_OK;
  float* rows = nullptr;
  const int rc = ce_noalloc_scratch(&rows);
  if (rc != HB_NOALLOC_OK) return rc;
  hb::ce_fwd_kernel<false><<<M, hb::CE_THREADS, 0, stream>>>(static_cast<const __nv_bfloat16*>(logits), ld, V, targets,
                                                             ignore_index, lse, rows, nullptr);
  if (cudaGetLastError() != cudaSuccess) return HB_NOALLOC_ERR_CUDA;
  hb::mean_loss_kernel<<<1, 1024, 0, stream>>>(rows, targets, M, ignore_index, loss_mean, nullptr);
  if (cudaGetLastError() != cudaSuccess) return HB_NOALLOC_ERR_CUDA;
  return HB_NOALLOC_OK;
}
