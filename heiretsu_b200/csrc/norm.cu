// LayerNorm forward/backward and column reductions (bias gradients).
//
// Replaces nn.LayerNorm (reference gpt_model.py:111-119, :237, pipeline.py:83)
// and the bias-gradient reductions autograd performs for tp_linear.py:226/:310.
//
// Layout: rows of H contiguous elements (H % 4 == 0, H <= 2048). One warp per
// row; each lane keeps its share of the row in registers as float4, so the
// row is read from HBM once and written once.
#include <cuda_bf16.h>
#include <cstdlib>

#include "common.cuh"
#include "dropout.cuh"
#include "host_utils.h"

namespace hb {

// Rows are processed one per warp; each lane holds V4 float4 of the row
// (V4 = ceil(H / 128), a template parameter so no register is wasted).
// The backward kernel runs two CTAs per SM whose warps stride over the rows
// (all loads of a row issued before any arithmetic), keeps the dgamma /
// dbeta partials in registers, sums its warps' partials in a fixed order
// and writes one partial row per CTA; a second kernel reduces those rows in
// a fixed order, so the result is deterministic.
constexpr int LN_ROWS_PER_CTA = 8;   // forward: 8 warps, one row each
constexpr int LN_BWD_WARPS = 8;

template <int V4, bool F16>
__global__ void __launch_bounds__(256) ln_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                     const float* __restrict__ b, __nv_bfloat16* __restrict__ y,
                                                     float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                     int M, int H, float eps) {
  const int row = blockIdx.x * LN_ROWS_PER_CTA + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int H4 = H >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (long)row * H);
  float4 v[V4];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < V4; ++i) {
    const int j = lane + 32 * i;
    v[i] = (j < H4) ? xr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
    s += v[i].x + v[i].y + v[i].z + v[i].w;
  }
  const float mu = warp_sum(s) / H;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < V4; ++i) {
    const int j = lane + 32 * i;
    if (j < H4) {
      const float a = v[i].x - mu, c = v[i].y - mu, d = v[i].z - mu, e = v[i].w - mu;
      ss += a * a + c * c + d * d + e * e;
    }
  }
  const float rstd = rsqrtf(warp_sum(ss) / H + eps);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  uint2* yr = reinterpret_cast<uint2*>(y + (long)row * H);
#pragma unroll
  for (int i = 0; i < V4; ++i) {
    const int j = lane + 32 * i;
    if (j < H4) {
      const float4 ww = w4[j], bb = b4[j];
      const float o0 = (v[i].x - mu) * rstd * ww.x + bb.x;
      const float o1 = (v[i].y - mu) * rstd * ww.y + bb.y;
      const float o2 = (v[i].z - mu) * rstd * ww.z + bb.z;
      const float o3 = (v[i].w - mu) * rstd * ww.w + bb.w;
      yr[j] = make_uint2(pack16<F16>(o0, o1), pack16<F16>(o2, o3));
    }
  }
  if (lane == 0) {
    mean_out[row] = mu;
    rstd_out[row] = rstd;
  }
}

// Reduce-scatter consumer: x_new = x + sum_s parts[s] + bias (fp32 residual
// shard), and, if w != nullptr, y = LN(x_new) in bf16 with its statistics.
// parts: `nsrc` bf16 slots of [M, H] at stride `src_stride` elements.
template <int V4, bool F16>
__global__ void __launch_bounds__(256) resid_sum_ln_kernel(const float* __restrict__ x,
                                                           const __nv_bfloat16* __restrict__ parts, int nsrc,
                                                           long src_stride, const float* __restrict__ bias,
                                                           float* __restrict__ x_new, const float* __restrict__ w,
                                                           const float* __restrict__ b, __nv_bfloat16* __restrict__ y,
                                                           float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                           int M, int H, float eps) {
  const int row = blockIdx.x * LN_ROWS_PER_CTA + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int H4 = H >> 2;
  float4 v[V4];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < V4; ++i) {
    const int j = lane + 32 * i;
    if (j < H4) {
      float4 a = reinterpret_cast<const float4*>(x + (long)row * H)[j];
      const float4 bb = reinterpret_cast<const float4*>(bias)[j];
      a.x += bb.x;
      a.y += bb.y;
      a.z += bb.z;
      a.w += bb.w;
      for (int q = 0; q < nsrc; ++q) {
        const uint2 raw = reinterpret_cast<const uint2*>(parts + q * src_stride + (long)row * H)[j];
        a.x += lo16<F16>(raw.x);
        a.y += hi16<F16>(raw.x);
        a.z += lo16<F16>(raw.y);
        a.w += hi16<F16>(raw.y);
      }
      v[i] = a;
      reinterpret_cast<float4*>(x_new + (long)row * H)[j] = a;
    } else {
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    s += v[i].x + v[i].y + v[i].z + v[i].w;
  }
  if (w == nullptr) return;
  const float mu = warp_sum(s) / H;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < V4; ++i) {
    const int j = lane + 32 * i;
    if (j < H4) {
      const float a = v[i].x - mu, c = v[i].y - mu, d = v[i].z - mu, e = v[i].w - mu;
      ss += a * a + c * c + d * d + e * e;
    }
  }
  const float rstd = rsqrtf(warp_sum(ss) / H + eps);
  uint2* yr = reinterpret_cast<uint2*>(y + (long)row * H);
#pragma unroll
  for (int i = 0; i < V4; ++i) {
    const int j = lane + 32 * i;
    if (j < H4) {
      const float4 ww = reinterpret_cast<const float4*>(w)[j], bb = reinterpret_cast<const float4*>(b)[j];
      yr[j] = make_uint2(pack16<F16>((v[i].x - mu) * rstd * ww.x + bb.x, (v[i].y - mu) * rstd * ww.y + bb.y),
                         pack16<F16>((v[i].z - mu) * rstd * ww.z + bb.z, (v[i].w - mu) * rstd * ww.w + bb.w));
    }
  }
  if (lane == 0) {
    mean_out[row] = mu;
    rstd_out[row] = rstd;
  }
}

// Backward. dy fp32 [M, H] (gradient of the LN output), x fp32 [M, H].
//   dres fp32 [M, H] = dres_in + dx   (dres may alias dres_in: residual gradient in place)
//   dres16 bf16 [M, H] = dres          (operand copy for the next dgrad/wgrad GEMMs)
//   part fp32 [gridDim.x, 2, H]        per-CTA partial dgamma (row 0) and dbeta (row 1)
// Per-CTA partials are accumulated with shared-memory atomics (no per-thread
// accumulators), which keeps registers low enough for 3 CTAs per SM.
//
// HOIST (the default; HB_LN_BWD_HOIST=0 selects the plain order): the incoming residual
// gradient of a row is loaded in one batch after the row's reductions and
// before any of its outputs is stored. Without it, each dres_in load follows
// the previous element's dres store, and since dres may alias dres_in the
// compiler must keep that order: V4 dependent DRAM round trips per row. The
// batch reuses the normalised-input registers, which are dead by then, so the
// register count stays the same; the arithmetic is unchanged (same fused
// multiply-add per element).
template <int V4, bool HOIST, bool F16>
__global__ void __launch_bounds__(256, 2) ln_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                                        const float* __restrict__ mean, const float* __restrict__ rstd,
                                                        const float* __restrict__ w, const float* dres_in,
                                                        float* dres, __nv_bfloat16* __restrict__ dres16,
                                                        float* __restrict__ part, int M, int H, int dy_srcs,
                                                        long dy_src_stride) {
  extern __shared__ float sacc[];  // [LN_BWD_WARPS][2][H]: each warp's dgamma, dbeta partials
  const int warp_in = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int H4 = H >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4 gacc[V4], bacc[V4];
#pragma unroll
  for (int i = 0; i < V4; ++i) gacc[i] = bacc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  // Warps stride over rows; dgamma / dbeta partials stay in registers.
#pragma unroll 1
  for (int r = blockIdx.x * LN_BWD_WARPS + warp_in; r < M; r += gridDim.x * LN_BWD_WARPS) {
    const float4* xr = reinterpret_cast<const float4*>(x + (long)r * H);
    const float4* dyr = reinterpret_cast<const float4*>(dy + (long)r * H);
    float4 xv[V4], dv[V4];
#pragma unroll
    for (int i = 0; i < V4; ++i) {
      const int j = lane + 32 * i;
      const bool in = j < H4;
      xv[i] = in ? xr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
      dv[i] = in ? dyr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
      // dy may arrive as several partial sums (reduce-scatter slots), fixed order.
      for (int sidx = 1; sidx < dy_srcs && in; ++sidx) {
        const float4 e = reinterpret_cast<const float4*>(dy + sidx * dy_src_stride + (long)r * H)[j];
        dv[i].x += e.x;
        dv[i].y += e.y;
        dv[i].z += e.z;
        dv[i].w += e.w;
      }
    }
    const float mu = mean[r], rs = rstd[r];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < V4; ++i) {
      const int j = lane + 32 * i;
      xv[i] = make_float4((xv[i].x - mu) * rs, (xv[i].y - mu) * rs, (xv[i].z - mu) * rs, (xv[i].w - mu) * rs);
      if (j < H4) {
        gacc[i].x = fmaf(dv[i].x, xv[i].x, gacc[i].x);
        gacc[i].y = fmaf(dv[i].y, xv[i].y, gacc[i].y);
        gacc[i].z = fmaf(dv[i].z, xv[i].z, gacc[i].z);
        gacc[i].w = fmaf(dv[i].w, xv[i].w, gacc[i].w);
        bacc[i].x += dv[i].x;
        bacc[i].y += dv[i].y;
        bacc[i].z += dv[i].z;
        bacc[i].w += dv[i].w;
        const float4 ww = w4[j];
        dv[i] = make_float4(dv[i].x * ww.x, dv[i].y * ww.y, dv[i].z * ww.z, dv[i].w * ww.w);  // g = dy * w
      }
      s1 += dv[i].x + dv[i].y + dv[i].z + dv[i].w;
      s2 += dv[i].x * xv[i].x + dv[i].y * xv[i].y + dv[i].z * xv[i].z + dv[i].w * xv[i].w;
    }
    const float m1 = warp_sum(s1) / H, m2 = warp_sum(s2) / H;
    const float4* rin = reinterpret_cast<const float4*>(dres_in + (long)r * H);
    float4* rout = reinterpret_cast<float4*>(dres + (long)r * H);
    uint2* r16 = reinterpret_cast<uint2*>(dres16 + (long)r * H);
    if constexpr (HOIST) {
#pragma unroll
      for (int i = 0; i < V4; ++i) {  // per-element term; the normalised input is dead after this
        dv[i].x = dv[i].x - m1 - xv[i].x * m2;
        dv[i].y = dv[i].y - m1 - xv[i].y * m2;
        dv[i].z = dv[i].z - m1 - xv[i].z * m2;
        dv[i].w = dv[i].w - m1 - xv[i].w * m2;
      }
#pragma unroll
      for (int i = 0; i < V4; ++i) {  // every load of the row before any store of it
        const int j = lane + 32 * i;
        xv[i] = (j < H4) ? rin[j] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < V4; ++i) {
        const int j = lane + 32 * i;
        if (j < H4) {
          float4 o;
          o.x = fmaf(rs, dv[i].x, xv[i].x);
          o.y = fmaf(rs, dv[i].y, xv[i].y);
          o.z = fmaf(rs, dv[i].z, xv[i].z);
          o.w = fmaf(rs, dv[i].w, xv[i].w);
          rout[j] = o;
          r16[j] = make_uint2(pack16<F16>(o.x, o.y), pack16<F16>(o.z, o.w));
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < V4; ++i) {
        const int j = lane + 32 * i;
        if (j < H4) {
          float4 o = rin[j];
          o.x += rs * (dv[i].x - m1 - xv[i].x * m2);
          o.y += rs * (dv[i].y - m1 - xv[i].y * m2);
          o.z += rs * (dv[i].z - m1 - xv[i].z * m2);
          o.w += rs * (dv[i].w - m1 - xv[i].w * m2);
          rout[j] = o;
          r16[j] = make_uint2(pack16<F16>(o.x, o.y), pack16<F16>(o.z, o.w));
        }
      }
    }
  }
  // Per-CTA reduction of the warps' partials in a fixed order (deterministic).
  float4* mine = reinterpret_cast<float4*>(sacc + (long)warp_in * 2 * H);
#pragma unroll
  for (int i = 0; i < V4; ++i) {
    const int j = lane + 32 * i;
    if (j < H4) {
      mine[j] = gacc[i];
      mine[H4 + j] = bacc[i];
    }
  }
  __syncthreads();
  float* out = part + (long)blockIdx.x * 2 * H;
  for (int c = threadIdx.x; c < 2 * H; c += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int wi = 0; wi < LN_BWD_WARPS; ++wi) acc += sacc[(long)wi * 2 * H + c];
    out[c] = acc;
  }
}

// out0[c] / out1[c - split] += sum_r part[r, c]: 32 columns x 32 row-slices per
// block, each slice keeping four loads in flight (the partials are a few hundred
// rows, so the sum is latency-bound), fixed summation order (deterministic). In a
// graph-replayed LayerNorm backward at 8192 x 768 it measured the same as the
// earlier 8-slice form (28.6 vs 28.7 us for the pair of kernels).
constexpr int kReduceRowsThreads = 1024;
__global__ void __launch_bounds__(kReduceRowsThreads) reduce_rows_kernel(const float* __restrict__ part, int rows,
                                                                         int n, float* __restrict__ out0,
                                                                         float* __restrict__ out1, int split) {
  __shared__ float red[32][33];
  const int cl = threadIdx.x & 31, sl = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + cl;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  if (c < n) {
    int r = sl;
    for (; r + 96 < rows; r += 128) {
      a0 += part[(long)r * n + c];
      a1 += part[(long)(r + 32) * n + c];
      a2 += part[(long)(r + 64) * n + c];
      a3 += part[(long)(r + 96) * n + c];
    }
    for (; r < rows; r += 32) a0 += part[(long)r * n + c];
  }
  red[sl][cl] = (a0 + a1) + (a2 + a3);
  __syncthreads();
  if (sl == 0 && c < n) {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < 32; ++q) s += red[q][cl];
    if (c < split) out0[c] += s;
    else out1[c - split] += s;
  }
}

// Column sums of a bf16 matrix: out[c] += sum_r in[r, c]. Block = 8 warps
// covering 64 columns (2 per lane) and `rows_per_cta` rows.
template <bool F16>
__global__ void __launch_bounds__(256) colsum_bf16_kernel(const __nv_bfloat16* __restrict__ in, long ld, int M,
                                                          int N, int rows_per_cta, float* __restrict__ out) {
  __shared__ float red[8][64];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * 64 + lane * 2;
  const int r0 = blockIdx.y * rows_per_cta;
  const int r1 = min(M, r0 + rows_per_cta);
  float a0 = 0.f, a1 = 0.f;
  if (c < N) {
    for (int r = r0 + warp; r < r1; r += 8) {
      const uint32_t v = *reinterpret_cast<const uint32_t*>(in + (long)r * ld + c);
      a0 += lo16<F16>(v);
      a1 += hi16<F16>(v);
    }
  }
  red[warp][lane * 2] = a0;
  red[warp][lane * 2 + 1] = a1;
  __syncthreads();
  if (threadIdx.x < 64) {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < 8; ++q) s += red[q][threadIdx.x];
    const int cc = blockIdx.x * 64 + threadIdx.x;
    if (cc < N) atomicAdd(out + cc, s);
  }
}

// Wide variant (N % 8 == 0, 16-byte aligned rows): each lane sums 8 columns
// (one 16-byte load per row), a CTA covers 256 columns, and every warp keeps
// 8 row loads in flight; warps combine through shared memory, then one
// atomic per column per CTA.
template <bool F16>
__global__ void __launch_bounds__(256) colsum_bf16_wide_kernel(const __nv_bfloat16* __restrict__ in, long ld, int M,
                                                               int N, int rows_per_cta, float* __restrict__ out) {
  __shared__ float red[8][256 + 8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c0 = blockIdx.x * 256 + lane * 8;
  const int r0 = blockIdx.y * rows_per_cta;
  const int r1 = min(M, r0 + rows_per_cta);
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (c0 < N) {
    int r = r0 + warp;
    for (; r + 7 * 8 < r1; r += 64) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = __ldg(reinterpret_cast<const uint4*>(in + (long)(r + 8 * u) * ld + c0));
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint16_t* e = reinterpret_cast<const uint16_t*>(&v[u]);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += to_f32<F16>(e[j]);
      }
    }
    for (; r < r1; r += 8) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(in + (long)r * ld + c0));
      const uint16_t* e = reinterpret_cast<const uint16_t*>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += to_f32<F16>(e[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[warp][lane * 8 + j] = acc[j];
  __syncthreads();
  float sum = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) sum += red[q][threadIdx.x];
  const int cc = blockIdx.x * 256 + threadIdx.x;
  if (cc < N) atomicAdd(out + cc, sum);
}

// ----------------------------------------------------------------------------
// Host launchers (raw pointers; the torch-facing checks live in ops_host.cpp)
// ----------------------------------------------------------------------------
#define HB_LN_DISPATCH(V4, ...)                                  \
  switch (V4) {                                                  \
    case 1: { constexpr int kV = 1; __VA_ARGS__; } break;        \
    case 2: { constexpr int kV = 2; __VA_ARGS__; } break;        \
    case 4: { constexpr int kV = 4; __VA_ARGS__; } break;        \
    case 6: { constexpr int kV = 6; __VA_ARGS__; } break;        \
    case 8: { constexpr int kV = 8; __VA_ARGS__; } break;        \
    case 10: { constexpr int kV = 10; __VA_ARGS__; } break;      \
    case 12: { constexpr int kV = 12; __VA_ARGS__; } break;      \
    case 16: { constexpr int kV = 16; __VA_ARGS__; } break;      \
    default: throw std::runtime_error("layernorm: unsupported width"); \
  }

static int ln_v4(int H) {
  if (H % 4 != 0 || H > 2048) throw std::runtime_error("layernorm: H must be a multiple of 4, <= 2048");
  const int v = (H + 127) / 128;
  const int allowed[] = {1, 2, 4, 6, 8, 10, 12, 16};
  for (int a : allowed)
    if (a >= v) return a;
  return 16;
}

void ln_fwd_launch(const float* x, const float* w, const float* b, __nv_bfloat16* y, float* mean, float* rstd,
                   int M, int H, float eps, bool f16, cudaStream_t s) {
  if (M == 0) return;
  const int blocks = (M + LN_ROWS_PER_CTA - 1) / LN_ROWS_PER_CTA;
  if (f16) {
    HB_LN_DISPATCH(ln_v4(H), ln_fwd_kernel<kV, true><<<blocks, 256, 0, s>>>(x, w, b, y, mean, rstd, M, H, eps));
  } else {
    HB_LN_DISPATCH(ln_v4(H), ln_fwd_kernel<kV, false><<<blocks, 256, 0, s>>>(x, w, b, y, mean, rstd, M, H, eps));
  }
  HB_CUDA_CHECK(cudaGetLastError());
}

void resid_sum_ln_launch(const float* x, const __nv_bfloat16* parts, int nsrc, long src_stride, const float* bias,
                         float* x_new, const float* w, const float* b, __nv_bfloat16* y, float* mean, float* rstd,
                         int M, int H, float eps, bool f16, cudaStream_t s) {
  if (M == 0) return;
  const int blocks = (M + LN_ROWS_PER_CTA - 1) / LN_ROWS_PER_CTA;
  if (f16) {
    HB_LN_DISPATCH(ln_v4(H), resid_sum_ln_kernel<kV, true><<<blocks, 256, 0, s>>>(
                                 x, parts, nsrc, src_stride, bias, x_new, w, b, y, mean, rstd, M, H, eps));
  } else {
    HB_LN_DISPATCH(ln_v4(H), resid_sum_ln_kernel<kV, false><<<blocks, 256, 0, s>>>(
                                 x, parts, nsrc, src_stride, bias, x_new, w, b, y, mean, rstd, M, H, eps));
  }
  HB_CUDA_CHECK(cudaGetLastError());
}

int ln_bwd_num_ctas(int M, int device) {
  // Two resident CTAs per SM, never more CTAs than there are 8-row groups.
  const int full = 2 * num_sms(device);
  const int need = M > 0 ? (M + LN_BWD_WARPS - 1) / LN_BWD_WARPS : 1;
  return need < full ? need : full;
}

void ln_bwd_launch(const float* dy, const float* x, const float* mean, const float* rstd, const float* w,
                   const float* dres_in, float* dres, __nv_bfloat16* dres16, float* part, int num_ctas,
                   float* dgamma, float* dbeta, int M, int H, int dy_srcs, long dy_src_stride, bool f16,
                   cudaStream_t s) {
  if (M == 0) return;
  static const bool hoist = [] {
    // measured on a B200 at 8192 x 768: 34.8 us hoisted, 42.2 us in the plain order
    const char* e = std::getenv("HB_LN_BWD_HOIST");
    return e == nullptr || e[0] != '0';
  }();
  const size_t smem = (size_t)LN_BWD_WARPS * 2 * H * sizeof(float);
  // The four (hoist, 16-bit format) instantiations at width kV.
#define HB_LN_BWD_KERNEL(kV) \
  (hoist ? (f16 ? ln_bwd_kernel<kV, true, true> : ln_bwd_kernel<kV, true, false>) \
         : (f16 ? ln_bwd_kernel<kV, false, true> : ln_bwd_kernel<kV, false, false>))
  if (smem > 48 * 1024) {
    static bool attr_set[64][17][2][2] = {};
    const int dev = current_device();
    const int v = ln_v4(H);
    if (!attr_set[dev][v][hoist][f16]) {
      HB_LN_DISPATCH(v, HB_CUDA_CHECK(cudaFuncSetAttribute(HB_LN_BWD_KERNEL(kV),
                                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)));
      attr_set[dev][v][hoist][f16] = true;
    }
  }
  HB_LN_DISPATCH(ln_v4(H), HB_LN_BWD_KERNEL(kV)<<<num_ctas, 256, smem, s>>>(dy, x, mean, rstd, w, dres_in, dres,
                                                                            dres16, part, M, H, dy_srcs,
                                                                            dy_src_stride));
#undef HB_LN_BWD_KERNEL
  HB_CUDA_CHECK(cudaGetLastError());
  reduce_rows_kernel<<<(2 * H + 31) / 32, kReduceRowsThreads, 0, s>>>(part, num_ctas, 2 * H, dgamma, dbeta, H);
  HB_CUDA_CHECK(cudaGetLastError());
}

// out = 16-bit(g * mask): 4 elements (2 mask pairs) per thread.
template <bool F16>
__global__ void dropout_bf16_kernel(const float* __restrict__ g, __nv_bfloat16* __restrict__ out, long M, int H,
                                    DropoutArgs d) {
  const uint32_t key = dropout_key(*d.seed, d.site);
  const long n4 = M * (long)H / 4;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    const long e = 4 * i;
    const long row = e / H, col = e % H;
    const uint64_t pair = ((uint64_t)(d.row0 + row) * (uint64_t)H + (uint64_t)col) >> 1;
    float m0, m1, m2, m3;
    dropout_pair(dropout_bits(key, pair), d.thresh, d.scale, m0, m1);
    dropout_pair(dropout_bits(key, pair + 1), d.thresh, d.scale, m2, m3);
    const float4 v = reinterpret_cast<const float4*>(g)[i];
    reinterpret_cast<uint2*>(out)[i] = make_uint2(pack16<F16>(v.x * m0, v.y * m1), pack16<F16>(v.z * m2, v.w * m3));
  }
}

void dropout_bf16_launch(const float* g, __nv_bfloat16* out, long M, int H, const DropoutArgs& d, bool f16,
                         cudaStream_t s) {
  const long n4 = M * (long)H / 4;
  if (n4 == 0) return;
  const int blocks = (int)std::min<long>((n4 + 255) / 256, 4L * num_sms(current_device()));
  (f16 ? dropout_bf16_kernel<true> : dropout_bf16_kernel<false>)<<<blocks, 256, 0, s>>>(g, out, M, H, d);
  HB_CUDA_CHECK(cudaGetLastError());
}

void colsum_bf16_launch(const __nv_bfloat16* in, long ld, int M, int N, float* out, bool f16, cudaStream_t s) {
  if (M == 0 || N == 0) return;
  if (N % 8 == 0 && ld % 8 == 0 && reinterpret_cast<uintptr_t>(in) % 16 == 0) {
    const int rows_per_cta = 64;
    dim3 grid((N + 255) / 256, (M + rows_per_cta - 1) / rows_per_cta);
    (f16 ? colsum_bf16_wide_kernel<true> : colsum_bf16_wide_kernel<false>)<<<grid, 256, 0, s>>>(in, ld, M, N,
                                                                                               rows_per_cta, out);
    HB_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const int rows_per_cta = 256;
  dim3 grid((N + 63) / 64, (M + rows_per_cta - 1) / rows_per_cta);
  (f16 ? colsum_bf16_kernel<true> : colsum_bf16_kernel<false>)<<<grid, 256, 0, s>>>(in, ld, M, N, rows_per_cta, out);
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
