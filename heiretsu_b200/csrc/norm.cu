// LayerNorm forward/backward and column reductions (bias gradients).
//
// Replaces nn.LayerNorm (reference gpt_model.py:111-119, :237, pipeline.py:83)
// and the bias-gradient reductions autograd performs for tp_linear.py:226/:310.
//
// Layout: rows of H contiguous elements. One warp per row; each lane keeps its
// share of the row in registers as float4 (H % 4 == 0, H <= 32*4*MAXV), so the
// row is read from HBM once and written once.
#include <cuda_bf16.h>

#include "common.cuh"
#include "host_utils.h"

namespace hb {

constexpr int LN_MAXV = 16;  // float4 per lane: H <= 2048

// x fp32 [M, H] -> y bf16 [M, H]; mean, rstd fp32 [M].
__global__ void __launch_bounds__(256) ln_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                     const float* __restrict__ b, __nv_bfloat16* __restrict__ y,
                                                     float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                     int M, int H, float eps) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= M) return;
  const int H4 = H >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (long)warp * H);
  float4 v[LN_MAXV];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int j = lane + 32 * i;
    if (j < H4) {
      v[i] = xr[j];
      s += v[i].x + v[i].y + v[i].z + v[i].w;
    }
  }
  const float mu = warp_sum(s) / H;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int j = lane + 32 * i;
    if (j < H4) {
      const float a = v[i].x - mu, c = v[i].y - mu, d = v[i].z - mu, e = v[i].w - mu;
      ss += a * a + c * c + d * d + e * e;
    }
  }
  const float rstd = rsqrtf(warp_sum(ss) / H + eps);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  uint2* yr = reinterpret_cast<uint2*>(y + (long)warp * H);
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int j = lane + 32 * i;
    if (j < H4) {
      const float4 ww = w4[j], bb = b4[j];
      const float o0 = (v[i].x - mu) * rstd * ww.x + bb.x;
      const float o1 = (v[i].y - mu) * rstd * ww.y + bb.y;
      const float o2 = (v[i].z - mu) * rstd * ww.z + bb.z;
      const float o3 = (v[i].w - mu) * rstd * ww.w + bb.w;
      yr[j] = make_uint2(pack_bf16(o0, o1), pack_bf16(o2, o3));
    }
  }
  if (lane == 0) {
    mean_out[warp] = mu;
    rstd_out[warp] = rstd;
  }
}

// Backward. dy fp32 [M, H] (gradient of the LN output), x fp32 [M, H].
//   dres fp32 [M, H] += dx         (residual-stream gradient, updated in place)
//   dres16 bf16 [M, H] = dres      (operand copy for the next dgrad/wgrad GEMMs)
//   part fp32 [gridDim.x, 2, H]    per-CTA partial dgamma (row 0) and dbeta (row 1)
// If `dres_in` differs from `dres`, the result is dres = dres_in + dx.
__global__ void __launch_bounds__(256) ln_bwd_kernel(const float* __restrict__ dy, const float* __restrict__ x,
                                                     const float* __restrict__ mean, const float* __restrict__ rstd,
                                                     const float* __restrict__ w, const float* dres_in,
                                                     float* dres, __nv_bfloat16* __restrict__ dres16,
                                                     float* __restrict__ part, int M, int H, int rows_per_cta) {
  extern __shared__ float sred[];  // [8 warps][2][H]
  const int warp_in = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int H4 = H >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4 dg[LN_MAXV], db[LN_MAXV];
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    dg[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    db[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const int row0 = blockIdx.x * rows_per_cta;
  const int row1 = min(M, row0 + rows_per_cta);
  for (int r = row0 + warp_in; r < row1; r += nwarps) {
    const float4* xr = reinterpret_cast<const float4*>(x + (long)r * H);
    const float4* dyr = reinterpret_cast<const float4*>(dy + (long)r * H);
    const float mu = mean[r], rs = rstd[r];
    float4 xh[LN_MAXV], g[LN_MAXV];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < LN_MAXV; ++i) {
      const int j = lane + 32 * i;
      if (j < H4) {
        const float4 xv = xr[j], d = dyr[j], ww = w4[j];
        xh[i] = make_float4((xv.x - mu) * rs, (xv.y - mu) * rs, (xv.z - mu) * rs, (xv.w - mu) * rs);
        g[i] = make_float4(d.x * ww.x, d.y * ww.y, d.z * ww.z, d.w * ww.w);
        s1 += g[i].x + g[i].y + g[i].z + g[i].w;
        s2 += g[i].x * xh[i].x + g[i].y * xh[i].y + g[i].z * xh[i].z + g[i].w * xh[i].w;
        dg[i].x += d.x * xh[i].x;
        dg[i].y += d.y * xh[i].y;
        dg[i].z += d.z * xh[i].z;
        dg[i].w += d.w * xh[i].w;
        db[i].x += d.x;
        db[i].y += d.y;
        db[i].z += d.z;
        db[i].w += d.w;
      }
    }
    const float m1 = warp_sum(s1) / H, m2 = warp_sum(s2) / H;
    const float4* rin = reinterpret_cast<const float4*>(dres_in + (long)r * H);
    float4* rout = reinterpret_cast<float4*>(dres + (long)r * H);
    uint2* r16 = reinterpret_cast<uint2*>(dres16 + (long)r * H);
#pragma unroll
    for (int i = 0; i < LN_MAXV; ++i) {
      const int j = lane + 32 * i;
      if (j < H4) {
        float4 o = rin[j];
        o.x += rs * (g[i].x - m1 - xh[i].x * m2);
        o.y += rs * (g[i].y - m1 - xh[i].y * m2);
        o.z += rs * (g[i].z - m1 - xh[i].z * m2);
        o.w += rs * (g[i].w - m1 - xh[i].w * m2);
        rout[j] = o;
        r16[j] = make_uint2(pack_bf16(o.x, o.y), pack_bf16(o.z, o.w));
      }
    }
  }
  // Reduce the per-warp partials through shared memory.
  float* mine = sred + warp_in * 2 * H;
#pragma unroll
  for (int i = 0; i < LN_MAXV; ++i) {
    const int j = lane + 32 * i;
    if (j < H4) {
      reinterpret_cast<float4*>(mine)[j] = dg[i];
      reinterpret_cast<float4*>(mine + H)[j] = db[i];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * H; c += blockDim.x) {
    float acc = 0.f;
    for (int q = 0; q < nwarps; ++q) acc += sred[q * 2 * H + c];
    part[(long)blockIdx.x * 2 * H + c] = acc;
  }
}

// out[c] += sum_r part[r, c] for c < n (fixed summation order: deterministic).
__global__ void reduce_rows_kernel(const float* __restrict__ part, int rows, int n, float* __restrict__ out0,
                                   float* __restrict__ out1, int split) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n) return;
  float acc = 0.f;
  for (int r = 0; r < rows; ++r) acc += part[(long)r * n + c];
  if (c < split) out0[c] += acc;
  else out1[c - split] += acc;
}

// Column sums of a bf16 matrix: out[c] += sum_r in[r, c]. Block = 8 warps
// covering 64 columns (2 per lane) and `rows_per_cta` rows.
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
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(in + (long)r * ld + c);
      a0 += __bfloat162float(v.x);
      a1 += __bfloat162float(v.y);
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

// ----------------------------------------------------------------------------
// Host launchers (raw pointers; the torch-facing checks live in ops_host.cpp)
// ----------------------------------------------------------------------------
void ln_fwd_launch(const float* x, const float* w, const float* b, __nv_bfloat16* y, float* mean, float* rstd,
                   int M, int H, float eps, cudaStream_t s) {
  if (H % 4 != 0 || H > 32 * 4 * LN_MAXV) throw std::runtime_error("layernorm: H must be a multiple of 4, <= 2048");
  const int threads = 256;
  const int blocks = (M * 32 + threads - 1) / threads;
  ln_fwd_kernel<<<blocks, threads, 0, s>>>(x, w, b, y, mean, rstd, M, H, eps);
  HB_CUDA_CHECK(cudaGetLastError());
}

int ln_bwd_num_ctas(int M, int device) {
  const int ctas = 2 * num_sms(device);
  return M < ctas ? (M > 0 ? M : 1) : ctas;
}

void ln_bwd_launch(const float* dy, const float* x, const float* mean, const float* rstd, const float* w,
                   const float* dres_in, float* dres, __nv_bfloat16* dres16, float* part, int num_ctas,
                   float* dgamma, float* dbeta, int M, int H, cudaStream_t s) {
  if (H % 4 != 0 || H > 32 * 4 * LN_MAXV) throw std::runtime_error("layernorm: H must be a multiple of 4, <= 2048");
  const int rows_per_cta = (M + num_ctas - 1) / num_ctas;
  const size_t smem = 8 * 2 * H * sizeof(float);
  static bool attr = false;
  if (!attr) {
    HB_CUDA_CHECK(cudaFuncSetAttribute(ln_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 8 * 2 * 2048 * 4));
    attr = true;
  }
  ln_bwd_kernel<<<num_ctas, 256, smem, s>>>(dy, x, mean, rstd, w, dres_in, dres, dres16, part, M, H, rows_per_cta);
  HB_CUDA_CHECK(cudaGetLastError());
  reduce_rows_kernel<<<(2 * H + 255) / 256, 256, 0, s>>>(part, num_ctas, 2 * H, dgamma, dbeta, H);
  HB_CUDA_CHECK(cudaGetLastError());
}

void colsum_bf16_launch(const __nv_bfloat16* in, long ld, int M, int N, float* out, cudaStream_t s) {
  if (M == 0 || N == 0) return;
  const int rows_per_cta = 256;
  dim3 grid((N + 63) / 64, (M + rows_per_cta - 1) / rows_per_cta);
  colsum_bf16_kernel<<<grid, 256, 0, s>>>(in, ld, M, N, rows_per_cta, out);
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
