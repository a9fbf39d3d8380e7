// Causal flash attention with head_dim 128 on tcgen05 tensor cores.
//
// Same semantics and data layout as the head_dim 64 kernels (attention.cu):
// Q, K, V read in place from the QKV projection qkv[B*T, 3*Hs] (columns
// [Q | K | V], head h at h*128) through 3-D TMA maps {3*Hs, T, B}; output
// y[B*T, Hs]; the negated log2-domain LSE [B, nh, Tpad] passed from forward
// to backward. Replaces F.scaled_dot_product_attention(q, k, v,
// is_causal=True) (reference gpt_model.py:74-81) for the reference's default
// model (--n_head 6 --n_embed 768, train.py:184-185). A 128-wide row is two
// 128-byte swizzle atoms, so every 128 x 128 tile lives in shared memory as
// two 16 KB sub-tiles (columns 0..63 and 64..127), each one TMA box.
//
// Forward, one CTA per (query tile of 128, head, batch), 320 threads,
// heaviest tiles launched first:
//   warp 0      TMA: Q, then K0, K1, V0, K2, V1, ... into a 3-slot ring
//   warp 1      MMA: S_j = Q K_j^T into one of two TMEM score buffers
//               (double-buffered, so S_{j+1} is computed while the softmax
//               of S_j runs), O_lo/O_hi = P_j V_j (two N = 64 halves)
//   warps 2-9   softmax, thread = query row; the two warps on a TMEM lane
//               quarter split the columns: both take the row max over all
//               128 scores (identical arithmetic, so identical maxima), each
//               exponentiates its 64 columns into its half of P (bf16,
//               swizzled smem) and accumulates its 64 output columns in
//               registers with the online-softmax rescale. The two partial
//               row sums meet in shared memory at the end.
//   TMEM: S0 0..127, S1 128..255, O_lo 256/320 and O_hi 384/448 (double
//   buffered), 512 columns.
//
// Backward, one CTA per (key tile of 128, head, batch), 320 threads, over
// the query half-tiles u (64 queries each) at or after the key tile; half-
// tile j of the CTA belongs to softmax warpgroup g = j % 2:
//   S^T_g = K Q_u^T, dP^T_g = V dO_u^T   (128 keys x 64 queries each)
//   WG g (thread = key row): P^T, dS^T = P^T (dP^T - D) * scale -> smem
//   dV += P^T dO_u, dK += dS^T Q_u       (128 keys x 128, in TMEM all along)
//   dQ_u^T = K^T dS^T                    (128 x 64, into the S^T_g columns,
//                                         which the softmax has consumed)
//   WG g reads dQ_u^T out of TMEM, releases the columns for the next S^T_g,
//   and adds it to an fp32 accumulator by bulk tensor reduce-adds staged in
//   its own rows of P^T / dS^T.
//   TMEM: dV 0..127, dK 128..255, S^T_g at 256 + 128 g, dP^T_g 64 further:
//   512 columns. Shared memory: K, V (64 KB), a 3-deep ring of Q_u / dO_u
//   (96 KB), per-warpgroup P^T and dS^T (64 KB), LSE / D ring.
#include <cuda_bf16.h>

#include <stdexcept>

#include "attention_common.cuh"
#include "host_utils.h"

namespace hb {

namespace d128 {

constexpr int kD = 128;
constexpr int kSub = 16384;                    // one 128-row x 64-column sub-tile (bf16, 128B-swizzled)
constexpr int kTileBytes = 2 * kSub;           // 128 x 128 bf16
constexpr int FWD_SLOTS = 3;
constexpr int THREADS = 320;
constexpr int FWD_SMEM = kTileBytes /*Q*/ + FWD_SLOTS * kTileBytes /*K/V ring*/ + kTileBytes /*P*/ + 1024;

__device__ __forceinline__ int k_item(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int v_item(int j, int n) { return (j == n - 1) ? 2 * n - 1 : 2 * j + 2; }

// Online softmax of one 128x128 score tile for the calling thread's row and
// column half `g`: the row max over all 128 columns, then 2^(s*scale*log2e - m)
// over columns [64g, 64g+64), written as bf16 into P's atom g. Updates the
// running max m and this half's partial row sum l; returns the rescale factor
// of the previous output accumulator.
template <bool DIAG, bool DROP, bool F16>
__device__ __forceinline__ float softmax_half(uint32_t tS, uint32_t lane_off, uint8_t* sP, int g, int row, int key0,
                                              int q, float scale_log2, float& m, float& l, uint32_t dkey,
                                              uint64_t pair_row, uint32_t dthresh, float dscale) {
  float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    uint32_t va[32], vb[32];
    tmem_ld32_issue(tS + lane_off + (2 * h) * 32, va);
    tmem_ld32_issue(tS + lane_off + (2 * h + 1) * 32, vb);
    tmem_wait_ld_regs(va);
    tmem_pin_regs(vb);
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float x = __uint_as_float(va[i]), y = __uint_as_float(vb[i]);
      if (DIAG) {
        if (key0 + 2 * h * 32 + i > q) x = -INFINITY;
        if (key0 + (2 * h + 1) * 32 + i > q) y = -INFINITY;
      }
      mx[i & 3] = max3f(mx[i & 3], x, y);
    }
  }
  const float mt = max3f(mx[0], mx[1], fmaxf(mx[2], mx[3])) * scale_log2;
  const float m_new = fmaxf(m, mt);
  const float alpha = (m == -INFINITY) ? 0.f : fast_exp2(m - m_new);
  const uint64_t sl2 = f2_pack(scale_log2, scale_log2), nm2 = f2_pack(-m_new, -m_new);
  uint64_t sum2[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
  uint32_t va[32], vb[32];
  tmem_ld32_issue(tS + lane_off + (2 * g) * 32, va);
  tmem_ld32_issue(tS + lane_off + (2 * g + 1) * 32, vb);
  tmem_wait_ld_regs(va);
  tmem_pin_regs(vb);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const uint32_t* v = half ? vb : va;
    const int c = 2 * g + half;  // 32-column chunk of the row
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      float t0, t1;
      f2_unpack(f2_fma(f2_pack(__uint_as_float(v[i]), __uint_as_float(v[i + 1])), sl2, nm2), t0, t1);
      float p0 = fast_exp2(t0), p1 = fast_exp2(t1);
      if (DIAG) {
        if (key0 + c * 32 + i > q) p0 = 0.f;
        if (key0 + c * 32 + i + 1 > q) p1 = 0.f;
      }
      sum2[(i >> 1) & 1] = f2_add(sum2[(i >> 1) & 1], f2_pack(p0, p1));  // normaliser: undropped
      if (DROP) {
        float m0, m1;
        dropout_pair(dropout_bits(dkey, pair_row + ((key0 + c * 32 + i) >> 1)), dthresh, dscale, m0, m1);
        p0 *= m0;
        p1 *= m1;
      }
      pk[i >> 1] = pack16<F16>(p0, p1);
    }
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4)
      *reinterpret_cast<uint4*>(sP + sw128_off(row, c * 4 + q4)) =
          make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
  }
  float s0, s1, s2, s3;
  f2_unpack(sum2[0], s0, s1);
  f2_unpack(sum2[1], s2, s3);
  l = l * alpha + ((s0 + s1) + (s2 + s3));
  m = m_new;
  return alpha;
}

// o = o * alpha + (64 columns of a PV result in TMEM); o holds column pairs.
__device__ __forceinline__ void accumulate_o(uint64_t (&o)[32], uint32_t tO, float alpha) {
  uint32_t va[32], vb[32];
  tmem_ld32_issue(tO, va);
  tmem_ld32_issue(tO + 32, vb);
  tmem_wait_ld_regs(va);
  tmem_pin_regs(vb);
  const uint64_t a2 = f2_pack(alpha, alpha);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    o[i] = f2_fma(o[i], a2, f2_pack(__uint_as_float(va[2 * i]), __uint_as_float(va[2 * i + 1])));
    o[16 + i] = f2_fma(o[16 + i], a2, f2_pack(__uint_as_float(vb[2 * i]), __uint_as_float(vb[2 * i + 1])));
  }
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace d128

// ============================================================================
// Forward
// ============================================================================
template <bool DROP, bool F16>
__global__ void __launch_bounds__(d128::THREADS, 1)
    attn_fwd_d128_kernel(const __grid_constant__ CUtensorMap tm_qkv, AttnParams p) {
  using namespace d128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                             // [2 sub-tiles]
  uint8_t* sSlot = smem + kTileBytes;             // [FWD_SLOTS][2 sub-tiles]
  uint8_t* sP = sSlot + FWD_SLOTS * kTileBytes;   // [2 atoms of 64 keys]
  __shared__ uint64_t bar_q, bar_full[FWD_SLOTS], bar_empty[FWD_SLOTS], bar_s[2], bar_p, bar_o[2], bar_done;
  __shared__ uint32_t tmem_slot;
  __shared__ float l_part[2][kTile];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.T + kTile - 1) / kTile;
  const int bh = blockIdx.x % (p.B * p.nh);
  const int qt = n_qt - 1 - blockIdx.x / (p.B * p.nh);  // heaviest (most key tiles) first
  const int h = bh % p.nh;
  const int b = bh / p.nh;
  const int n_kv = qt + 1;

  if (threadIdx.x == 0) {
    mbar_init(&bar_q, 1);
    for (int s = 0; s < FWD_SLOTS; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    mbar_init(&bar_s[0], 1);
    mbar_init(&bar_s[1], 1);
    mbar_init(&bar_p, 8);  // every softmax warp has written its part of P_j
    mbar_init(&bar_o[0], 1);
    mbar_init(&bar_o[1], 1);
    mbar_init(&bar_done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tm_qkv);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  // S buffer s at s * 128; O half g, buffer b at 256 + g * 128 + b * 64

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(&bar_q, kTileBytes);
      tma_load_3d(sQ, &tm_qkv, &bar_q, h * kD, qt * kTile, b);
      tma_load_3d(sQ + kSub, &tm_qkv, &bar_q, h * kD + 64, qt * kTile, b);
      for (int idx = 0; idx < 2 * n_kv; ++idx) {
        int kv, is_v;
        if (idx == 0) {
          kv = 0, is_v = 0;
        } else if (idx == 2 * n_kv - 1) {
          kv = n_kv - 1, is_v = 1;
        } else if (idx & 1) {
          kv = (idx + 1) >> 1, is_v = 0;
        } else {
          kv = (idx - 2) >> 1, is_v = 1;
        }
        const int slot = idx % FWD_SLOTS;
        const uint32_t ph = (idx / FWD_SLOTS) & 1;
        if (!mbar_wait(&bar_empty[slot], ph ^ 1u, p.status, 60)) break;
        uint8_t* dst = sSlot + slot * kTileBytes;
        const int col = (is_v ? 2 : 1) * p.Hs + h * kD;
        mbar_arrive_expect_tx(&bar_full[slot], kTileBytes);
        tma_load_3d(dst, &tm_qkv, &bar_full[slot], col, kv * kTile, b);
        tma_load_3d(dst + kSub, &tm_qkv, &bar_full[slot], col + 64, kv * kTile, b);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = make_idesc_f16(128, 128, false, false, !F16);
      constexpr uint32_t idO = make_idesc_f16(128, 64, false, true, !F16);
      bool ok = mbar_wait(&bar_q, 0, p.status, 61);
      auto item = [&](int idx, uint32_t& addr) -> bool {
        const int slot = idx % FWD_SLOTS;
        if (!mbar_wait(&bar_full[slot], (idx / FWD_SLOTS) & 1, p.status, 62)) return false;
        tc_fence_after();
        addr = smem_u32(sSlot + slot * kTileBytes);
        return true;
      };
      const uint32_t qa = smem_u32(sQ), pa = smem_u32(sP);
      auto issue_s = [&](int buf, uint32_t ka) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t off = (k >> 2) * kSub + (k & 3) * 32;
          mma_f16_ss(tmem + buf * 128, sw128_desc(qa + off, 16, 1024), sw128_desc(ka + off, 16, 1024), idS, k > 0);
        }
        mma_commit(&bar_s[buf]);
      };
      auto issue_pv = [&](int j, uint32_t va) {
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const uint32_t tO = tmem + 256 + g * 128 + (j & 1) * 64;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)
            mma_f16_ss(tO, sw128_desc(pa + (ks >> 2) * kSub + (ks & 3) * 32, 16, 1024),
                       sw128_desc(va + g * kSub + ks * 2048, 8192, 1024), idO, ks > 0);
        }
        mma_commit(&bar_o[j & 1]);
      };
      uint32_t ka = 0, va = 0;
      if (ok && item(k_item(0), ka)) {
        issue_s(0, ka);
        mma_commit(&bar_empty[k_item(0) % FWD_SLOTS]);
      } else {
        ok = false;
      }
      if (ok && n_kv > 1) {
        if (item(k_item(1), ka)) {
          issue_s(1, ka);
          mma_commit(&bar_empty[k_item(1) % FWD_SLOTS]);
        } else {
          ok = false;
        }
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        // P_j complete (both column halves of every row): S buffer j % 2 is consumed too.
        if (!mbar_wait(&bar_p, j & 1, p.status, 63)) break;
        tc_fence_after();
        if (!item(v_item(j, n_kv), va)) break;
        issue_pv(j, va);
        mma_commit(&bar_empty[v_item(j, n_kv) % FWD_SLOTS]);
        if (j + 2 < n_kv) {
          if (!item(k_item(j + 2), ka)) break;
          issue_s(j & 1, ka);
          mma_commit(&bar_empty[k_item(j + 2) % FWD_SLOTS]);
        }
      }
      mma_commit(&bar_done);
      mbar_wait(&bar_done, 0, p.status, 64);
    }
  } else {
    const int g = (warp >= 6) ? 1 : 0;  // column half of S, P and O handled by this warp
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const int q = qt * kTile + row;
    const uint32_t tO0 = tmem + 256 + g * 128;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    uint32_t dkey = 0;
    uint64_t pair_row = 0;
    if (DROP) {
      dkey = dropout_key(*p.drop.seed, p.drop.site);
      pair_row = ((((uint64_t)b * p.nh_total + p.h0 + h) * p.T + q) * p.T) >> 1;
    }
    uint64_t o[32];  // this warp's 64 output columns of the row, as pairs
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = f2_pack(0.f, 0.f);
    bool ok = true;
    for (int j = 0; j < n_kv && ok; ++j) {
      if (!mbar_wait(&bar_s[j & 1], (j >> 1) & 1, p.status, 65)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // P smem is free once PV_{j-1} has completed.
      if (j > 0 && !mbar_wait(&bar_o[(j - 1) & 1], ((j - 1) >> 1) & 1, p.status, 66)) {
        ok = false;
        break;
      }
      const uint32_t tS = tmem + (j & 1) * 128;
      const float alpha =
          (j == qt) ? softmax_half<true, DROP, F16>(tS, lane_off, sP, g, row, j * kTile, q, p.scale_log2, m, l, dkey,
                                               pair_row, p.drop.thresh, p.drop.scale)
                    : softmax_half<false, DROP, F16>(tS, lane_off, sP, g, row, j * kTile, q, p.scale_log2, m, l, dkey,
                                                pair_row, p.drop.thresh, p.drop.scale);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_p);
      if (j > 0) {
        tc_fence_after();
        accumulate_o(o, tO0 + ((j - 1) & 1) * 64 + lane_off, alpha_prev);
      }
      alpha_prev = alpha;
    }
    if (ok && mbar_wait(&bar_o[(n_kv - 1) & 1], ((n_kv - 1) >> 1) & 1, p.status, 67)) {
      tc_fence_after();
      accumulate_o(o, tO0 + ((n_kv - 1) & 1) * 64 + lane_off, alpha_prev);
    } else {
      ok = false;
    }
    // The two column halves of a row hold partial sums over their own columns
    // (same maxima, same rescales): add them through shared memory.
    l_part[g][row] = l;
    named_bar_sync(1, 256);
    const float l_tot = l_part[0][row] + l_part[1][row];
    if (ok && q < p.T) {
      const float inv = 1.f / l_tot;
      const uint64_t inv2 = f2_pack(inv, inv);
      uint32_t w[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        float a0, a1;
        f2_unpack(f2_mul(o[i], inv2), a0, a1);
        w[i] = pack16<F16>(a0, a1);
      }
      __nv_bfloat16* dst = p.out + ((long)b * p.T + q) * p.ld_out + h * kD + g * 64;
#pragma unroll
      for (int gg = 0; gg < 8; ++gg)
        *reinterpret_cast<uint4*>(dst + gg * 8) = make_uint4(w[4 * gg], w[4 * gg + 1], w[4 * gg + 2], w[4 * gg + 3]);
      if (g == 0) p.lse[((long)b * p.nh + h) * p.Tpad + q] = -(m + log2f(l_tot));
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================
// Backward
// ============================================================================
namespace d128 {
constexpr int BWD_STAGES = 3;
constexpr int kHalfSub = 8192;                      // 64 rows x 64 columns bf16 (128B-swizzled)
constexpr int BWD_STAGE = 4 * kHalfSub;             // Q_u lo/hi, dO_u lo/hi
constexpr int OFF_V = kTileBytes;
constexpr int OFF_STAGE = 2 * kTileBytes;
constexpr int OFF_PT = OFF_STAGE + BWD_STAGES * BWD_STAGE;   // P^T_g at + g * 16 KB
constexpr int OFF_DST = OFF_PT + 2 * kSub;                   // dS^T_g at + g * 16 KB
constexpr int OFF_LD = OFF_DST + 2 * kSub;                   // [stage][lse 64 | D 64] fp32
constexpr int BWD_SMEM = OFF_LD + BWD_STAGES * 512 + 1024;
}  // namespace d128

template <bool DROP, bool F16>
__global__ void __launch_bounds__(d128::THREADS, 1)
    attn_bwd_d128_kernel(const __grid_constant__ CUtensorMap tm_kv, const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_do, const __grid_constant__ CUtensorMap tm_dq,
                         AttnParams p) {
  using namespace d128;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_kv, bar_full[BWD_STAGES], bar_empty[BWD_STAGES], bar_h[2], bar_p[2], bar_q[2],
      bar_dqfree[2], bar_done;
  __shared__ uint32_t tmem_slot;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_t = (p.T + kTile - 1) / kTile;
  const int n_h = (p.T + 63) / 64;  // query half-tiles of the sequence
  const int bh = blockIdx.x % (p.B * p.nh);
  const int kt = blockIdx.x / (p.B * p.nh);  // ascending: the CTAs with the most work launch first
  const int h = bh % p.nh;
  const int b = bh / p.nh;
  const int n_u = n_h - 2 * kt;  // half-tiles u = 2 kt + j, j < n_u
  (void)n_t;

  if (threadIdx.x == 0) {
    mbar_init(&bar_kv, 1);
    for (int s = 0; s < BWD_STAGES; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&bar_h[g], 1);
      mbar_init(&bar_p[g], 4);
      mbar_init(&bar_q[g], 1);
      mbar_init(&bar_dqfree[g], 4);
    }
    mbar_init(&bar_done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tm_kv);
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_do);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t tDV = tmem, tDK = tmem + 128;
  const long lse_base = ((long)b * p.nh + h) * p.Tpad;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(&bar_kv, 2 * kTileBytes);
      tma_load_3d(smem, &tm_kv, &bar_kv, p.Hs + h * kD, kt * kTile, b);
      tma_load_3d(smem + kSub, &tm_kv, &bar_kv, p.Hs + h * kD + 64, kt * kTile, b);
      tma_load_3d(smem + OFF_V, &tm_kv, &bar_kv, 2 * p.Hs + h * kD, kt * kTile, b);
      tma_load_3d(smem + OFF_V + kSub, &tm_kv, &bar_kv, 2 * p.Hs + h * kD + 64, kt * kTile, b);
      for (int j = 0; j < n_u; ++j) {
        const int u = 2 * kt + j, st = j % BWD_STAGES;
        if (!mbar_wait(&bar_empty[st], ((j / BWD_STAGES) & 1) ^ 1u, p.status, 70)) break;
        uint8_t* s = smem + OFF_STAGE + st * BWD_STAGE;
        uint8_t* ld = smem + OFF_LD + st * 512;
        mbar_arrive_expect_tx(&bar_full[st], BWD_STAGE + 512);
        tma_load_3d(s, &tm_q, &bar_full[st], h * kD, u * 64, b);
        tma_load_3d(s + kHalfSub, &tm_q, &bar_full[st], h * kD + 64, u * 64, b);
        tma_load_3d(s + 2 * kHalfSub, &tm_do, &bar_full[st], h * kD, u * 64, b);
        tma_load_3d(s + 3 * kHalfSub, &tm_do, &bar_full[st], h * kD + 64, u * 64, b);
        bulk_load(ld, p.lse + lse_base + u * 64, 256, &bar_full[st]);
        bulk_load(ld + 256, p.dvec + lse_base + u * 64, 256, &bar_full[st]);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idH = make_idesc_f16(128, 64, false, false, !F16);   // S^T, dP^T
      constexpr uint32_t idKV = make_idesc_f16(128, 128, false, true, !F16);  // dV, dK
      constexpr uint32_t idQ = make_idesc_f16(128, 64, true, true, !F16);     // dQ^T
      const uint32_t ka = smem_u32(smem), va = smem_u32(smem + OFF_V);
      auto stage_ready = [&](int j) -> bool {
        if (!mbar_wait(&bar_full[j % BWD_STAGES], (j / BWD_STAGES) & 1, p.status, 71)) return false;
        tc_fence_after();
        return true;
      };
      auto issue_sdp = [&](int j) {
        const int g = j & 1;
        const uint32_t qa = smem_u32(smem + OFF_STAGE + (j % BWD_STAGES) * BWD_STAGE);
        const uint32_t doa = qa + 2 * kHalfSub;
        const uint32_t tS = tmem + 256 + g * 128;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t ko = (k >> 2) * kSub + (k & 3) * 32, qo = (k >> 2) * kHalfSub + (k & 3) * 32;
          mma_f16_ss(tS, sw128_desc(ka + ko, 16, 1024), sw128_desc(qa + qo, 16, 1024), idH, k > 0);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t ko = (k >> 2) * kSub + (k & 3) * 32, qo = (k >> 2) * kHalfSub + (k & 3) * 32;
          mma_f16_ss(tS + 64, sw128_desc(va + ko, 16, 1024), sw128_desc(doa + qo, 16, 1024), idH, k > 0);
        }
        mma_commit(&bar_h[g]);
      };
      bool ok = mbar_wait(&bar_kv, 0, p.status, 72);
      for (int j = 0; j < 2 && j < n_u && ok; ++j) {
        if (!stage_ready(j)) {
          ok = false;
          break;
        }
        issue_sdp(j);
      }
      for (int j = 0; j < n_u && ok; ++j) {
        const int g = j & 1;
        if (!mbar_wait(&bar_p[g], (j >> 1) & 1, p.status, 73)) break;
        tc_fence_after();
        const uint32_t qa = smem_u32(smem + OFF_STAGE + (j % BWD_STAGES) * BWD_STAGE);
        const uint32_t doa = qa + 2 * kHalfSub;
        const uint32_t pa = smem_u32(smem + OFF_PT + g * kSub), dsa = smem_u32(smem + OFF_DST + g * kSub);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {  // 64 queries, 16 per step
          mma_f16_ss(tDV, sw128_desc(pa + ks * 32, 16, 1024), sw128_desc(doa + ks * 2048, kHalfSub, 1024), idKV,
                     (j > 0 || ks > 0));
          mma_f16_ss(tDK, sw128_desc(dsa + ks * 32, 16, 1024), sw128_desc(qa + ks * 2048, kHalfSub, 1024), idKV,
                     (j > 0 || ks > 0));
        }
        const uint32_t tQ = tmem + 256 + g * 128;  // dQ^T lands in the consumed S^T_g columns
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)  // 128 keys, 16 per step
          mma_f16_ss(tQ, sw128_desc(ka + ks * 2048, kSub, 1024), sw128_desc(dsa + ks * 2048, 8192, 1024), idQ,
                     ks > 0);
        mma_commit(&bar_q[g]);
        mma_commit(&bar_empty[j % BWD_STAGES]);
        if (j + 2 < n_u) {
          if (!mbar_wait(&bar_dqfree[g], (j >> 1) & 1, p.status, 74)) break;
          tc_fence_after();
          if (!stage_ready(j + 2)) break;
          issue_sdp(j + 2);
        }
      }
      mma_commit(&bar_done);
      mbar_wait(&bar_done, 0, p.status, 75);
    }
  } else {
    const int g = (warp >= 6) ? 1 : 0;  // half-tiles j with j % 2 == g
    const int sub = warp & 3;
    const int r = sub * 32 + lane;  // key row of S^T, dP^T, dK, dV; dh row of dQ^T
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const int key = kt * kTile + r;
    const uint32_t tS = tmem + 256 + g * 128, tDP = tS + 64;
    uint8_t* sPT = smem + OFF_PT + g * kSub;
    uint8_t* sDST = smem + OFF_DST + g * kSub;
    uint32_t dkey = 0;
    uint64_t drop_bh = 0;
    if (DROP) {
      dkey = dropout_key(*p.drop.seed, p.drop.site);
      drop_bh = ((uint64_t)b * p.nh_total + p.h0 + h) * p.T;
    }
    const uint64_t sl2 = f2_pack(p.scale_log2, p.scale_log2), sc2 = f2_pack(p.scale, p.scale);
    bool ok = true;
    for (int j = g; j < n_u && ok; j += 2) {
      const int u = 2 * kt + j, st = j % BWD_STAGES;
      const int q0 = u * 64;
      if (!mbar_wait(&bar_full[st], (j / BWD_STAGES) & 1, p.status, 76) ||
          !mbar_wait(&bar_h[g], (j >> 1) & 1, p.status, 77)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (j >= 2) {  // this warp's staging rows (dQ of half-tile j-2) have been read by their reduce
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
      }
      const float4* lse4 = reinterpret_cast<const float4*>(smem + OFF_LD + st * 512);
      const float4* d4 = lse4 + 16;
      const bool masked = (q0 < kt * kTile + kTile) || (q0 + 64 > p.T);
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t sr[32], dr[32];
        tmem_ld32_issue(tS + c * 32 + lane_off, sr);
        tmem_ld32_issue(tDP + c * 32 + lane_off, dr);
        tmem_wait_ld_regs(sr);
        tmem_pin_regs(dr);
        uint32_t pp[16], dd[16];
#pragma unroll
        for (int i4 = 0; i4 < 8; ++i4) {
          const float4 L = lse4[c * 8 + i4];
          const float4 Dv = d4[c * 8 + i4];
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            const int i = i4 * 4 + e;
            const int qq = q0 + c * 32 + i;
            const uint64_t nl = e ? f2_pack(L.z, L.w) : f2_pack(L.x, L.y);
            const uint64_t nd = e ? f2_pack(Dv.z, Dv.w) : f2_pack(Dv.x, Dv.y);
            float t0, t1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[i]), __uint_as_float(sr[i + 1])), sl2, nl), t0, t1);
            float p0 = fast_exp2(t0), p1 = fast_exp2(t1);
            uint64_t dp2 = f2_pack(__uint_as_float(dr[i]), __uint_as_float(dr[i + 1]));
            float z0 = 1.f, z1 = 1.f;
            if (DROP) {
              const uint64_t e0 = (drop_bh + qq) * (uint64_t)p.T + key;
              const uint64_t e1 = e0 + p.T;
              const uint32_t b0 = dropout_bits(dkey, e0 >> 1), b1 = dropout_bits(dkey, e1 >> 1);
              const uint32_t u0 = (key & 1) ? (b0 >> 16) : (b0 & 0xFFFFu);
              const uint32_t u1 = (key & 1) ? (b1 >> 16) : (b1 & 0xFFFFu);
              z0 = u0 >= p.drop.thresh ? p.drop.scale : 0.f;
              z1 = u1 >= p.drop.thresh ? p.drop.scale : 0.f;
              dp2 = f2_mul(dp2, f2_pack(z0, z1));
            }
            float d0, d1;
            f2_unpack(f2_mul(f2_fma(dp2, sc2, nd), f2_pack(p0, p1)), d0, d1);
            if (DROP) {
              p0 *= z0;
              p1 *= z1;
            }
            if (masked) {
              if (key > qq || qq >= p.T) p0 = d0 = 0.f;
              if (key > qq + 1 || qq + 1 >= p.T) p1 = d1 = 0.f;
            }
            pp[i >> 1] = pack16<F16>(p0, p1);
            dd[i >> 1] = pack16<F16>(d0, d1);
          }
        }
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const uint32_t off = sw128_off(r, c * 4 + q4);
          *reinterpret_cast<uint4*>(sPT + off) = make_uint4(pp[4 * q4], pp[4 * q4 + 1], pp[4 * q4 + 2], pp[4 * q4 + 3]);
          *reinterpret_cast<uint4*>(sDST + off) = make_uint4(dd[4 * q4], dd[4 * q4 + 1], dd[4 * q4 + 2], dd[4 * q4 + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_p[g]);
      // dQ^T of this half-tile: wait for its MMA, take it out of TMEM, free the columns.
      if (!mbar_wait(&bar_q[g], (j >> 1) & 1, p.status, 78)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float v0[32], v1[32];
      tmem_ld32(tS + lane_off, v0);       // queries q0 .. q0+31 of dh row r
      tmem_ld32(tS + 32 + lane_off, v1);  // queries q0+32 .. q0+63
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_dqfree[g]);
      // Stage [32 queries][32 dh] fp32 boxes (128B-swizzled rows) in this warp's own
      // P^T and dS^T rows, which the finished MMAs no longer read.
      uint8_t* stg0 = sPT + sub * 4096;
      uint8_t* stg1 = sDST + sub * 4096;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const uint32_t off = i * 128 + ((((lane >> 2) ^ (i & 7)) << 4) | ((lane & 3) << 2));
        *reinterpret_cast<float*>(stg0 + off) = v0[i];
        *reinterpret_cast<float*>(stg1 + off) = v1[i];
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_3d(&tm_dq, stg0, h * kD + sub * 32, q0, b);
        if (q0 + 32 < p.T) tma_reduce_add_3d(&tm_dq, stg1, h * kD + sub * 32, q0 + 32, b);
        bulk_commit_group();
      }
    }
    // dK, dV: every MMA of the CTA has completed once bar_done fires.
    if (ok && mbar_wait(&bar_done, 0, p.status, 79)) {
      tc_fence_after();
      __nv_bfloat16* drow = p.out + ((long)b * p.T + key) * p.ld_out;
      float v[32];
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          tmem_ld32((which == 0 ? tDK : tDV) + g * 64 + c * 32 + lane_off, v);
          if (key < p.T) {
            __nv_bfloat16* dst = drow + (which == 0 ? p.Hs : 2 * p.Hs) + h * kD + g * 64 + c * 32;
#pragma unroll
            for (int q8 = 0; q8 < 4; ++q8)
              *reinterpret_cast<uint4*>(dst + q8 * 8) =
                  make_uint4(pack16<F16>(v[q8 * 8 + 0], v[q8 * 8 + 1]), pack16<F16>(v[q8 * 8 + 2], v[q8 * 8 + 3]),
                             pack16<F16>(v[q8 * 8 + 4], v[q8 * 8 + 5]), pack16<F16>(v[q8 * 8 + 6], v[q8 * 8 + 7]));
          }
        }
      }
    }
    if (lane == 0) bulk_wait_group0();  // every dQ reduce has landed
    __syncwarp();
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ----------------------------------------------------------------------------
// Host side
// ----------------------------------------------------------------------------
void attn_bwd_prepass(const __nv_bfloat16* o, long ld_o, const __nv_bfloat16* dO, long ld_do, float* dvec,
                      float* dq_acc, int B, int T, int nh, int dh, int Tpad, float scale, bool f16, cudaStream_t s);
void attn_bwd_dq_finish(const float* dq_acc, __nv_bfloat16* dqkv, long ld_dqkv, long rows, int Hs, bool f16,
                        cudaStream_t s);

// The four (dropout, 16-bit format) instantiations of a kernel template.
#define HB_ATTN128_PICK(kern, drop_on, f16)                                                  \
  ((drop_on) ? ((f16) ? kern<true, true> : kern<true, false>)                                \
             : ((f16) ? kern<false, true> : kern<false, false>))

static AttnParams d128_params(int B, int T, int nh, int Tpad, float scale, const DropoutArgs& drop, int h0,
                              int nh_total, int* status) {
  AttnParams p{};
  p.B = B, p.T = T, p.nh = nh, p.Hs = nh * d128::kD, p.Tpad = Tpad;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.drop = drop;
  p.h0 = h0;
  p.nh_total = nh_total;
  p.status = status;
  p.trace = nullptr;
  return p;
}

void attn_fwd_d128_launch(const __nv_bfloat16* qkv, long ld_qkv, __nv_bfloat16* out, long ld_out, float* lse, int B,
                          int T, int nh, int Tpad, float scale, const DropoutArgs& drop, int h0, int nh_total,
                          int* status, bool f16, cudaStream_t s) {
  static bool attr[64] = {};  // the shared-memory opt-in is per device
  const int dev = current_device();
  if (!attr[dev]) {
    for (int d = 0; d < 2; ++d)
      for (int h = 0; h < 2; ++h)
        HB_CUDA_CHECK(cudaFuncSetAttribute(HB_ATTN128_PICK(attn_fwd_d128_kernel, d, h),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, d128::FWD_SMEM));
    attr[dev] = true;
  }
  AttnParams p = d128_params(B, T, nh, Tpad, scale, drop, h0, nh_total, status);
  p.out = out, p.ld_out = ld_out, p.lse = lse;
  const CUtensorMap tm = attn_seq_map(qkv, B, T, ld_qkv, 3 * p.Hs, 128);
  const int n_qt = (T + kTile - 1) / kTile;
  HB_ATTN128_PICK(attn_fwd_d128_kernel, drop.thresh != 0, f16)<<<B * nh * n_qt, d128::THREADS, d128::FWD_SMEM, s>>>(
      tm, p);
  HB_CUDA_CHECK(cudaGetLastError());
}

void attn_bwd_d128_launch(const __nv_bfloat16* qkv, long ld_qkv, const __nv_bfloat16* o, long ld_o,
                          const __nv_bfloat16* dO, long ld_do, const float* lse, float* dvec, float* dq_acc,
                          __nv_bfloat16* dqkv, long ld_dqkv, int B, int T, int nh, int Tpad, float scale,
                          const DropoutArgs& drop, int h0, int nh_total, int* status, bool f16, cudaStream_t s) {
  static bool attr[64] = {};
  const int dev = current_device();
  if (!attr[dev]) {
    for (int d = 0; d < 2; ++d)
      for (int h = 0; h < 2; ++h)
        HB_CUDA_CHECK(cudaFuncSetAttribute(HB_ATTN128_PICK(attn_bwd_d128_kernel, d, h),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, d128::BWD_SMEM));
    attr[dev] = true;
  }
  const int Hs = nh * d128::kD;
  const long rows = (long)B * T;
  attn_bwd_prepass(o, ld_o, dO, ld_do, dvec, dq_acc, B, T, nh, d128::kD, Tpad, scale, f16, s);
  AttnParams p = d128_params(B, T, nh, Tpad, scale, drop, h0, nh_total, status);
  p.out = dqkv, p.ld_out = ld_dqkv, p.lse = const_cast<float*>(lse), p.dvec = dvec, p.dq_acc = dq_acc;
  const CUtensorMap tkv = attn_seq_map(qkv, B, T, ld_qkv, 3 * Hs, 128);
  const CUtensorMap tq = attn_seq_map(qkv, B, T, ld_qkv, 3 * Hs, 64);
  const CUtensorMap td = attn_seq_map(dO, B, T, ld_do, Hs, 64);
  // dQ accumulator as {Hs, T, B} fp32: 32x32 reduce boxes never cross into the next sequence.
  const uint64_t qdims[3] = {static_cast<uint64_t>(Hs), static_cast<uint64_t>(T), static_cast<uint64_t>(B)};
  const uint64_t qstr[2] = {static_cast<uint64_t>(Hs) * 4, static_cast<uint64_t>(Hs) * 4 * T};
  const uint32_t qbox[3] = {32, 32, 1};
  const CUtensorMap tdq =
      make_tmap(CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dq_acc, qdims, qstr, qbox, CU_TENSOR_MAP_SWIZZLE_128B);
  const int n_t = (T + kTile - 1) / kTile;
  HB_ATTN128_PICK(attn_bwd_d128_kernel, drop.thresh != 0, f16)<<<B * nh * n_t, d128::THREADS, d128::BWD_SMEM, s>>>(
      tkv, tq, td, tdq, p);
  HB_CUDA_CHECK(cudaGetLastError());
  attn_bwd_dq_finish(dq_acc, dqkv, ld_dqkv, rows, Hs, f16, s);
}

// ----------------------------------------------------------------------------
// Narrow heads (head_dim 16 or 32) run the head_dim 64 kernels on copies
// whose heads are zero-padded to 64 columns: the padding adds 0 to every
// score and produces output / gradient columns that are dropped. Used by the
// small test models (reference tests/tests_equiv.py: n_embd 64, 4 heads).
// ----------------------------------------------------------------------------
// dst[row, s*nh*64 + h*64 + d] = d < dh ? src[row, s*nh*dh + h*dh + d] : 0   (s < nsec sections)
__global__ void attn_pad_heads_kernel(const __nv_bfloat16* __restrict__ src, long ld_src, __nv_bfloat16* dst,
                                      long ld_dst, long rows, int nsec, int nh, int dh) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long per_row = (long)nsec * nh * 64;
  if (i >= rows * per_row) return;
  const long row = i / per_row;
  const int c = static_cast<int>(i % per_row);
  const int d = c % 64, sh = c / 64;  // sh = s * nh + h
  dst[row * ld_dst + c] = d < dh ? src[row * ld_src + (long)sh * dh + d] : __float2bfloat16(0.f);
}

// dst[row, s*nh*dh + h*dh + d] = src[row, s*nh*64 + h*64 + d]
__global__ void attn_unpad_heads_kernel(const __nv_bfloat16* __restrict__ src, long ld_src, __nv_bfloat16* dst,
                                        long ld_dst, long rows, int nsec, int nh, int dh) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long per_row = (long)nsec * nh * dh;
  if (i >= rows * per_row) return;
  const long row = i / per_row;
  const int c = static_cast<int>(i % per_row);
  const int d = c % dh, sh = c / dh;
  dst[row * ld_dst + c] = src[row * ld_src + (long)sh * 64 + d];
}

void attn_pad_heads(const __nv_bfloat16* src, long ld_src, __nv_bfloat16* dst, long ld_dst, long rows, int nsec,
                    int nh, int dh, cudaStream_t s) {
  const long n = rows * nsec * nh * 64;
  attn_pad_heads_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(src, ld_src, dst, ld_dst, rows, nsec,
                                                                               nh, dh);
  HB_CUDA_CHECK(cudaGetLastError());
}

void attn_unpad_heads(const __nv_bfloat16* src, long ld_src, __nv_bfloat16* dst, long ld_dst, long rows, int nsec,
                      int nh, int dh, cudaStream_t s) {
  const long n = rows * nsec * nh * dh;
  attn_unpad_heads_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(src, ld_src, dst, ld_dst, rows,
                                                                                 nsec, nh, dh);
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
