// Causal flash attention (head_dim 64) on tcgen05 tensor cores.
//
// Replaces F.scaled_dot_product_attention(q, k, v, is_causal=True)
// (reference gpt_model.py:74-81). Q, K and V are read in place from the QKV
// projection output qkv[B*T, 3*Hs] (columns [Q | K | V], each head-major,
// head h at h*64) through one 3-D TMA map {3*Hs, T, B}: a 128-token tile
// never crosses into the next sequence, and rows >= T read as zeros.
//
// Forward, one CTA per (pair of adjacent query tiles 2q, 2q+1, head, batch),
// 320 threads, heaviest pairs launched first; both tiles share each K/V load:
//   warp 0      TMA: Q_A, Q_B, then K0, K1, V0, K2, V1, ... into a 3-slot ring
//   warp 1      MMA: S_X = Q_X K_j^T (128x128 fp32 in TMEM), O_X (+)= P_X V_j
//   warps 2-5   softmax of tile A, warps 6-9 softmax of tile B (thread =
//               query row): row max and exp2 over S in TMEM, P -> 16-bit in
//               128B-swizzled smem (A operand of the PV MMA).
//   O is accumulated in TMEM by the PV MMAs (softmax_tile_ot: the whole score
//   row is loaded at once, exponentials use a reference max that moves only
//   past a threshold, and O is rescaled in TMEM only then); with dropout each
//   PV writes a fresh TMEM buffer that the softmax warps add into registers
//   with the online-softmax rescale (softmax_tile).
//   While one warpgroup runs its softmax, the MMA warp computes the other
//   tile's S or PV, so tensor core and ALUs overlap inside the CTA. A
//   warpgroup releases S as soon as its last TMEM load of S has landed, and
//   the next S is computed while it still exponentiates.
//   TMEM: per tile S [128 cols] + O [64 cols] (with dropout: 2 x 64).
//
// Backward, one CTA per (key tile of 128, head, batch), 320 threads, FA2
// order over the query tiles i >= key tile:
//   S^T = K Q_i^T and dP^T = V dO_i^T are issued as two 64-query halves; the
//   warpgroup of half g (warps 2-5: g = 0, warps 6-9: g = 1; thread = key
//   row) turns its half into P^T and dS^T = P^T (dP^T - D) * scale in smem,
//   then dV += P^T dO_i, dK += dS^T Q_i and dQ_i = dS K (the same smem tiles
//   serve as K-major or MN-major operands); dQ_i is added to an fp32
//   accumulator by bulk tensor reduce-adds (one 32x32 block per warp).
//   As soon as a warpgroup has stored its half of P^T / dS^T, the MMA warp
//   issues that half of the next tile's S^T / dP^T, ahead of the current
//   tile's dV / dK / dQ, so the next softmax starts one MMA later; dQ
//   alternates between two TMEM buffers and is drained off that path.
#include <cuda_bf16.h>

#include <cstdlib>
#include <stdexcept>

#include "attention_common.cuh"
#include "host_utils.h"

namespace hb {

constexpr int kD = 64;
constexpr int kTileBytes = kTile * kD * 2;  // 16 KB
static uint64_t* g_attn_trace = nullptr;
static long g_attn_trace_rows = 0;  // CTAs the trace buffer has rows for

// The trace buffer for a launch of `grid` CTAs: launches with more CTAs than the
// buffer has rows are not traced (each CTA writes its own row).
static uint64_t* attn_trace_for(long grid) { return grid <= g_attn_trace_rows ? g_attn_trace : nullptr; }

// ============================================================================
// Forward
// ============================================================================
constexpr int FWD_SLOTS = 3;
constexpr int FWD_THREADS = 320;
constexpr int FWD_SMEM = 2 * kTileBytes /*Q_A, Q_B*/ + FWD_SLOTS * kTileBytes + 4 * kTileBytes /*P_A, P_B*/ + 1024;

// Position of K_j / V_j in the load sequence K0, K1, V0, K2, V1, ..., K_{n-1}, V_{n-2}, V_{n-1}.
__device__ __forceinline__ int fwd_k_item(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int fwd_v_item(int j, int n) { return (j == n - 1) ? 2 * n - 1 : 2 * j + 2; }

// Exponentials of 32-column chunk c of this thread's score row (keys key0 + 32c
// ..), relative to the reference max (nm2 = -m, packed): P = 2^(s * scale * log2 e
// - m) goes to the swizzled P tile (dropped out where the mask says so), the
// undropped values add to the row-sum pairs sum2. Arguments and sums run on fp32
// pairs; EXPF moves a share of the exponentials to the FMA pipe.
template <bool DIAG, bool DROP, bool F16, int EXPF>
__device__ __forceinline__ void exp_chunk(const uint32_t (&v)[32], int c, uint8_t* sP, int row, int key0, int q,
                                          uint64_t sl2, uint64_t nm2, uint64_t (&sum2)[2], uint32_t dkey,
                                          uint64_t pair_row, uint32_t dthresh, float dscale) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {  // eight columns per 16-byte store, stored as soon as they are packed
    uint32_t pk[4];
#pragma unroll
    for (int i = 8 * g; i < 8 * g + 8; i += 2) {
      float t0, t1;
      f2_unpack(f2_fma(f2_pack(__uint_as_float(v[i]), __uint_as_float(v[i + 1])), sl2, nm2), t0, t1);
      float p0 = fast_exp2(t0), p1;
      if ((EXPF == 1 && (i & 6) == 6) || (EXPF == 2 && (i & 2) == 2)) {
        p1 = exp2_fma(t1);  // this share on the FMA pipe
      } else {
        p1 = fast_exp2(t1);
      }
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
      pk[(i >> 1) & 3] = pack16<F16>(p0, p1);
    }
    *reinterpret_cast<uint4*>(sP + sw128_off(row, c * 4 + g)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  }
}

// Online softmax of one 128x128 score tile held in TMEM, for the calling
// thread's row: updates (m, l), writes P (bf16) to the swizzled smem tile and
// returns the rescale factor of the previous accumulator. TMEM is read in
// pairs of 32-column chunks (two loads in flight, one wait). The row max
// uses three-input max over independent chains and is taken on raw scores
// (the scale is positive); exponent arguments and row sums are computed on
// fp32 pairs (one f32x2 instruction for two columns).
//
// P smem is still being read by the previous PV MMA until `pv_bar` completes its
// phase `pv_phase` (no wait when pv_bar is null): the wait sits between the max
// pass and the first P store, so the max pass overlaps that MMA. Once the last
// TMEM load of S has completed, each warp arrives on `s_free`: the MMA warp may
// then compute the next S into the same columns while this warp still
// exponentiates and stores its last 64 columns. `ok` turns false when the wait
// gives up.
template <bool DIAG, bool DROP, bool F16, int EXPF>
__device__ __forceinline__ float softmax_tile(uint32_t tS, uint32_t lane_off, uint8_t* sP, int row, int key0, int q,
                                              float scale_log2, float& m, float& l, uint32_t dkey, uint64_t pair_row,
                                              uint32_t dthresh, float dscale, uint64_t* pv_bar, uint32_t pv_phase,
                                              uint64_t* s_free, int* status, bool& ok, uint64_t* stamp) {
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
  if (stamp != nullptr) *stamp = globaltimer_ns();  // phase trace: row max done
  if (pv_bar != nullptr && !mbar_wait(pv_bar, pv_phase, status, 27)) {
    ok = false;
    return 0.f;
  }
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    uint32_t va[32], vb[32];
    tmem_ld32_issue(tS + lane_off + (2 * h) * 32, va);
    tmem_ld32_issue(tS + lane_off + (2 * h + 1) * 32, vb);
    tmem_wait_ld_regs(va);
    tmem_pin_regs(vb);
    if (h == 1) {  // every read of S is complete
      tc_fence_before();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(s_free);
    }
#pragma unroll
    for (int half = 0; half < 2; ++half)
      exp_chunk<DIAG, DROP, F16, EXPF>(half ? vb : va, 2 * h + half, sP, row, key0, q, sl2, nm2, sum2, dkey, pair_row,
                                        dthresh, dscale);
  }
  float s0, s1, s2, s3;
  f2_unpack(sum2[0], s0, s1);
  f2_unpack(sum2[1], s2, s3);
  l = l * alpha + ((s0 + s1) + (s2 + s3));
  m = m_new;
  return alpha;
}

// Softmax of one score tile when O is accumulated in TMEM by the PV MMAs (the
// default form). The whole 128-score row is loaded at once (four loads in
// flight, one wait) and S is released to the MMA warp right after; the row max
// and the exponentials then run from registers. The exponentials are taken
// against a reference max m that only moves when the tile's max exceeds it by
// more than kRescaleLog2 (or on the first tile): P <= 2^kRescaleLog2 then, and
// O in TMEM (with l) is rescaled by 2^(m_old - m_new) only on such a move, after
// the previous PV has completed and before this P is handed over. m, l and the
// final O / l are all relative to the same reference, so the result is exact
// whatever the reference.
constexpr float kRescaleLog2 = 8.f;

template <bool DIAG, bool DROP, bool F16, int EXPF>
__device__ __forceinline__ void softmax_tile_ot(uint32_t tS, uint32_t tO, uint32_t lane_off, uint8_t* sP, int row,
                                                int key0, int q, float scale_log2, bool first, float& m, float& l,
                                                uint32_t dkey, uint64_t pair_row, uint32_t dthresh, float dscale,
                                                uint64_t* pv_bar, uint32_t pv_phase, uint64_t* s_free, int* status,
                                                bool& ok, uint64_t* stamp) {
  uint32_t v0[32], v1[32], v2[32], v3[32];
  tmem_ld32_issue(tS + lane_off, v0);
  tmem_ld32_issue(tS + lane_off + 32, v1);
  tmem_ld32_issue(tS + lane_off + 64, v2);
  tmem_ld32_issue(tS + lane_off + 96, v3);
  tmem_wait_ld_regs(v0);
  tmem_pin_regs(v1);
  tmem_pin_regs(v2);
  tmem_pin_regs(v3);
  tc_fence_before();  // every read of S is complete: the next S may be computed
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(s_free);
  float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float a = __uint_as_float(v0[i]), b = __uint_as_float(v1[i]);
    float c = __uint_as_float(v2[i]), d = __uint_as_float(v3[i]);
    if (DIAG) {
      if (key0 + i > q) a = -INFINITY;
      if (key0 + 32 + i > q) b = -INFINITY;
      if (key0 + 64 + i > q) c = -INFINITY;
      if (key0 + 96 + i > q) d = -INFINITY;
    }
    mx[i & 3] = max3f(mx[i & 3], max3f(a, b, c), d);
  }
  const float mt = max3f(mx[0], mx[1], fmaxf(mx[2], mx[3])) * scale_log2;
  float alpha = 1.f;
  if (first) {
    m = mt;
  } else if (mt > m + kRescaleLog2) {
    alpha = fast_exp2(m - mt);
    m = mt;
  }
  if (stamp != nullptr) *stamp = globaltimer_ns();  // phase trace: row max done
  if (pv_bar != nullptr && !mbar_wait(pv_bar, pv_phase, status, 27)) {  // P smem and O: previous PV done
    ok = false;
    return;
  }
  const uint64_t sl2 = f2_pack(scale_log2, scale_log2), nm2 = f2_pack(-m, -m);
  uint64_t sum2[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
  exp_chunk<DIAG, DROP, F16, EXPF>(v0, 0, sP, row, key0, q, sl2, nm2, sum2, dkey, pair_row, dthresh, dscale);
  exp_chunk<DIAG, DROP, F16, EXPF>(v1, 1, sP, row, key0, q, sl2, nm2, sum2, dkey, pair_row, dthresh, dscale);
  exp_chunk<DIAG, DROP, F16, EXPF>(v2, 2, sP, row, key0, q, sl2, nm2, sum2, dkey, pair_row, dthresh, dscale);
  exp_chunk<DIAG, DROP, F16, EXPF>(v3, 3, sP, row, key0, q, sl2, nm2, sum2, dkey, pair_row, dthresh, dscale);
  if (__any_sync(0xffffffffu, alpha != 1.f)) {  // the reference max moved: O *= alpha
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      float o[32];
      tmem_ld32(tO + lane_off + h * 32, o);
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] *= alpha;
      tmem_st32(tO + lane_off + h * 32, o);
    }
  }
  float s0, s1, s2, s3;
  f2_unpack(sum2[0], s0, s1);
  f2_unpack(sum2[1], s2, s3);
  l = l * alpha + ((s0 + s1) + (s2 + s3));
}

// o = o * alpha + (PV result in TMEM, 64 columns of this thread's row); o
// holds column pairs.
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

// OT: O accumulated in TMEM by the PV MMAs (softmax_tile_ot); otherwise each PV
// writes a fresh TMEM buffer that the softmax warps add into registers.
template <bool DROP, bool F16, bool OT>
__global__ void __launch_bounds__(FWD_THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                          // [2][16 KB]
  uint8_t* sSlot = smem + 2 * kTileBytes;      // [3][16 KB]
  uint8_t* sP = sSlot + FWD_SLOTS * kTileBytes;  // [2][32 KB]
  __shared__ uint64_t bar_q, bar_full[FWD_SLOTS], bar_empty[FWD_SLOTS], bar_s[2], bar_sfree[2], bar_p[2], bar_o[2][2],
      bar_done;
  __shared__ uint32_t tmem_slot;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.T + kTile - 1) / kTile;
  const int n_pairs = (n_qt + 1) / 2;
  // Adjacent query tiles (2q, 2q+1) share a CTA, so the two softmax
  // warpgroups see 2q+1 and 2q+2 key tiles: always both busy. Pairs are
  // launched heaviest first (pair index slowest-varying, descending), which
  // keeps the causal work imbalance out of the tail wave.
  const int bh = blockIdx.x % (p.B * p.nh);
  const int pair = n_pairs - 1 - blockIdx.x / (p.B * p.nh);
  const int h = bh % p.nh;
  const int b = bh / p.nh;
  const int qt[2] = {2 * pair, min(2 * pair + 1, n_qt - 1)};
  const bool hasA = qt[0] < qt[1];
  const int n_kv = qt[1] + 1;

  if (threadIdx.x == 0) {
    mbar_init(&bar_q, 1);
    for (int s = 0; s < FWD_SLOTS; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&bar_s[g], 1);
      mbar_init(&bar_sfree[g], 4);
      mbar_init(&bar_p[g], 4);
      mbar_init(&bar_o[g][0], 1);
      mbar_init(&bar_o[g][1], 1);
    }
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
  if (threadIdx.x == 0) HB_TRACE(0);
  // per tile g: S at g*256, O buffers at g*256 + 128 + {0, 64}

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(&bar_q, (hasA ? 2 : 1) * kTileBytes);
      tma_load_3d(sQ + kTileBytes, &tm_qkv, &bar_q, h * kD, qt[1] * kTile, b);
      if (hasA) tma_load_3d(sQ, &tm_qkv, &bar_q, h * kD, qt[0] * kTile, b);
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
        if (!mbar_wait(&bar_empty[slot], ph ^ 1u, p.status, 20)) break;
        mbar_arrive_expect_tx(&bar_full[slot], kTileBytes);
        tma_load_3d(sSlot + slot * kTileBytes, &tm_qkv, &bar_full[slot], (is_v ? 2 : 1) * p.Hs + h * kD,
                    kv * kTile, b);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = make_idesc_f16(128, 128, false, false, !F16);
      constexpr uint32_t idO = make_idesc_f16(128, 64, false, true, !F16);
      bool ok = mbar_wait(&bar_q, 0, p.status, 21);
      HB_TRACE(1);
      auto item = [&](int idx, uint32_t& addr) -> bool {
        const int slot = idx % FWD_SLOTS;
        if (!mbar_wait(&bar_full[slot], (idx / FWD_SLOTS) & 1, p.status, 22)) return false;
        tc_fence_after();
        addr = smem_u32(sSlot + slot * kTileBytes);
        return true;
      };
      auto issue_s = [&](int g, uint32_t ka) {
        const uint32_t qa = smem_u32(sQ + g * kTileBytes);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_f16_ss(tmem + g * 256, sw128_desc(qa + k * 32, 16, 1024), sw128_desc(ka + k * 32, 16, 1024), idS, k > 0);
        mma_commit(&bar_s[g]);
      };
      auto issue_pv = [&](int g, int j, uint32_t va) {
        const uint32_t pa = smem_u32(sP + g * 2 * kTileBytes);
        const uint32_t tO = tmem + g * 256 + 128 + (OT ? 0 : (j & 1) * 64);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_f16_ss(tO, sw128_desc(pa + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024),
                     sw128_desc(va + ks * 2048, 8192, 1024), idO, (OT && j > 0) || ks > 0);
        mma_commit(&bar_o[g][OT ? 0 : (j & 1)]);
      };
      uint32_t ka = 0, va = 0;
      if (ok && item(fwd_k_item(0), ka)) {
        if (hasA) issue_s(0, ka);
        issue_s(1, ka);
        mma_commit(&bar_empty[fwd_k_item(0) % FWD_SLOTS]);
      } else {
        ok = false;
      }
      // Step j: S_{j+1} of each tile as soon as its softmax has read S_j (s_free),
      // then PV_j of each tile once its P_j is in smem.
      for (int j = 0; j < n_kv && ok; ++j) {
        const bool next = j + 1 < n_kv;
        const bool a_on = hasA && j <= qt[0];
        if (a_on && j + 1 <= qt[0]) {
          if (!mbar_wait(&bar_sfree[0], j & 1, p.status, 29)) break;
          tc_fence_after();
          if (!item(fwd_k_item(j + 1), ka)) break;
          issue_s(0, ka);
        }
        if (next) {
          if (!mbar_wait(&bar_sfree[1], j & 1, p.status, 30)) break;
          tc_fence_after();
          if (!item(fwd_k_item(j + 1), ka)) break;
          issue_s(1, ka);
          mma_commit(&bar_empty[fwd_k_item(j + 1) % FWD_SLOTS]);
        }
        if (a_on) {
          if (!mbar_wait(&bar_p[0], j & 1, p.status, 23)) break;
          tc_fence_after();
          if (!item(fwd_v_item(j, n_kv), va)) break;
          issue_pv(0, j, va);
        }
        if (!mbar_wait(&bar_p[1], j & 1, p.status, 24)) break;
        tc_fence_after();
        if (!item(fwd_v_item(j, n_kv), va)) break;
        issue_pv(1, j, va);
        mma_commit(&bar_empty[fwd_v_item(j, n_kv) % FWD_SLOTS]);
      }
      mma_commit(&bar_done);
      mbar_wait(&bar_done, 0, p.status, 25);
    }
  } else {
    const int g = (warp >= 6) ? 1 : 0;
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    if (OT && (g == 1 || hasA)) {
      const int my_qt = qt[g];
      const int n = my_qt + 1;
      const int q = my_qt * kTile + row;
      const uint32_t tS = tmem + g * 256, tO = tmem + g * 256 + 128;
      uint8_t* myP = sP + g * 2 * kTileBytes;
      float m = 0.f, l = 0.f;  // reference max (log2 domain; set by the first tile) and row sum
      uint32_t dkey = 0;
      uint64_t pair_row = 0;
      if (DROP) {
        dkey = dropout_key(*p.drop.seed, p.drop.site);
        pair_row = ((((uint64_t)b * p.nh_total + p.h0 + h) * p.T + q) * p.T) >> 1;
      }
      bool ok = true;
      for (int j = 0; j < n && ok; ++j) {
        if (!mbar_wait(&bar_s[g], j & 1, p.status, 26)) {
          ok = false;
          break;
        }
        if (lane == 0 && sub == 0 && j < 8) HB_TRACE(8 + 24 * g + j);
        tc_fence_after();
        if (lane == 0 && sub == 0 && j < 8) HB_TRACE(16 + 24 * g + j);
        // P smem and O in TMEM are free once PV_{j-1} has completed (waited inside, after the row max).
        uint64_t* pv_bar = j > 0 ? &bar_o[g][0] : nullptr;
        const uint32_t pv_phase = (j - 1) & 1;
        uint64_t* stamp = (p.trace != nullptr && lane == 0 && sub == 0 && j < 8)
                              ? p.trace + (long)blockIdx.x * kTraceSlots + 56 + 8 * g + j
                              : nullptr;
#define HB_SOFTMAX_OT(DIAG, EXPF)                                                                                 \
  softmax_tile_ot<DIAG, DROP, F16, EXPF>(tS, tO, lane_off, myP, row, j * kTile, q, p.scale_log2, j == 0, m, l, dkey, \
                                         pair_row, p.drop.thresh, p.drop.scale, pv_bar, pv_phase, &bar_sfree[g],    \
                                         p.status, ok, stamp)
        // Two bodies: the diagonal tile's, and the off-diagonal one with one
        // exponential in eight on the FMA pipe (measured as fast as selecting the
        // share at run time among three compiled bodies: 49.1 us).
        if (j == my_qt) {
          HB_SOFTMAX_OT(true, 0);
        } else {
          HB_SOFTMAX_OT(false, 1);
        }
#undef HB_SOFTMAX_OT
        if (!ok) break;
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_p[g]);
        if (lane == 0 && sub == 0 && j < 8) HB_TRACE(24 + 24 * g + j);
      }
      if (ok && mbar_wait(&bar_o[g][0], (n - 1) & 1, p.status, 28)) {
        tc_fence_after();
        float oa[32], ob[32];
        tmem_ld32(tO + lane_off, oa);
        tmem_ld32(tO + lane_off + 32, ob);
        if (q < p.T) {
          const float inv = 1.f / l;
          uint32_t w[32];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            w[i] = pack16<F16>(oa[2 * i] * inv, oa[2 * i + 1] * inv);
            w[16 + i] = pack16<F16>(ob[2 * i] * inv, ob[2 * i + 1] * inv);
          }
          __nv_bfloat16* dst = p.out + ((long)b * p.T + q) * p.ld_out + h * kD;
#pragma unroll
          for (int gg = 0; gg < 8; ++gg)
            *reinterpret_cast<uint4*>(dst + gg * 8) = make_uint4(w[4 * gg], w[4 * gg + 1], w[4 * gg + 2], w[4 * gg + 3]);
          p.lse[((long)b * p.nh + h) * p.Tpad + q] = -(m + log2f(l));
        }
      }
    } else if (!OT && (g == 1 || hasA)) {
      const int my_qt = qt[g];
      const int n = my_qt + 1;
      const int q = my_qt * kTile + row;
      const uint32_t tS = tmem + g * 256, tO0 = tmem + g * 256 + 128;
      uint8_t* myP = sP + g * 2 * kTileBytes;
      float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
      uint32_t dkey = 0;
      uint64_t pair_row = 0;
      if (DROP) {
        dkey = dropout_key(*p.drop.seed, p.drop.site);
        pair_row = ((((uint64_t)b * p.nh_total + p.h0 + h) * p.T + q) * p.T) >> 1;
      }
      uint64_t o[32];  // output row as 32 column pairs
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] = f2_pack(0.f, 0.f);
      bool ok = true;
      for (int j = 0; j < n && ok; ++j) {
        if (!mbar_wait(&bar_s[g], j & 1, p.status, 26)) {
          ok = false;
          break;
        }
        if (lane == 0 && sub == 0 && j < 8) HB_TRACE(8 + 24 * g + j);
        tc_fence_after();
        if (lane == 0 && sub == 0 && j < 8) HB_TRACE(16 + 24 * g + j);
        // P smem is free once PV_{j-1} has completed (waited inside, after the max pass).
        uint64_t* pv_bar = j > 0 ? &bar_o[g][(j - 1) & 1] : nullptr;
        const uint32_t pv_phase = ((j - 1) >> 1) & 1;
        uint64_t* stamp = (p.trace != nullptr && lane == 0 && sub == 0 && j < 8)
                              ? p.trace + (long)blockIdx.x * kTraceSlots + 56 + 8 * g + j
                              : nullptr;
#define HB_SOFTMAX(DIAG, EXPF)                                                                               \
  softmax_tile<DIAG, DROP, F16, EXPF>(tS, lane_off, myP, row, j * kTile, q, p.scale_log2, m, l, dkey, pair_row, \
                                      p.drop.thresh, p.drop.scale, pv_bar, pv_phase, &bar_sfree[g], p.status, ok, \
                                      stamp)
        float alpha;
        if (j == my_qt) {
          alpha = HB_SOFTMAX(true, 0);
        } else if (p.exp_fma == 1) {
          alpha = HB_SOFTMAX(false, 1);
        } else if (p.exp_fma == 2) {
          alpha = HB_SOFTMAX(false, 2);
        } else {
          alpha = HB_SOFTMAX(false, 0);
        }
#undef HB_SOFTMAX
        if (!ok) break;
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_p[g]);
        if (lane == 0 && sub == 0 && j < 8) HB_TRACE(24 + 24 * g + j);
        if (j > 0) {
          tc_fence_after();
          accumulate_o(o, tO0 + ((j - 1) & 1) * 64 + lane_off, alpha_prev);
        }
        alpha_prev = alpha;
      }
      if (ok && mbar_wait(&bar_o[g][(n - 1) & 1], ((n - 1) >> 1) & 1, p.status, 28)) {
        tc_fence_after();
        accumulate_o(o, tO0 + ((n - 1) & 1) * 64 + lane_off, alpha_prev);
        if (q < p.T) {
          const float inv = 1.f / l;
          const uint64_t inv2 = f2_pack(inv, inv);
          uint32_t w[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float a0, a1;
            f2_unpack(f2_mul(o[i], inv2), a0, a1);
            w[i] = pack16<F16>(a0, a1);
          }
          __nv_bfloat16* dst = p.out + ((long)b * p.T + q) * p.ld_out + h * kD;
#pragma unroll
          for (int gg = 0; gg < 8; ++gg)
            *reinterpret_cast<uint4*>(dst + gg * 8) = make_uint4(w[4 * gg], w[4 * gg + 1], w[4 * gg + 2], w[4 * gg + 3]);
          p.lse[((long)b * p.nh + h) * p.Tpad + q] = -(m + log2f(l));
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
  if (threadIdx.x == 0) HB_TRACE(2);
}

// ============================================================================
// Backward
// ============================================================================
constexpr int BWD_STAGE = 2 * kTileBytes + 2048;  // Q_i, dO_i, lse_i (512 B), D_i (512 B), padded to 1 KB multiple
constexpr int BWD_STAGES = 2;
constexpr int BWD_THREADS = 320;
constexpr int BWD_DQ_STG = 8 * 4096;  // per softmax warp: 32 query rows x 32 fp32 dQ columns, 128B-swizzled
constexpr int BWD_SMEM = 2 * kTileBytes /*K,V*/ + BWD_STAGES * BWD_STAGE + 4 * kTileBytes /*P^T, dS^T*/ +
                         BWD_DQ_STG + 1024;

template <bool DROP, bool F16>
__global__ void __launch_bounds__(BWD_THREADS, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_dq, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + kTileBytes;
  uint8_t* sStage = smem + 2 * kTileBytes;
  uint8_t* sP = sStage + BWD_STAGES * BWD_STAGE;
  uint8_t* sDS = sP + 2 * kTileBytes;
  uint8_t* sDQ = sDS + 2 * kTileBytes;
  __shared__ uint64_t bar_kv, bar_full[BWD_STAGES], bar_empty[BWD_STAGES], bar_h[2], bar_p[2], bar_mma, bar_done;
  __shared__ uint32_t tmem_slot;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_t = (p.T + kTile - 1) / kTile;
  // Key tile slowest-varying, ascending: the CTAs with the most query tiles launch first.
  const int bh = blockIdx.x % (p.B * p.nh);
  const int kt = blockIdx.x / (p.B * p.nh);
  const int h = bh % p.nh;
  const int b = bh / p.nh;
  const int n_i = n_t - kt;  // query tiles kt .. n_t-1

  if (threadIdx.x == 0) {
    mbar_init(&bar_kv, 1);
    for (int s = 0; s < BWD_STAGES; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&bar_h[g], 1);
      mbar_init(&bar_p[g], 4);
    }
    mbar_init(&bar_mma, 1);
    mbar_init(&bar_done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tm_qkv);
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
  if (threadIdx.x == 0) HB_TRACE(0);
  // dQ alternates between two 64-column buffers (tile ii in buffer ii & 1), so the
  // softmax warps drain tile ii-1's dQ after handing over tile ii's P^T / dS^T.
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 320, tDQ = tmem + 384;
  const long lse_base = ((long)b * p.nh + h) * p.Tpad;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(&bar_kv, 2 * kTileBytes);
      tma_load_3d(sK, &tm_qkv, &bar_kv, p.Hs + h * kD, kt * kTile, b);
      tma_load_3d(sV, &tm_qkv, &bar_kv, 2 * p.Hs + h * kD, kt * kTile, b);
      for (int ii = 0; ii < n_i; ++ii) {
        const int qi = kt + ii, st = ii % BWD_STAGES;
        if (!mbar_wait(&bar_empty[st], ((ii / BWD_STAGES) & 1) ^ 1u, p.status, 40)) break;
        uint8_t* s = sStage + st * BWD_STAGE;
        mbar_arrive_expect_tx(&bar_full[st], 2 * kTileBytes + 1024);
        tma_load_3d(s, &tm_qkv, &bar_full[st], h * kD, qi * kTile, b);
        tma_load_3d(s + kTileBytes, &tm_do, &bar_full[st], h * kD, qi * kTile, b);
        bulk_load(s + 2 * kTileBytes, p.lse + lse_base + qi * kTile, 512, &bar_full[st]);
        bulk_load(s + 2 * kTileBytes + 512, p.dvec + lse_base + qi * kTile, 512, &bar_full[st]);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idH = make_idesc_f16(128, 64, false, false, !F16);   // S^T / dP^T halves
      constexpr uint32_t idKM = make_idesc_f16(128, 64, false, true, !F16);   // dV, dK
      constexpr uint32_t idQ = make_idesc_f16(128, 64, true, true, !F16);     // dQ
      const uint32_t ka = smem_u32(sK), va = smem_u32(sV), pa = smem_u32(sP), dsa = smem_u32(sDS);
      auto stage_ready = [&](int ii) -> bool {
        if (!mbar_wait(&bar_full[ii % BWD_STAGES], (ii / BWD_STAGES) & 1, p.status, 41)) return false;
        tc_fence_after();
        return true;
      };
      auto issue_half = [&](int ii, int g) {
        const uint32_t qa = smem_u32(sStage + (ii % BWD_STAGES) * BWD_STAGE) + g * 8192;
        const uint32_t doa = qa + kTileBytes;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_f16_ss(tS + g * 64, sw128_desc(ka + k * 32, 16, 1024), sw128_desc(qa + k * 32, 16, 1024), idH, k > 0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_f16_ss(tDP + g * 64, sw128_desc(va + k * 32, 16, 1024), sw128_desc(doa + k * 32, 16, 1024), idH, k > 0);
        mma_commit(&bar_h[g]);
      };
      bool ok = mbar_wait(&bar_kv, 0, p.status, 42) && stage_ready(0);
      HB_TRACE(1);
      if (ok) {
        issue_half(0, 0);
        issue_half(0, 1);
      }
      for (int ii = 0; ii < n_i && ok; ++ii) {
        const uint32_t qa = smem_u32(sStage + (ii % BWD_STAGES) * BWD_STAGE);
        const uint32_t doa = qa + kTileBytes;
        // Half g of P^T / dS^T in smem means half g of S^T / dP^T has been read:
        // the next tile's half g goes to the tensor core first (it heads the
        // softmax warps' critical path), then this tile's dV / dK / dQ.
        if (!mbar_wait(&bar_p[0], ii & 1, p.status, 43)) break;
        if (ii < 8) HB_TRACE(8 + ii);
        tc_fence_after();
        const bool next = ii + 1 < n_i;
        if (next) {
          if (!stage_ready(ii + 1)) break;
          issue_half(ii + 1, 0);
        }
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          mma_f16_ss(tDV, sw128_desc(pa + ks * 32, 16, 1024), sw128_desc(doa + ks * 2048, 8192, 1024), idKM,
                     (ii > 0 || ks > 0));
          mma_f16_ss(tDK, sw128_desc(dsa + ks * 32, 16, 1024), sw128_desc(qa + ks * 2048, 8192, 1024), idKM,
                     (ii > 0 || ks > 0));
        }
        if (!mbar_wait(&bar_p[1], ii & 1, p.status, 44)) break;
        if (ii < 8) HB_TRACE(16 + ii);
        tc_fence_after();
        if (next) issue_half(ii + 1, 1);
#pragma unroll
        for (int ks = 4; ks < 8; ++ks) {
          mma_f16_ss(tDV, sw128_desc(pa + 16384 + (ks - 4) * 32, 16, 1024), sw128_desc(doa + ks * 2048, 8192, 1024),
                     idKM, 1u);
          mma_f16_ss(tDK, sw128_desc(dsa + 16384 + (ks - 4) * 32, 16, 1024), sw128_desc(qa + ks * 2048, 8192, 1024),
                     idKM, 1u);
        }
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_f16_ss(tDQ + (ii & 1) * 64, sw128_desc(dsa + ks * 2048, 16384, 1024),
                     sw128_desc(ka + ks * 2048, 8192, 1024), idQ, ks > 0);
        mma_commit(&bar_mma);
        mma_commit(&bar_empty[ii % BWD_STAGES]);
      }
      mma_commit(&bar_done);
      mbar_wait(&bar_done, 0, p.status, 45);
    }
  } else {
    const int g = (warp >= 6) ? 1 : 0;  // query half handled by this warpgroup
    const int sub = warp & 3;
    const int r = sub * 32 + lane;  // key row (S^T, dP^T, dK, dV) / query row (dQ)
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const int key = kt * kTile + r;
    bool ok = true;
    uint32_t dkey = 0;
    uint64_t drop_bh = 0;  // (b * nh_total + h0 + h) * T: first query row of this head
    if (DROP) {
      dkey = dropout_key(*p.drop.seed, p.drop.site);
      drop_bh = ((uint64_t)b * p.nh_total + p.h0 + h) * p.T;
    }
    // dQ rows of this warp (32 queries x 32 columns) leave through one bulk
    // tensor reduce-add into the fp32 accumulator (the add happens in L2).
    uint8_t* dq_stg = sDQ + (warp - 2) * 4096;
    auto flush_dq = [&](int ii) {
      const int qi = kt + ii;
      tc_fence_after();
      float v[32];
      tmem_ld32(tDQ + (ii & 1) * 64 + g * 32 + lane_off, v);
      if (lane == 0) bulk_wait_group_read0();  // the previous reduce has read the staging tile
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float4*>(dq_stg + lane * 128 + ((j ^ (lane & 7)) << 4)) =
            make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_3d(&tm_dq, dq_stg, h * kD + g * 32, qi * kTile + sub * 32, b);
        bulk_commit_group();
      }
    };
    for (int ii = 0; ii < n_i && ok; ++ii) {
      const int qi = kt + ii, st = ii % BWD_STAGES;
      if (!mbar_wait(&bar_full[st], (ii / BWD_STAGES) & 1, p.status, 46) ||
          !mbar_wait(&bar_h[g], ii & 1, p.status, 47)) {
        ok = false;
        break;
      }
      if (lane == 0 && sub == 0 && ii < 8) HB_TRACE(24 + 24 * g + ii);
      tc_fence_after();
      const float* s_lse = reinterpret_cast<const float*>(sStage + st * BWD_STAGE + 2 * kTileBytes) + g * 64;
      const float* s_d = s_lse + 128;
      const bool diag = (qi == kt);
      // Only the diagonal tile and a tile crossing T need per-element masks.
      const bool masked_tile = diag || (qi + 1) * kTile > p.T;
      const float4* lse4 = reinterpret_cast<const float4*>(s_lse);
      const float4* d4 = reinterpret_cast<const float4*>(s_d);
      bool waited = (ii == 0);  // P^T / dS^T smem is free before the first tile
      // Two 32-column chunks of this half: both TMEM loads in flight at once,
      // P^T and dS^T packed to bf16 and stored right away (few live registers).
#pragma unroll 1
      for (int c = 0; c < 2 && ok; ++c) {
        uint32_t sr[32], dr[32];
        tmem_ld32_issue(tS + g * 64 + c * 32 + lane_off, sr);
        tmem_ld32_issue(tDP + g * 64 + c * 32 + lane_off, dr);
        tmem_wait_ld_regs(sr);
        tmem_pin_regs(dr);
        uint32_t pp[16], dd[16];
        const uint64_t sl2 = f2_pack(p.scale_log2, p.scale_log2), sc2 = f2_pack(p.scale, p.scale);
        // dropout: this thread's key is fixed; element (query qq, key) lives in
        // pair (row_qq + key) / 2 and takes the half selected by key's parity
        const uint64_t q_first = (uint64_t)qi * kTile + g * 64 + c * 32;
#pragma unroll
        for (int i4 = 0; i4 < 8; ++i4) {
          // staged per query column: -lse (log2 domain) and -scale * D
          const float4 L = lse4[c * 8 + i4];
          const float4 Dv = d4[c * 8 + i4];
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            const int i = i4 * 4 + e;
            const uint64_t nl = e ? f2_pack(L.z, L.w) : f2_pack(L.x, L.y);
            const uint64_t nd = e ? f2_pack(Dv.z, Dv.w) : f2_pack(Dv.x, Dv.y);
            float t0, t1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[i]), __uint_as_float(sr[i + 1])), sl2, nl), t0, t1);
            float p0 = fast_exp2(t0), p1 = fast_exp2(t1);  // P = 2^(s * scale * log2 e - lse)
            uint64_t dp2 = f2_pack(__uint_as_float(dr[i]), __uint_as_float(dr[i + 1]));
            float z0 = 1.f, z1 = 1.f;
            if (DROP) {  // dP = Z * dO V^T;  dV operand P * Z
              const uint64_t e0 = (drop_bh + q_first + i) * (uint64_t)p.T + key;
              const uint64_t e1 = e0 + p.T;
              const uint32_t b0 = dropout_bits(dkey, e0 >> 1), b1 = dropout_bits(dkey, e1 >> 1);
              const uint32_t u0 = (key & 1) ? (b0 >> 16) : (b0 & 0xFFFFu);
              const uint32_t u1 = (key & 1) ? (b1 >> 16) : (b1 & 0xFFFFu);
              z0 = u0 >= p.drop.thresh ? p.drop.scale : 0.f;
              z1 = u1 >= p.drop.thresh ? p.drop.scale : 0.f;
              dp2 = f2_mul(dp2, f2_pack(z0, z1));
            }
            // dS = P * (dP * scale - D * scale)
            const uint64_t u = f2_fma(dp2, sc2, nd);
            float d0, d1;
            f2_unpack(f2_mul(u, f2_pack(p0, p1)), d0, d1);
            if (DROP) {
              p0 *= z0;
              p1 *= z1;
            }
            if (masked_tile) {
              const int qq = qi * kTile + g * 64 + c * 32 + i;
              if ((diag && key > qq) || qq >= p.T) p0 = d0 = 0.f;
              if ((diag && key > qq + 1) || qq + 1 >= p.T) p1 = d1 = 0.f;
            }
            pp[i >> 1] = pack16<F16>(p0, p1);
            dd[i >> 1] = pack16<F16>(d0, d1);
          }
        }
        // The previous tile's MMAs read P^T / dS^T smem: wait once before
        // overwriting this half (its dQ is drained after the hand-over below).
        if (!waited) {
          if (!mbar_wait(&bar_mma, (ii - 1) & 1, p.status, 48)) {
            ok = false;
            break;
          }
          if (lane == 0 && sub == 0 && ii < 8) HB_TRACE(32 + 24 * g + ii);
          waited = true;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t off = sw128_off(r, g * 8 + c * 4 + q);
          *reinterpret_cast<uint4*>(sP + off) = make_uint4(pp[4 * q], pp[4 * q + 1], pp[4 * q + 2], pp[4 * q + 3]);
          *reinterpret_cast<uint4*>(sDS + off) = make_uint4(dd[4 * q], dd[4 * q + 1], dd[4 * q + 2], dd[4 * q + 3]);
        }
      }
      if (!ok) break;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_p[g]);
      if (lane == 0 && sub == 0 && ii < 8) HB_TRACE(40 + 24 * g + ii);
      // Tile ii-1's dQ (complete: bar_mma was waited above) leaves its buffer
      // before this warpgroup can hand over tile ii+1, whose dQ MMA reuses it.
      if (ii > 0) flush_dq(ii - 1);
    }
    if (ok && mbar_wait(&bar_mma, (n_i - 1) & 1, p.status, 49)) {
      flush_dq(n_i - 1);
      // dK, dV columns [g*32, g*32+32) -> bf16 into the K / V columns of dqkv.
      __nv_bfloat16* drow = p.out + ((long)b * p.T + key) * p.ld_out;
      float v[32];
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        tmem_ld32((which == 0 ? tDK : tDV) + g * 32 + lane_off, v);
        if (key < p.T) {
          __nv_bfloat16* dst = drow + (which == 0 ? p.Hs : 2 * p.Hs) + h * kD + g * 32;
#pragma unroll
          for (int q8 = 0; q8 < 4; ++q8)
            *reinterpret_cast<uint4*>(dst + q8 * 8) =
                make_uint4(pack16<F16>(v[q8 * 8 + 0], v[q8 * 8 + 1]), pack16<F16>(v[q8 * 8 + 2], v[q8 * 8 + 3]),
                           pack16<F16>(v[q8 * 8 + 4], v[q8 * 8 + 5]), pack16<F16>(v[q8 * 8 + 6], v[q8 * 8 + 7]));
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
  if (threadIdx.x == 0) HB_TRACE(2);
}

// dvec[b, h, t] = -scale * D,  D = sum_d dO[b*T+t, h*DH+d] * O[b*T+t, h*DH+d]   (fp32)
template <int DH, bool F16>
__global__ void attn_bwd_dvec_kernel(const __nv_bfloat16* __restrict__ o, long ld_o, const __nv_bfloat16* __restrict__ dO,
                                     long ld_do, float* __restrict__ dvec, int B, int T, int nh, int Tpad,
                                     float scale) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)B * T * nh) return;
  const int h = i % nh;
  const long row = i / nh;
  const int b = row / T, t = row % T;
  const uint4* a = reinterpret_cast<const uint4*>(o + row * ld_o + h * DH);
  const uint4* g = reinterpret_cast<const uint4*>(dO + row * ld_do + h * DH);
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < DH / 8; ++k) {
    const uint4 x = a[k], y = g[k];
    const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, yw[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) s += lo16<F16>(xw[q]) * lo16<F16>(yw[q]) + hi16<F16>(xw[q]) * hi16<F16>(yw[q]);
  }
  dvec[((long)b * nh + h) * Tpad + t] = -scale * s;
}

// dqkv[:, c] = 16-bit(dq_acc[:, c]) for the Q columns c < Hs
template <bool F16>
__global__ void attn_bwd_dq_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dqkv, long ld,
                                   long rows, int Hs) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long n4 = rows * Hs / 4;
  if (i >= n4) return;
  const long e = i * 4;
  const long row = e / Hs;
  const int c = e % Hs;
  const float4 v = reinterpret_cast<const float4*>(dq_acc)[i];
  *reinterpret_cast<uint2*>(dqkv + row * ld + c) = make_uint2(pack16<F16>(v.x, v.y), pack16<F16>(v.z, v.w));
}

// Backward pre-pass of every head width: dvec = -scale * rowsum(dO * O) and a
// zeroed fp32 dQ accumulator.
void attn_bwd_prepass(const __nv_bfloat16* o, long ld_o, const __nv_bfloat16* dO, long ld_do, float* dvec,
                      float* dq_acc, int B, int T, int nh, int dh, int Tpad, float scale, bool f16, cudaStream_t s) {
  const long rows = (long)B * T;
  const unsigned grid = static_cast<unsigned>((rows * nh + 255) / 256);
  auto kern = dh == 64 ? (f16 ? attn_bwd_dvec_kernel<64, true> : attn_bwd_dvec_kernel<64, false>)
                       : (f16 ? attn_bwd_dvec_kernel<128, true> : attn_bwd_dvec_kernel<128, false>);
  if (dh != 64 && dh != 128) throw std::runtime_error("attention backward: head_dim must be 64 or 128 here");
  kern<<<grid, 256, 0, s>>>(o, ld_o, dO, ld_do, dvec, B, T, nh, Tpad, scale);
  HB_CUDA_CHECK(cudaGetLastError());
  HB_CUDA_CHECK(cudaMemsetAsync(dq_acc, 0, sizeof(float) * rows * nh * dh, s));
}

// dQ accumulator -> bf16 Q columns of dqkv.
void attn_bwd_dq_finish(const float* dq_acc, __nv_bfloat16* dqkv, long ld_dqkv, long rows, int Hs, bool f16,
                        cudaStream_t s) {
  auto kern = f16 ? attn_bwd_dq_kernel<true> : attn_bwd_dq_kernel<false>;
  kern<<<(rows * Hs / 4 + 255) / 256, 256, 0, s>>>(dq_acc, dqkv, ld_dqkv, rows, Hs);
  HB_CUDA_CHECK(cudaGetLastError());
}

// ----------------------------------------------------------------------------
CUtensorMap attn_seq_map(const void* base, int B, int T, long ld, int cols, int box_rows) {
  const uint64_t dims[3] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(T), static_cast<uint64_t>(B)};
  const uint64_t strides[2] = {static_cast<uint64_t>(ld) * 2, static_cast<uint64_t>(ld) * 2 * T};
  const uint32_t box[3] = {64, static_cast<uint32_t>(box_rows), 1};
  return make_tmap_bf16(3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}
static CUtensorMap qkv_map(const void* base, int B, int T, long ld, int cols) {
  return attn_seq_map(base, B, T, ld, cols, 128);
}

// The four (dropout, 16-bit format) instantiations of a kernel template.
#define HB_ATTN_PICK(kern, drop_on, f16)                                                     \
  ((drop_on) ? ((f16) ? kern<true, true> : kern<true, false>)                                \
             : ((f16) ? kern<false, true> : kern<false, false>))

// HB_ATTN_FWD_OT=0 selects the head_dim 64 forward that accumulates O in registers
// (the default accumulates O in TMEM: attn_fwd_kernel<., ., true>).
static bool attn_fwd_ot() {
  static const bool on = [] {
    const char* v = std::getenv("HB_ATTN_FWD_OT");
    return !(v && v[0] == '0');
  }();
  return on;
}

// The forward's eight (dropout, 16-bit format, O in TMEM) instantiations.
#define HB_ATTN_FWD_PICK(drop_on, f16, ot)                                                                  \
  ((ot) ? ((drop_on) ? ((f16) ? attn_fwd_kernel<true, true, true> : attn_fwd_kernel<true, false, true>)     \
                     : ((f16) ? attn_fwd_kernel<false, true, true> : attn_fwd_kernel<false, false, true>))  \
        : ((drop_on) ? ((f16) ? attn_fwd_kernel<true, true, false> : attn_fwd_kernel<true, false, false>)   \
                     : ((f16) ? attn_fwd_kernel<false, true, false> : attn_fwd_kernel<false, false, false>)))

// HB_ATTN_EXP_FMA (0, 1, 2) sets AttnParams::exp_fma of the head_dim 64 forward (default 1).
static int attn_exp_fma() {
  static const int m = [] {
    const char* v = std::getenv("HB_ATTN_EXP_FMA");
    return (v && v[0] >= '0' && v[0] <= '2') ? v[0] - '0' : 1;
  }();
  return m;
}

void attn_fwd_launch(const __nv_bfloat16* qkv, long ld_qkv, __nv_bfloat16* out, long ld_out, float* lse, int B,
                     int T, int nh, int Tpad, float scale, const DropoutArgs& drop, int h0, int nh_total, int* status,
                     bool f16, cudaStream_t s) {
  static bool attr[64] = {};  // the shared-memory opt-in is per device
  const int dev = current_device();
  if (!attr[dev]) {
    for (int d = 0; d < 2; ++d)
      for (int h = 0; h < 2; ++h)
        for (int o = 0; o < 2; ++o)
          HB_CUDA_CHECK(cudaFuncSetAttribute(HB_ATTN_FWD_PICK(d, h, o), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             FWD_SMEM));
    attr[dev] = true;
  }
  AttnParams p{};
  p.drop = drop;
  p.h0 = h0;
  p.nh_total = nh_total;
  p.B = B, p.T = T, p.nh = nh, p.Hs = nh * kD, p.out = out, p.ld_out = ld_out, p.lse = lse, p.Tpad = Tpad;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = status;
  p.exp_fma = attn_exp_fma();
  const CUtensorMap tm = qkv_map(qkv, B, T, ld_qkv, 3 * p.Hs);
  const int n_qt = (T + kTile - 1) / kTile;
  const int n_pairs = (n_qt + 1) / 2;
  p.trace = attn_trace_for((long)B * nh * n_pairs);
  // With dropout the O-in-TMEM form keeps the whole score row and the mask hashing
  // live at once and spills, so dropout runs the register-accumulator form.
  const bool drop_on = drop.thresh != 0;
  HB_ATTN_FWD_PICK(drop_on, f16, attn_fwd_ot() && !drop_on)<<<B * nh * n_pairs, FWD_THREADS, FWD_SMEM, s>>>(tm, p);
  HB_CUDA_CHECK(cudaGetLastError());
}

void attn_bwd_launch(const __nv_bfloat16* qkv, long ld_qkv, const __nv_bfloat16* o, long ld_o,
                     const __nv_bfloat16* dO, long ld_do, const float* lse, float* dvec, float* dq_acc,
                     __nv_bfloat16* dqkv, long ld_dqkv, int B, int T, int nh, int Tpad, float scale,
                     const DropoutArgs& drop, int h0, int nh_total, int* status, bool f16, cudaStream_t s) {
  static bool attr[64] = {};  // the shared-memory opt-in is per device
  const int dev = current_device();
  if (!attr[dev]) {
    for (int d = 0; d < 2; ++d)
      for (int h = 0; h < 2; ++h)
        HB_CUDA_CHECK(cudaFuncSetAttribute(HB_ATTN_PICK(attn_bwd_kernel, d, h),
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, BWD_SMEM));
    attr[dev] = true;
  }
  const int Hs = nh * kD;
  const long rows = (long)B * T;
  attn_bwd_prepass(o, ld_o, dO, ld_do, dvec, dq_acc, B, T, nh, kD, Tpad, scale, f16, s);
  AttnParams p{};
  p.B = B, p.T = T, p.nh = nh, p.Hs = Hs, p.out = dqkv, p.ld_out = ld_dqkv, p.lse = const_cast<float*>(lse);
  p.Tpad = Tpad, p.dvec = dvec, p.dq_acc = dq_acc;
  p.drop = drop;
  p.h0 = h0;
  p.nh_total = nh_total;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = status;
  p.trace = attn_trace_for((long)B * nh * ((T + kTile - 1) / kTile));
  const CUtensorMap tq = qkv_map(qkv, B, T, ld_qkv, 3 * Hs);
  const CUtensorMap td = qkv_map(dO, B, T, ld_do, Hs);
  // dQ accumulator as {Hs, T, B} fp32: 32x32 reduce boxes never cross into the next sequence.
  const uint64_t qdims[3] = {static_cast<uint64_t>(Hs), static_cast<uint64_t>(T), static_cast<uint64_t>(B)};
  const uint64_t qstr[2] = {static_cast<uint64_t>(Hs) * 4, static_cast<uint64_t>(Hs) * 4 * T};
  const uint32_t qbox[3] = {32, 32, 1};
  const CUtensorMap tdq =
      make_tmap(CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dq_acc, qdims, qstr, qbox, CU_TENSOR_MAP_SWIZZLE_128B);
  const int n_t = (T + kTile - 1) / kTile;
  HB_ATTN_PICK(attn_bwd_kernel, drop.thresh != 0, f16)<<<B * nh * n_t, BWD_THREADS, BWD_SMEM, s>>>(tq, td, tdq, p);
  HB_CUDA_CHECK(cudaGetLastError());
  attn_bwd_dq_finish(dq_acc, dqkv, ld_dqkv, rows, Hs, f16, s);
}

// Trace buffer for the next attention launches (nullptr turns tracing off).
// Forward slots per CTA: 0 start, 1 Q ready (MMA warp), 2 end; for KV tile j < 8
// and query tile g: 8+24g+j S ready, 16+24g+j softmax start (the previous PV is
// waited for inside, after the row max), 56+8g+j row max done, 24+24g+j P written.
// Backward slots per CTA: 0 start, 1 K/V and first Q/dO ready, 2 end; for query
// tile i < 8: 8+i / 16+i P^T half 0 / half 1 consumed by the MMA warp; for half g:
// 24+24g+i S^T/dP^T ready, 32+24g+i previous tile's MMAs done, 40+24g+i P^T/dS^T written.
void attn_set_trace(uint64_t* trace, long rows) {
  g_attn_trace = trace;
  g_attn_trace_rows = trace != nullptr ? rows : 0;
}

}  // namespace hb
