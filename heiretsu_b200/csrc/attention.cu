// Causal flash attention (head_dim 64) on tcgen05 tensor cores.
//
// Replaces F.scaled_dot_product_attention(q, k, v, is_causal=True)
// (reference gpt_model.py:74-81). Q, K and V are read in place from the QKV
// projection output qkv[B*T, 3*Hs] (columns [Q | K | V], each head-major,
// head h at h*64) through one 3-D TMA map {3*Hs, T, B}: a 128-token tile
// never crosses into the next sequence, and rows >= T read as zeros.
//
// Forward, one CTA per (query tile of 128, head, batch), 192 threads:
//   warp 0     TMA: Q once, then K0, K1, V0, K2, V1, ... into a 3-slot ring
//   warp 1     MMA: S = Q K^T (128x128, fp32 in TMEM); O_j = P_j V_j (128x64)
//   warps 2-5  softmax: thread = query row; two passes over S in TMEM (row
//              max, then exp2 + row sum), P -> bf16 in 128B-swizzled smem
//              (the A operand of the PV MMA), O accumulated in registers with
//              the online-softmax rescale, final O / l and LSE stored.
//   TMEM: S [0,128), O double buffer [128,192) [192,256). 96 KB smem, so two
//   CTAs share an SM and one's softmax overlaps the other's MMAs.
//
// Backward, one CTA per (key tile of 128, head, batch), FA2 order:
//   S^T = K Q_i^T and dP^T = V dO_i^T (thread = key row), P^T and
//   dS^T = P^T (dP^T - D) * scale to smem, then dV += P^T dO_i,
//   dK += dS^T Q_i and dQ_i = dS K (the same smem tiles serve as K-major or
//   MN-major operands), dQ_i added to an fp32 accumulator with vector atomics.
#include <cuda_bf16.h>

#include "common.cuh"
#include "host_utils.h"

namespace hb {

struct AttnParams {
  int B, T, nh, Hs;         // Hs = nh * 64 (this rank's heads)
  __nv_bfloat16* out;       // forward: y [B*T, ld_out]; backward: dqkv [B*T, ld_out]
  long ld_out;
  float* lse;               // [B, nh, Tpad] log2-domain LSE of the scaled scores
  int Tpad;
  const float* dvec;        // backward: D = rowsum(dO * O) [B, nh, Tpad]
  float* dq_acc;            // backward: fp32 dQ accumulator [B*T, Hs]
  float scale;              // 1/sqrt(64)
  float scale_log2;         // scale * log2(e)
  int* status;
};

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Byte offset of 16-byte chunk `c16` (0..15 over 128 bf16 columns) of row `r`
// in a K-major 128-byte-swizzled tile of 128 rows x 128 bf16 (two 16 KB atoms).
__device__ __forceinline__ uint32_t sw128_off(int r, int c16) {
  return (c16 >> 3) * 16384 + r * 128 + (((c16 & 7) ^ (r & 7)) << 4);
}

constexpr int kTile = 128;
constexpr int kD = 64;
constexpr int kTileBytes = kTile * kD * 2;  // 16 KB

// ============================================================================
// Forward
// ============================================================================
constexpr int FWD_SLOTS = 3;
constexpr int FWD_SMEM = kTileBytes /*Q*/ + FWD_SLOTS * kTileBytes + 2 * kTileBytes /*P*/ + 1024;

__global__ void __launch_bounds__(192) attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sSlot = smem + kTileBytes;
  uint8_t* sP = sSlot + FWD_SLOTS * kTileBytes;
  __shared__ uint64_t bar_q, bar_full[FWD_SLOTS], bar_empty[FWD_SLOTS], bar_s, bar_p, bar_o[2], bar_done;
  __shared__ uint32_t tmem_slot;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.T + kTile - 1) / kTile;
  int bid = blockIdx.x;
  const int qt = n_qt - 1 - (bid % n_qt);  // heaviest tiles first
  bid /= n_qt;
  const int h = bid % p.nh;
  const int b = bid / p.nh;
  const int n_kv = qt + 1;

  if (threadIdx.x == 0) {
    mbar_init(&bar_q, 1);
    for (int s = 0; s < FWD_SLOTS; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    mbar_init(&bar_s, 1);
    mbar_init(&bar_p, 4);
    mbar_init(&bar_o[0], 1);
    mbar_init(&bar_o[1], 1);
    mbar_init(&bar_done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tm_qkv);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t tS = tmem, tO0 = tmem + 128;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(&bar_q, kTileBytes);
      tma_load_3d(sQ, &tm_qkv, &bar_q, h * kD, qt * kTile, b);
      // Ring order = MMA consumption order: K0, then (K_{j+1}, V_j) for each j.
      int slot = 0;
      uint32_t phase = 0;
      auto load = [&](int kv, int is_v) -> bool {
        if (!mbar_wait(&bar_empty[slot], phase ^ 1u, p.status, 20)) return false;
        mbar_arrive_expect_tx(&bar_full[slot], kTileBytes);
        tma_load_3d(sSlot + slot * kTileBytes, &tm_qkv, &bar_full[slot], (is_v ? 2 : 1) * p.Hs + h * kD,
                    kv * kTile, b);
        if (++slot == FWD_SLOTS) {
          slot = 0;
          phase ^= 1u;
        }
        return true;
      };
      if (load(0, 0)) {
        for (int j = 0; j < n_kv; ++j) {
          if (j + 1 < n_kv && !load(j + 1, 0)) break;
          if (!load(j, 1)) break;
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = make_idesc_f16(128, 128, false, false, true);
      constexpr uint32_t idO = make_idesc_f16(128, 64, false, true, true);
      const uint32_t qa = smem_u32(sQ), pa = smem_u32(sP);
      int slot = 0;
      uint32_t phase = 0;
      bool ok = mbar_wait(&bar_q, 0, p.status, 21);
      auto take = [&](uint32_t& addr) -> bool {
        if (!mbar_wait(&bar_full[slot], phase, p.status, 22)) return false;
        tc_fence_after();
        addr = smem_u32(sSlot + slot * kTileBytes);
        return true;
      };
      auto release = [&]() {
        mma_commit(&bar_empty[slot]);
        if (++slot == FWD_SLOTS) {
          slot = 0;
          phase ^= 1u;
        }
      };
      uint32_t ka = 0, va = 0;
      if (ok && take(ka)) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_f16_ss(tS, sw128_desc(qa + k * 32, 16, 1024), sw128_desc(ka + k * 32, 16, 1024), idS, k > 0);
        release();
        mma_commit(&bar_s);
      } else {
        ok = false;
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        if (!mbar_wait(&bar_p, j & 1, p.status, 23)) break;
        tc_fence_after();
        if (j + 1 < n_kv) {
          if (!take(ka)) break;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f16_ss(tS, sw128_desc(qa + k * 32, 16, 1024), sw128_desc(ka + k * 32, 16, 1024), idS, k > 0);
          release();
          mma_commit(&bar_s);
        }
        if (!take(va)) break;
        const uint32_t tO = tO0 + (j & 1) * 64;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t ad = sw128_desc(pa + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
          const uint64_t bd = sw128_desc(va + ks * 2048, 8192, 1024);
          mma_f16_ss(tO, ad, bd, idO, ks > 0);
        }
        release();
        mma_commit(&bar_o[j & 1]);
      }
      mma_commit(&bar_done);
      mbar_wait(&bar_done, 0, p.status, 24);
    }
  } else {
    // Softmax / output warps: thread <-> query row.
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const int q = qt * kTile + row;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    float o[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) o[i] = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv && ok; ++j) {
      if (!mbar_wait(&bar_s, j & 1, p.status, 25)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool diag = (j == qt);
      float v[32];
      float mt = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(tS + lane_off + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = j * kTile + c * 32 + i;
          const float s = (diag && key > q) ? -INFINITY : v[i] * p.scale_log2;
          mt = fmaxf(mt, s);
        }
      }
      const float m_new = fmaxf(m, mt);
      const float alpha = (m == -INFINITY) ? 0.f : exp2f(m - m_new);
      // P smem is free once PV_{j-1} has completed.
      if (j > 0 && !mbar_wait(&bar_o[(j - 1) & 1], ((j - 1) >> 1) & 1, p.status, 26)) {
        ok = false;
        break;
      }
      float rs = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(tS + lane_off + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = j * kTile + c * 32 + i;
          const float pv = (diag && key > q) ? 0.f : exp2f(v[i] * p.scale_log2 - m_new);
          v[i] = pv;
          rs += pv;
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const uint4 pk = make_uint4(pack_bf16(v[g * 8 + 0], v[g * 8 + 1]), pack_bf16(v[g * 8 + 2], v[g * 8 + 3]),
                                      pack_bf16(v[g * 8 + 4], v[g * 8 + 5]), pack_bf16(v[g * 8 + 6], v[g * 8 + 7]));
          *reinterpret_cast<uint4*>(sP + sw128_off(row, c * 4 + g)) = pk;
        }
      }
      l = l * alpha + rs;
      m = m_new;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_p);
      if (j > 0) {
        const uint32_t tO = tO0 + ((j - 1) & 1) * 64;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tmem_ld32(tO + lane_off + c * 32, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c * 32 + i] = o[c * 32 + i] * alpha_prev + v[i];
        }
      }
      alpha_prev = alpha;
    }
    if (ok && mbar_wait(&bar_o[(n_kv - 1) & 1], ((n_kv - 1) >> 1) & 1, p.status, 27)) {
      tc_fence_after();
      const uint32_t tO = tO0 + ((n_kv - 1) & 1) * 64;
      float v[32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld32(tO + lane_off + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[c * 32 + i] = o[c * 32 + i] * alpha_prev + v[i];
      }
      if (q < p.T) {
        const float inv = 1.f / l;
        __nv_bfloat16* dst = p.out + ((long)b * p.T + q) * p.ld_out + h * kD;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          *reinterpret_cast<uint4*>(dst + g * 8) =
              make_uint4(pack_bf16(o[g * 8 + 0] * inv, o[g * 8 + 1] * inv), pack_bf16(o[g * 8 + 2] * inv, o[g * 8 + 3] * inv),
                         pack_bf16(o[g * 8 + 4] * inv, o[g * 8 + 5] * inv), pack_bf16(o[g * 8 + 6] * inv, o[g * 8 + 7] * inv));
        }
        p.lse[((long)b * p.nh + h) * p.Tpad + q] = m + log2f(l);
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ============================================================================
// Backward
// ============================================================================
constexpr int BWD_STAGE = 2 * kTileBytes + 1024;  // Q_i, dO_i, lse_i (512 B), D_i (512 B)
constexpr int BWD_STAGES = 2;
constexpr int BWD_SMEM = 2 * kTileBytes /*K,V*/ + BWD_STAGES * BWD_STAGE + 4 * kTileBytes /*P^T, dS^T*/ + 1024;

__global__ void __launch_bounds__(192) attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                                                       const __grid_constant__ CUtensorMap tm_do, AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + kTileBytes;
  uint8_t* sStage = smem + 2 * kTileBytes;
  uint8_t* sP = sStage + BWD_STAGES * BWD_STAGE;
  uint8_t* sDS = sP + 2 * kTileBytes;
  __shared__ uint64_t bar_kv, bar_full[BWD_STAGES], bar_empty[BWD_STAGES], bar_sdp, bar_p, bar_mma, bar_done;
  __shared__ uint32_t tmem_slot;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_t = (p.T + kTile - 1) / kTile;
  int bid = blockIdx.x;
  const int kt = bid % n_t;  // low key tiles have the most query tiles: launched first
  bid /= n_t;
  const int h = bid % p.nh;
  const int b = bid / p.nh;
  const int n_i = n_t - kt;  // query tiles kt .. n_t-1

  if (threadIdx.x == 0) {
    mbar_init(&bar_kv, 1);
    for (int s = 0; s < BWD_STAGES; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    mbar_init(&bar_sdp, 1);
    mbar_init(&bar_p, 4);
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
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 320, tDQ = tmem + 384;
  const long lse_base = ((long)b * p.nh + h) * p.Tpad;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(&bar_kv, 2 * kTileBytes);
      tma_load_3d(sK, &tm_qkv, &bar_kv, p.Hs + h * kD, kt * kTile, b);
      tma_load_3d(sV, &tm_qkv, &bar_kv, 2 * p.Hs + h * kD, kt * kTile, b);
      int st = 0;
      uint32_t phase = 0;
      for (int ii = 0; ii < n_i; ++ii) {
        const int qi = kt + ii;
        if (!mbar_wait(&bar_empty[st], phase ^ 1u, p.status, 40)) break;
        uint8_t* s = sStage + st * BWD_STAGE;
        mbar_arrive_expect_tx(&bar_full[st], 2 * kTileBytes + 1024);
        tma_load_3d(s, &tm_qkv, &bar_full[st], h * kD, qi * kTile, b);
        tma_load_3d(s + kTileBytes, &tm_do, &bar_full[st], h * kD, qi * kTile, b);
        bulk_load(s + 2 * kTileBytes, p.lse + lse_base + qi * kTile, 512, &bar_full[st]);
        bulk_load(s + 2 * kTileBytes + 512, p.dvec + lse_base + qi * kTile, 512, &bar_full[st]);
        if (++st == BWD_STAGES) {
          st = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idSS = make_idesc_f16(128, 128, false, false, true);  // S^T, dP^T
      constexpr uint32_t idKM = make_idesc_f16(128, 64, false, true, true);    // dV, dK
      constexpr uint32_t idQ = make_idesc_f16(128, 64, true, true, true);      // dQ
      const uint32_t ka = smem_u32(sK), va = smem_u32(sV), pa = smem_u32(sP), dsa = smem_u32(sDS);
      int st = 0;
      uint32_t phase = 0;
      bool ok = mbar_wait(&bar_kv, 0, p.status, 41);
      for (int ii = 0; ii < n_i && ok; ++ii) {
        if (!mbar_wait(&bar_full[st], phase, p.status, 42)) break;
        tc_fence_after();
        const uint32_t qa = smem_u32(sStage + st * BWD_STAGE);
        const uint32_t doa = qa + kTileBytes;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_f16_ss(tS, sw128_desc(ka + k * 32, 16, 1024), sw128_desc(qa + k * 32, 16, 1024), idSS, k > 0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_f16_ss(tDP, sw128_desc(va + k * 32, 16, 1024), sw128_desc(doa + k * 32, 16, 1024), idSS, k > 0);
        mma_commit(&bar_sdp);
        if (!mbar_wait(&bar_p, ii & 1, p.status, 43)) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t aoff = (ks >> 2) * 16384 + (ks & 3) * 32;
          // dV += P^T dO_i   (B = dO_i viewed MN-major: N = d, K = query)
          mma_f16_ss(tDV, sw128_desc(pa + aoff, 16, 1024), sw128_desc(doa + ks * 2048, 8192, 1024), idKM,
                     (ii > 0 || ks > 0));
          // dK += dS^T Q_i
          mma_f16_ss(tDK, sw128_desc(dsa + aoff, 16, 1024), sw128_desc(qa + ks * 2048, 8192, 1024), idKM,
                     (ii > 0 || ks > 0));
          // dQ_i = dS K   (A = dS^T viewed MN-major: M = query, K = key)
          mma_f16_ss(tDQ, sw128_desc(dsa + ks * 2048, 16384, 1024), sw128_desc(ka + ks * 2048, 8192, 1024), idQ,
                     ks > 0);
        }
        mma_commit(&bar_empty[st]);
        mma_commit(&bar_mma);
        if (++st == BWD_STAGES) {
          st = 0;
          phase ^= 1u;
        }
      }
      mma_commit(&bar_done);
      mbar_wait(&bar_done, 0, p.status, 44);
    }
  } else {
    const int sub = warp & 3;
    const int r = sub * 32 + lane;  // key row for S^T/dP^T/dK/dV, query row for dQ
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const int key = kt * kTile + r;
    int st = 0;
    uint32_t phase = 0;
    bool ok = true;
    auto flush_dq = [&](int qi) {
      // dQ_i (fp32, TMEM) -> global accumulator.
      tc_fence_after();
      const int qrow = qi * kTile + r;
      float v[32];
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        tmem_ld32(tDQ + lane_off + c * 32, v);
        if (qrow < p.T) {
          float4* dst = reinterpret_cast<float4*>(p.dq_acc + ((long)b * p.T + qrow) * p.Hs + h * kD + c * 32);
#pragma unroll
          for (int g = 0; g < 8; ++g) atomicAdd(dst + g, make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]));
        }
      }
    };
    for (int ii = 0; ii < n_i && ok; ++ii) {
      const int qi = kt + ii;
      if (!mbar_wait(&bar_full[st], phase, p.status, 45) || !mbar_wait(&bar_sdp, ii & 1, p.status, 46)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const float* s_lse = reinterpret_cast<const float*>(sStage + st * BWD_STAGE + 2 * kTileBytes);
      const float* s_d = s_lse + 128;
      // P^T / dS^T smem and the dQ TMEM columns are free once the MMAs of the
      // previous query tile are complete; flush that tile's dQ first.
      if (ii > 0) {
        if (!mbar_wait(&bar_mma, (ii - 1) & 1, p.status, 47)) {
          ok = false;
          break;
        }
        flush_dq(qi - 1);
      }
      const bool diag = (qi == kt);
      float sv[32], dp[32];
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(tS + lane_off + c * 32, sv);
        tmem_ld32(tDP + lane_off + c * 32, dp);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int qq = qi * kTile + c * 32 + i;
          const bool masked = (diag && key > qq) || qq >= p.T;
          const float pr = masked ? 0.f : exp2f(sv[i] * p.scale_log2 - s_lse[c * 32 + i]);
          sv[i] = pr;
          dp[i] = masked ? 0.f : pr * (dp[i] - s_d[c * 32 + i]) * p.scale;
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const uint32_t off = sw128_off(r, c * 4 + g);
          *reinterpret_cast<uint4*>(sP + off) =
              make_uint4(pack_bf16(sv[g * 8 + 0], sv[g * 8 + 1]), pack_bf16(sv[g * 8 + 2], sv[g * 8 + 3]),
                         pack_bf16(sv[g * 8 + 4], sv[g * 8 + 5]), pack_bf16(sv[g * 8 + 6], sv[g * 8 + 7]));
          *reinterpret_cast<uint4*>(sDS + off) =
              make_uint4(pack_bf16(dp[g * 8 + 0], dp[g * 8 + 1]), pack_bf16(dp[g * 8 + 2], dp[g * 8 + 3]),
                         pack_bf16(dp[g * 8 + 4], dp[g * 8 + 5]), pack_bf16(dp[g * 8 + 6], dp[g * 8 + 7]));
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_p);
      if (++st == BWD_STAGES) {
        st = 0;
        phase ^= 1u;
      }
    }
    if (ok && mbar_wait(&bar_mma, (n_i - 1) & 1, p.status, 48)) {
      flush_dq(kt + n_i - 1);
      // dK, dV -> bf16 into the K / V columns of dqkv (tcgen05.ld is
      // warp-collective, so every lane loads; only rows < T store).
      __nv_bfloat16* drow = p.out + ((long)b * p.T + key) * p.ld_out;
      float v[32];
#pragma unroll 1
      for (int which = 0; which < 2; ++which) {
        const uint32_t tsrc = which == 0 ? tDK : tDV;
        __nv_bfloat16* dst = drow + (which == 0 ? p.Hs : 2 * p.Hs) + h * kD;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          tmem_ld32(tsrc + lane_off + c * 32, v);
          if (key < p.T) {
#pragma unroll
            for (int g = 0; g < 4; ++g)
              *reinterpret_cast<uint4*>(dst + c * 32 + g * 8) =
                  make_uint4(pack_bf16(v[g * 8 + 0], v[g * 8 + 1]), pack_bf16(v[g * 8 + 2], v[g * 8 + 3]),
                             pack_bf16(v[g * 8 + 4], v[g * 8 + 5]), pack_bf16(v[g * 8 + 6], v[g * 8 + 7]));
          }
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// D[b, h, t] = sum_d dO[b*T+t, h*64+d] * O[b*T+t, h*64+d]   (fp32)
__global__ void attn_bwd_dvec_kernel(const __nv_bfloat16* __restrict__ o, long ld_o, const __nv_bfloat16* __restrict__ dO,
                                     long ld_do, float* __restrict__ dvec, int B, int T, int nh, int Tpad) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)B * T * nh) return;
  const int h = i % nh;
  const long row = i / nh;
  const int b = row / T, t = row % T;
  const uint4* a = reinterpret_cast<const uint4*>(o + row * ld_o + h * kD);
  const uint4* g = reinterpret_cast<const uint4*>(dO + row * ld_do + h * kD);
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint4 x = a[k], y = g[k];
    const __nv_bfloat16* xe = reinterpret_cast<const __nv_bfloat16*>(&x);
    const __nv_bfloat16* ye = reinterpret_cast<const __nv_bfloat16*>(&y);
#pragma unroll
    for (int q = 0; q < 8; ++q) s += __bfloat162float(xe[q]) * __bfloat162float(ye[q]);
  }
  dvec[((long)b * nh + h) * Tpad + t] = s;
}

// dqkv[:, h*64 + d] = bf16(dq_acc)
__global__ void attn_bwd_dq_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dqkv, long ld,
                                   long rows, int Hs) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long n4 = rows * Hs / 4;
  if (i >= n4) return;
  const long e = i * 4;
  const long row = e / Hs;
  const int c = e % Hs;
  const float4 v = reinterpret_cast<const float4*>(dq_acc)[i];
  *reinterpret_cast<uint2*>(dqkv + row * ld + c) = make_uint2(pack_bf16(v.x, v.y), pack_bf16(v.z, v.w));
}

// ----------------------------------------------------------------------------
static CUtensorMap qkv_map(const void* base, int B, int T, long ld, int cols) {
  const uint64_t dims[3] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(T), static_cast<uint64_t>(B)};
  const uint64_t strides[2] = {static_cast<uint64_t>(ld) * 2, static_cast<uint64_t>(ld) * 2 * T};
  const uint32_t box[3] = {64, 128, 1};
  return make_tmap_bf16(3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

void attn_fwd_launch(const __nv_bfloat16* qkv, long ld_qkv, __nv_bfloat16* out, long ld_out, float* lse, int B,
                     int T, int nh, int Tpad, int* status, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    HB_CUDA_CHECK(cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FWD_SMEM));
    attr = true;
  }
  AttnParams p{};
  p.B = B, p.T = T, p.nh = nh, p.Hs = nh * kD, p.out = out, p.ld_out = ld_out, p.lse = lse, p.Tpad = Tpad;
  p.scale = 0.125f;
  p.scale_log2 = 0.125f * 1.4426950408889634f;
  p.status = status;
  const CUtensorMap tm = qkv_map(qkv, B, T, ld_qkv, 3 * p.Hs);
  const int n_qt = (T + kTile - 1) / kTile;
  attn_fwd_kernel<<<B * nh * n_qt, 192, FWD_SMEM, s>>>(tm, p);
  HB_CUDA_CHECK(cudaGetLastError());
}

void attn_bwd_launch(const __nv_bfloat16* qkv, long ld_qkv, const __nv_bfloat16* o, long ld_o,
                     const __nv_bfloat16* dO, long ld_do, const float* lse, float* dvec, float* dq_acc,
                     __nv_bfloat16* dqkv, long ld_dqkv, int B, int T, int nh, int Tpad, int* status, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    HB_CUDA_CHECK(cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BWD_SMEM));
    attr = true;
  }
  const int Hs = nh * kD;
  const long rows = (long)B * T;
  attn_bwd_dvec_kernel<<<(rows * nh + 255) / 256, 256, 0, s>>>(o, ld_o, dO, ld_do, dvec, B, T, nh, Tpad);
  HB_CUDA_CHECK(cudaGetLastError());
  HB_CUDA_CHECK(cudaMemsetAsync(dq_acc, 0, sizeof(float) * rows * Hs, s));
  AttnParams p{};
  p.B = B, p.T = T, p.nh = nh, p.Hs = Hs, p.out = dqkv, p.ld_out = ld_dqkv, p.lse = const_cast<float*>(lse);
  p.Tpad = Tpad, p.dvec = dvec, p.dq_acc = dq_acc;
  p.scale = 0.125f;
  p.scale_log2 = 0.125f * 1.4426950408889634f;
  p.status = status;
  const CUtensorMap tq = qkv_map(qkv, B, T, ld_qkv, 3 * Hs);
  const CUtensorMap td = qkv_map(dO, B, T, ld_do, Hs);
  const int n_t = (T + kTile - 1) / kTile;
  attn_bwd_kernel<<<B * nh * n_t, 192, BWD_SMEM, s>>>(tq, td, p);
  HB_CUDA_CHECK(cudaGetLastError());
  attn_bwd_dq_kernel<<<(rows * Hs / 4 + 255) / 256, 256, 0, s>>>(dq_acc, dqkv, ld_dqkv, rows, Hs);
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
