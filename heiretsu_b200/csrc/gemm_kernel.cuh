#pragma once
// tcgen05 GEMM core for sm_100a.
//
// D[m, n] = sum_k A(m, k) * B(n, k), 16-bit operands (bf16 or fp16, one format
// per launch), fp32 accumulation in tensor memory, fused epilogues. This single kernel template serves every
// linear layer of the model (reference: tp_linear.py:148, :224, :301 einsums;
// moe.py:45, :90-92 nn.Linear; gpt_model.py:240 lm_head):
//   forward  y = x W^T        A = x  [M,K] K-major,  B = W [N,K] K-major
//   dgrad    dx = dy W        A = dy [M,N] K-major,  B = W stored [N,K] -> MN-major
//   wgrad    dW = dy^T x      A = dy stored [M,N] -> MN-major, B = x stored [M,K] -> MN-major
// so no transposed copy of any activation or weight is ever materialised.
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: streams 128xBK A tiles and BNxBK B tiles into a
//               STAGES-deep shared-memory ring (128-byte swizzle, no multicast).
//   warp 1      allocates TMEM; one elected thread issues tcgen05.mma
//               (128 x BN x 16) and commits each stage back to the producer.
//   warps 2..9  epilogue: tcgen05.ld the fp32 accumulator (thread = row),
//               apply bias / GELU / dGELU / residual (+ dropout), store through
//               TMA (or into a peer's receive slot for the TP reduce-scatter, and
//               into every EP rank's combine slot for the expert-parallel combine).
//               With an all-gather prologue they first pull peers' token shards.
//               Two warps share each TMEM lane quarter and split the tile's
//               columns, so eight warps drain a tile while the next one
//               accumulates.
// The accumulator is double-buffered in TMEM (2 x BN columns) so the
// epilogue of tile i overlaps the main loop of tile i+1.
#include "common.cuh"
#include "host_utils.h"
#include "gemm_params.h"
#include "dropout.cuh"

namespace hb {

constexpr int kEpiWarps = 8;
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
constexpr int kStgBytes = 32 * 128;  // per epilogue warp: 32 rows x 128 bytes, XOR-swizzled

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (BN >= 192) ? 4 : 6;
  // two accumulators of BN columns; TMEM is allocated in powers of two
  static constexpr int TMEM_COLS = (2 * BN <= 256) ? 256 : 512;
  static constexpr int STG_OFFSET = STAGES * STAGE_BYTES;  // per-warp epilogue staging tiles
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + kEpiWarps * kStgBytes + 1024 /*align*/ + 256 /*barriers*/;
};

// ---------------------------------------------------------------------------
// Epilogue. Each epilogue warp owns 32 accumulator rows (its TMEM lane
// quarter) and processes 32 columns at a time: thread t holds row t's 32
// values after tcgen05.ld. Global traffic goes through a per-warp staging
// tile in shared memory, so every global load/store is coalesced (lanes
// cover consecutive 16-byte segments of a row) while the arithmetic stays
// row-per-thread. The staging tile is XOR-swizzled on 16-byte segments
// (fp32 rows of 128 B: seg ^ (row & 7); bf16 rows of 64 B: seg ^ ((row >> 1) & 3)),
// which makes both access patterns bank-conflict free without padding.
// Operands the epilogue reads (residual, GELU pre-activation, accumulated
// gradient) are fetched into registers one chunk ahead -- the first chunk
// before the accumulator is even ready -- so DRAM latency overlaps the MMAs.
// ---------------------------------------------------------------------------
template <bool F32>
__device__ __forceinline__ int stg_off(int r, int seg) {
  return F32 ? r * 128 + ((seg ^ (r & 7)) << 4) : r * 64 + ((seg ^ ((r >> 1) & 3)) << 4);
}

// Coalesced global loads of a [32 rows][32 cols] tile into registers (zeros outside M x N).
template <bool F32>
__device__ __forceinline__ void gload_tile(uint4 (&pre)[8], const void* src, long ld, int m_base, int n0, int M, int N,
                                           int lane) {
  constexpr int SEGS = F32 ? 8 : 4;  // 16-byte segments per row
  constexpr int ESZ = F32 ? 4 : 2;
#pragma unroll
  for (int it = 0; it < SEGS; ++it) {
    const int idx = it * 32 + lane;
    const int r = idx / SEGS, seg = idx % SEGS;
    const int gm = m_base + r, gn = n0 + seg * (16 / ESZ);
    pre[it] = make_uint4(0, 0, 0, 0);
    if (gm < M && gn < N)
      pre[it] = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(src) + ((long)gm * ld + gn) * ESZ));
  }
}

template <bool F32>
__device__ __forceinline__ void stg_fill(uint8_t* stg, const uint4 (&pre)[8], int lane) {
  constexpr int SEGS = F32 ? 8 : 4;
#pragma unroll
  for (int it = 0; it < SEGS; ++it) {
    const int idx = it * 32 + lane;
    *reinterpret_cast<uint4*>(stg + stg_off<F32>(idx / SEGS, idx % SEGS)) = pre[it];
  }
}

// Coalesced copy staging -> global (all shared loads first, then the stores).
template <bool F32>
__device__ __forceinline__ void stg_store(const uint8_t* stg, void* dst, long ld, int m_base, int n0, int M, int N,
                                          int lane) {
  constexpr int SEGS = F32 ? 8 : 4;
  constexpr int ESZ = F32 ? 4 : 2;
  uint4 val[SEGS];
#pragma unroll
  for (int it = 0; it < SEGS; ++it) {
    const int idx = it * 32 + lane;
    val[it] = *reinterpret_cast<const uint4*>(stg + stg_off<F32>(idx / SEGS, idx % SEGS));
  }
#pragma unroll
  for (int it = 0; it < SEGS; ++it) {
    const int idx = it * 32 + lane;
    const int r = idx / SEGS, seg = idx % SEGS;
    const int gm = m_base + r, gn = n0 + seg * (16 / ESZ);
    if (gm < M && gn < N)
      *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(dst) + ((long)gm * ld + gn) * ESZ) = val[it];
  }
}

// Coalesced staging -> global vector atomic add (fp32 split-K partials).
__device__ __forceinline__ void stg_atomic_add(const uint8_t* stg, float* dst, long ld, int m_base, int n0, int M,
                                               int N, int lane) {
  float4 val[8];
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int idx = it * 32 + lane;
    val[it] = *reinterpret_cast<const float4*>(stg + stg_off<true>(idx / 8, idx % 8));
  }
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int idx = it * 32 + lane;
    const int r = idx / 8, seg = idx % 8;
    const int gm = m_base + r, gn = n0 + seg * 4;
    if (gm < M && gn < N) atomicAdd(reinterpret_cast<float4*>(dst + (long)gm * ld + gn), val[it]);
  }
}

// Row-per-thread write of 32 values into this thread's staging row.
template <bool F16>
__device__ __forceinline__ void stg_put16(uint8_t* stg, int lane, const float (&v)[32]) {
#pragma unroll
  for (int g = 0; g < 4; ++g)
    *reinterpret_cast<uint4*>(stg + stg_off<false>(lane, g)) =
        make_uint4(pack16<F16>(v[8 * g], v[8 * g + 1]), pack16<F16>(v[8 * g + 2], v[8 * g + 3]),
                   pack16<F16>(v[8 * g + 4], v[8 * g + 5]), pack16<F16>(v[8 * g + 6], v[8 * g + 7]));
}
__device__ __forceinline__ void stg_put_bf16(uint8_t* stg, int lane, const float (&v)[32], bool f16) {
  if (f16) {
    stg_put16<true>(stg, lane, v);
  } else {
    stg_put16<false>(stg, lane, v);
  }
}

// GELU epilogue core: pk <- the 16-bit pre-activation pairs; v <- GELU of those
// rounded values (so backward differentiates exactly what forward applied).
template <bool F16>
__device__ __forceinline__ void gelu_chunk16(float (&v)[32], uint32_t (&pk)[16], int mode) {
#pragma unroll
  for (int j = 0; j < 16; ++j) pk[j] = pack16<F16>(v[2 * j], v[2 * j + 1]);
  if (mode == 2) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      v[2 * j] = gelu_tanh_mufu(lo16<F16>(pk[j]));
      v[2 * j + 1] = gelu_tanh_mufu(hi16<F16>(pk[j]));
    }
  } else if (mode == 1) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {  // half the exponentials on the transcendental unit, half on the FMA pipe
      v[2 * j] = gelu_tanh(lo16<F16>(pk[j]));
      v[2 * j + 1] = gelu_tanh_fma(hi16<F16>(pk[j]));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      v[2 * j] = gelu_tanh(lo16<F16>(pk[j]));
      v[2 * j + 1] = gelu_tanh(hi16<F16>(pk[j]));
    }
  }
}
__device__ __forceinline__ void gelu_chunk(float (&v)[32], uint32_t (&pk)[16], bool f16, int mode) {
  if (f16) {
    gelu_chunk16<true>(v, pk, mode);
  } else {
    gelu_chunk16<false>(v, pk, mode);
  }
}

// v[i] *= GELU'(16-bit pre-activation of column i), eight columns from one 16-byte word.
template <bool F16>
__device__ __forceinline__ void dgelu8(float* v, const uint4 raw, int mode) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  if (mode == 2) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      v[2 * q] *= gelu_tanh_grad_mufu(lo16<F16>(w[q]));
      v[2 * q + 1] *= gelu_tanh_grad_mufu(hi16<F16>(w[q]));
    }
  } else if (mode == 1) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      v[2 * q] *= gelu_tanh_grad(lo16<F16>(w[q]));
      v[2 * q + 1] *= gelu_tanh_grad_fma(hi16<F16>(w[q]));
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      v[2 * q] *= gelu_tanh_grad(lo16<F16>(w[q]));
      v[2 * q + 1] *= gelu_tanh_grad(hi16<F16>(w[q]));
    }
  }
}
__device__ __forceinline__ void stg_put_f32(uint8_t* stg, int lane, const float (&v)[32]) {
#pragma unroll
  for (int g = 0; g < 8; ++g)
    *reinterpret_cast<float4*>(stg + stg_off<true>(lane, g)) =
        make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
}

template <int EPI>
constexpr bool epi_reads_operand() {
  return EPI == kEpiF32Resid || EPI == kEpiF32Acc || EPI == kEpiBf16Dgelu;
}

// Fetch the operand tile this epilogue chunk reads (if any) into registers.
template <int EPI>
__device__ __forceinline__ void epi_prefetch(const GemmParams& p, const void* C, int m_base, int n0, int lane,
                                             uint4 (&pre)[8]) {
  if constexpr (EPI == kEpiF32Resid) {
    gload_tile<true>(pre, p.resid, p.ldr, m_base, n0, p.M, p.N, lane);
  } else if constexpr (EPI == kEpiF32Acc) {
    gload_tile<true>(pre, C, p.ldc, m_base, n0, p.M, p.N, lane);
  } else if constexpr (EPI == kEpiBf16Dgelu) {
    gload_tile<false>(pre, p.aux, p.ldaux, m_base, n0, p.M, p.N, lane);
  }
}

// Step 1: combine the prefetched operand with the accumulator row (frees `pre`).
template <int EPI>
__device__ __forceinline__ void epi_apply_operand(float (&v)[32], uint8_t* stg, const uint4 (&pre)[8], int lane,
                                                  bool f16, int gelu_mode) {
  if constexpr (EPI == kEpiF32Resid || EPI == kEpiF32Acc) {
    stg_fill<true>(stg, pre, lane);
    __syncwarp();
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const float4 r = *reinterpret_cast<const float4*>(stg + stg_off<true>(lane, g));
      v[4 * g] += r.x;
      v[4 * g + 1] += r.y;
      v[4 * g + 2] += r.z;
      v[4 * g + 3] += r.w;
    }
    __syncwarp();
  }
  if constexpr (EPI == kEpiBf16Dgelu) {
    stg_fill<false>(stg, pre, lane);
    __syncwarp();
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const uint4 raw = *reinterpret_cast<const uint4*>(stg + stg_off<false>(lane, g));
      if (f16) {
        dgelu8<true>(v + 8 * g, raw, gelu_mode);
      } else {
        dgelu8<false>(v + 8 * g, raw, gelu_mode);
      }
    }
    __syncwarp();
  }
}

// Expert-parallel combine: this thread's output row, scaled by its routing
// weight, pushed into slot k, row t of every EP rank's receive buffer. The row
// is first rounded to the 16-bit output format (the value C holds), so a slot
// holds round16(w * round16(acc)): the term the one-GPU combine adds.
__device__ __forceinline__ void epi_combine_push(const GemmParams& p, int row, int n0, const float (&v)[32]) {
  if (row >= p.M) return;
  const int inv = p.cmb_inv[row];
  if (inv < 0) return;  // padding row of an expert segment
  const float w = p.cmb_w[inv];
  const int t = inv / p.cmb_K, k = inv - t * p.cmb_K;
  uint32_t pk[16];
  if (p.f16) {
#pragma unroll
    for (int j = 0; j < 16; ++j) pk[j] = pack16<true>(w * round16<true>(v[2 * j]), w * round16<true>(v[2 * j + 1]));
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      pk[j] = pack16<false>(w * round16<false>(v[2 * j]), w * round16<false>(v[2 * j + 1]));
  }
  const long off = (((long)k * p.cmb_N + t) * p.N + n0) * 2;  // bytes
#pragma unroll 1
  for (int r = 0; r < p.cmb_world; ++r) {
    uint4* d = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.cmb_dst[r]) + off);
#pragma unroll
    for (int q = 0; q < 4; ++q) d[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
  }
}

// Residual dropout of one 32-column chunk of this thread's row:
// v = mask * (v + bias), mask from the counter-based hash of the element index.
__device__ __forceinline__ void epi_bias_dropout(const GemmParams& p, uint32_t key, int row, int n0, float (&v)[32]) {
  if (p.bias != nullptr) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      if (n0 + j < p.N) {
        const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + n0 + j));
        v[j] += b.x;
        v[j + 1] += b.y;
        v[j + 2] += b.z;
        v[j + 3] += b.w;
      }
    }
  }
  const uint64_t pair0 = ((uint64_t)(p.drop.row0 + row) * (uint64_t)p.N + (uint64_t)n0) >> 1;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    float m0, m1;
    dropout_pair(dropout_bits(key, pair0 + j), p.drop.thresh, p.drop.scale, m0, m1);
    v[2 * j] *= m0;
    v[2 * j + 1] *= m1;
  }
}

// Step 2: bias, activation and the stores of one 32x32 chunk into C.
template <int EPI>
__device__ __forceinline__ void epi_finish(const GemmParams& p, void* C, int m_base, int n0, float (&v)[32],
                                           uint8_t* stg, int lane, bool bias_done = false) {
  if (!bias_done && p.bias != nullptr &&
      (EPI == kEpiBf16 || EPI == kEpiBf16Gelu || EPI == kEpiF32 || EPI == kEpiF32Resid)) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      if (n0 + j < p.N) {
        const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + n0 + j));
        v[j] += b.x;
        v[j + 1] += b.y;
        v[j + 2] += b.z;
        v[j + 3] += b.w;
      }
    }
  }
  if constexpr (EPI == kEpiBf16Gelu) {
    // Pre-activation (rounded to the 16-bit format) goes to AUX; GELU of that
    // rounded value goes to C, so backward differentiates exactly what forward applied.
    uint32_t pk[16];
    gelu_chunk(v, pk, p.f16 != 0, p.gelu_mode);
#pragma unroll
    for (int g = 0; g < 4; ++g)
      *reinterpret_cast<uint4*>(stg + stg_off<false>(lane, g)) =
          make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
    __syncwarp();
    stg_store<false>(stg, p.aux, p.ldaux, m_base, n0, p.M, p.N, lane);
    __syncwarp();
  }
  if constexpr (EPI == kEpiBf16 || EPI == kEpiBf16Gelu || EPI == kEpiBf16Dgelu) {
    stg_put_bf16(stg, lane, v, p.f16 != 0);
    __syncwarp();
    stg_store<false>(stg, C, p.ldc, m_base, n0, p.M, p.N, lane);
  } else if constexpr (EPI == kEpiF32Atomic) {
    stg_put_f32(stg, lane, v);
    __syncwarp();
    stg_atomic_add(stg, reinterpret_cast<float*>(C), p.ldc, m_base, n0, p.M, p.N, lane);
  } else {
    stg_put_f32(stg, lane, v);
    __syncwarp();
    stg_store<true>(stg, C, p.ldc, m_base, n0, p.M, p.N, lane);
  }
  __syncwarp();
}

// Step 2, TMA form: bias / activation, stage the chunk, one lane issues the
// bulk store (or reduce-add). `row` is the chunk's first row in the C map.
// The caller has waited for the previous bulk copies to finish reading `stg`.
template <int EPI>
__device__ __forceinline__ void epi_finish_tma(const GemmParams& p, const CUtensorMap* tmC, const CUtensorMap* tmX,
                                               int row, int n0, float (&v)[32], uint8_t* stg, int lane,
                                               bool bias_done = false) {
  if (!bias_done && p.bias != nullptr &&
      (EPI == kEpiBf16 || EPI == kEpiBf16Gelu || EPI == kEpiF32 || EPI == kEpiF32Resid)) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      if (n0 + j < p.N) {
        const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + n0 + j));
        v[j] += b.x;
        v[j + 1] += b.y;
        v[j + 2] += b.z;
        v[j + 3] += b.w;
      }
    }
  }
  if constexpr (EPI == kEpiBf16Gelu) {
    // pre-activation (16-bit) -> first 2 KB of the staging tile; GELU of the
    // rounded value -> second 2 KB; two stores.
    uint32_t pk[16];
    gelu_chunk(v, pk, p.f16 != 0, p.gelu_mode);
#pragma unroll
    for (int g = 0; g < 4; ++g)
      *reinterpret_cast<uint4*>(stg + stg_off<false>(lane, g)) =
          make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
    stg_put_bf16(stg + 2048, lane, v, p.f16 != 0);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmX, stg, n0, row);
      tma_store_2d(tmC, stg + 2048, n0, row);
      bulk_commit_group();
    }
  } else if constexpr (EPI == kEpiBf16 || EPI == kEpiBf16Dgelu) {
    stg_put_bf16(stg, lane, v, p.f16 != 0);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmC, stg, n0, row);
      bulk_commit_group();
    }
  } else {
    stg_put_f32(stg, lane, v);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if constexpr (EPI == kEpiF32Acc || EPI == kEpiF32Atomic) {
        tma_reduce_add_2d(tmC, stg, n0, row);  // C += chunk, added in L2
      } else {
        tma_store_2d(tmC, stg, n0, row);
      }
      bulk_commit_group();
    }
  }
}

// ---------------------------------------------------------------------------
// All-gather prologue helpers
// ---------------------------------------------------------------------------
constexpr int kAgUnitRows = 16;

__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// One warp copies 16-row units of the peers' shards (NVLink loads) into the
// local gathered matrix, then publishes them on the m-block's counter.
__device__ __forceinline__ void ag_copy_units(const GemmParams& p, int gw, int nw, int lane) {
  const int units_per_rank = p.ag_rows / kAgUnitRows;
  const int total = units_per_rank * p.ag_world;
  const long row_bytes = (long)p.K * 2;
  const long unit_vecs = kAgUnitRows * row_bytes / 16;
  for (int u = gw; u < total; u += nw) {
    const int src = (p.ag_rank + u / units_per_rank) % p.ag_world;
    const int lu = u % units_per_rank;
    const uint4* from = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.ag_src[src]) +
                                                       (long)lu * kAgUnitRows * row_bytes);
    uint4* to = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.ag_dst) +
                                         ((long)src * p.ag_rows + (long)lu * kAgUnitRows) * row_bytes);
    long i = lane;
    for (; i + 96 < unit_vecs; i += 128) {
      const uint4 a = from[i], b = from[i + 32], c = from[i + 64], d = from[i + 96];
      to[i] = a;
      to[i + 32] = b;
      to[i + 64] = c;
      to[i + 96] = d;
    }
    for (; i < unit_vecs; i += 32) to[i] = from[i];
    __syncwarp();
    __threadfence();
    if (lane == 0) red_release_gpu_add(p.ag_flags + (src * p.ag_rows + lu * kAgUnitRows) / 128, 1);
  }
}

// Producer side: wait (bounded) until all units of m-block mb are gathered,
// then order those generic-proxy writes before this thread's TMA reads.
__device__ __forceinline__ bool ag_wait_rows(const GemmParams& p, int mb) {
  const int need = 128 / kAgUnitRows;
  const int* f = p.ag_flags + mb;
  if (ld_acquire_gpu(f) < need) {
    const uint64_t t0 = globaltimer_ns();
    int spins = 0;
    while (ld_acquire_gpu(f) < need) {
      if (((++spins) & 255) == 0 && globaltimer_ns() - t0 > HB_WAIT_TIMEOUT_NS) {
        record_error(p.status, kPeerTimeout, 6);
        return false;
      }
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmX, GemmParams p) {
  using Cfg = GemmCfg<BN>;
  constexpr int BM = Cfg::BM, BK = Cfg::BK, STAGES = Cfg::STAGES;
  constexpr int A_BYTES = Cfg::A_BYTES, STAGE_BYTES = Cfg::STAGE_BYTES;
  constexpr uint32_t TMEM_COLS = Cfg::TMEM_COLS;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::STG_OFFSET + kEpiWarps * kStgBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* mma_done = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Row-grouped GEMMs learn their row count from the device (padded expert segments).
  const int num_m = (p.grp_mode == 1) ? p.grp_off[p.grp_n] / BM : (p.M + BM - 1) / BM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n * p.splits * (p.grp_mode == 2 ? p.grp_n : 1);
  const int num_kb_total = (p.K + BK - 1) / BK;
  // Tile t -> (group/split, m-block, n-block) and its k-block range.
  auto decode = [&](int t, int& mb, int& nb, int& kb0, int& nkb, int& grp) {
    const int mn = num_m * num_n;
    const int sp = t / mn;
    const int r = t % mn;
    if (p.raster_n) {
      mb = r / num_n, nb = r % num_n;
    } else {
      mb = r % num_m, nb = r / num_m;
    }
    if (p.ag_world > 1) mb = (mb + p.ag_rank * (p.ag_rows / BM)) % num_m;  // local shard first, then ring order
    grp = 0;
    if (p.grp_mode == 2) {
      grp = sp;
      kb0 = p.grp_off[grp] / BK;
      nkb = (p.grp_off[grp + 1] - p.grp_off[grp]) / BK;
      return;
    }
    if (p.grp_mode == 1) {
      const int row = mb * BM;
      while (grp + 1 < p.grp_n && p.grp_off[grp + 1] <= row) ++grp;
    }
    kb0 = sp * p.kb_per_split;
    nkb = min(p.kb_per_split, num_kb_total - kb0);
  };

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);
    }
    mbar_init(mma_done, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb, kb0, num_kb, grp;
        decode(t, mb, nb, kb0, num_kb, grp);
        const int b_grp_off = (p.grp_mode == 1) ? grp * p.grp_b_off : 0;
        if (p.ag_world > 1 && !ag_wait_rows(p, mb)) {
          ok = false;
          break;
        }
        for (int kbi = 0; kbi < num_kb; ++kbi) {
          const int kb = kb0 + kbi;
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          uint8_t* sA = smem + stage * STAGE_BYTES;
          uint8_t* sB = sA + A_BYTES;
          if constexpr (!A_MN) {
            tma_load_2d(sA, &tmA, &full[stage], kb * BK, mb * BM);
          } else {
#pragma unroll
            for (int a = 0; a < BM / 64; ++a) tma_load_2d(sA + a * 8192, &tmA, &full[stage], mb * BM + a * 64, kb * BK);
          }
          if constexpr (!B_MN) {
            tma_load_2d(sB, &tmB, &full[stage], kb * BK, nb * BN + b_grp_off);
          } else {
#pragma unroll
            for (int a = 0; a < BN / 64; ++a)
              tma_load_2d(sB + a * 8192, &tmB, &full[stage], nb * BN + a * 64, kb * BK + b_grp_off);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Never leave the CTA with TMA writes into shared memory in flight:
      // wait (bounded) for the last load issued into every stage.
      if (!ok) {
        for (int s = 0; s < STAGES; ++s) {
          const int back = (stage - 1 - s + 2 * STAGES) % STAGES;
          const uint32_t ph = (back < stage) ? phase : (phase ^ 1u);
          mbar_wait(&full[back], ph, nullptr, 0);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      const uint32_t idesc = make_idesc_f16(BM, BN, A_MN, B_MN, p.f16 == 0);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.status, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        int mb_, nb_, kb0_, num_kb, grp_;
        decode(t, mb_, nb_, kb0_, num_kb, grp_);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? sw128_desc(a_addr + k * 2048, 8192, 1024) : sw128_desc(a_addr + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sw128_desc(b_addr + k * 2048, 8192, 1024) : sw128_desc(b_addr + k * 32, 16, 1024);
            mma_f16_ss(d_tmem, ad, bd, idesc, (kb | k) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        mma_commit(&tfull[acc]);
      }
      // All MMAs issued by this thread must be complete before TMEM is freed.
      mma_commit(mma_done);
      mbar_wait(mma_done, 0, p.status, 5);
    }
  } else {
    const int eid = warp - 2;       // 0 .. kEpiWarps-1
    const int quarter = warp & 3;   // TMEM lanes this warp may access: 32 * (warp % 4) ..
    constexpr int CH = BN / 64;     // 32-column chunks per warp (the two warps of a quarter split the tile)
    const int c0 = (eid >> 2) * CH;
    uint8_t* stg = smem + Cfg::STG_OFFSET + eid * kStgBytes;
    if (p.ag_world > 1) ag_copy_units(p, blockIdx.x * kEpiWarps + eid, gridDim.x * kEpiWarps, lane);
    uint32_t drop_key = 0;
    if (EPI == kEpiF32Resid && p.drop.thresh != 0) drop_key = dropout_key(*p.drop.seed, p.drop.site);
    int local = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      int mb, nb, kb0_, nkb_, grp;
      decode(t, mb, nb, kb0_, nkb_, grp);
      const int m_base = mb * BM + quarter * 32;
      void* C = p.C;
      if (p.grp_mode == 2) {
        // this expert's block of the stacked weight gradient
        C = static_cast<uint8_t*>(p.C) + (long)grp * p.grp_c_off * p.ldc * 4;
      } else if (p.rs_world > 1) {
        // partial tile -> slot rs_rank of the owning rank's receive buffer (over NVLink)
        const int owner = m_base / p.rs_rows;
        const int esz = (EPI == kEpiBf16) ? 2 : 4;
        C = static_cast<uint8_t*>(p.rs_dst[owner]) +
            ((long)p.rs_rank * p.rs_rows - (long)owner * p.rs_rows) * p.ldc * esz;
      }
      const bool tma = p.tma_epi != 0;
      const int row = (p.grp_mode == 2 ? grp * p.grp_c_off : 0) + m_base;  // chunk row in the C map
      // With TMA the accumulating epilogue is a reduce-add in L2: no operand read.
      const bool reads = epi_reads_operand<EPI>() && !(tma && EPI == kEpiF32Acc);
      uint4 pre[8];
      const int n_first = nb * BN + c0 * 32;
      if (reads && nkb_ > 0 && n_first < p.N) epi_prefetch<EPI>(p, C, m_base, n_first, lane, pre);
      if (!mbar_wait(&tfull[acc], acc_phase, p.status, 4)) break;
      tc_fence_after();
      if (nkb_ > 0) {  // an empty expert segment accumulated nothing and stores nothing
#pragma unroll 1
        for (int c = 0; c < CH; ++c) {
          const int n0 = n_first + c * 32;
          if (n0 >= p.N) break;
          float v[32];
          tmem_ld32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN + (c0 + c) * 32, v);
          if (tma) {  // the staging tile is reused: the previous bulk copies must have read it
            if (lane == 0) bulk_wait_group_read0();
            __syncwarp();
          }
          bool bias_done = false;
          if constexpr (EPI == kEpiF32Resid) {
            if (p.drop.thresh != 0) {  // C = R + dropout(acc + bias)
              epi_bias_dropout(p, drop_key, m_base + lane, n0, v);
              bias_done = true;
            }
          }
          if (reads) epi_apply_operand<EPI>(v, stg, pre, lane, p.f16 != 0, p.gelu_mode);
          if (reads && c + 1 < CH && n0 + 32 < p.N) epi_prefetch<EPI>(p, C, m_base, n0 + 32, lane, pre);
          if (tma) {
            epi_finish_tma<EPI>(p, &tmC, &tmX, row, n0, v, stg, lane, bias_done);
          } else {
            epi_finish<EPI>(p, C, m_base, n0, v, stg, lane, bias_done);
          }
          if constexpr (EPI == kEpiBf16) {
            if (p.cmb_world > 0) epi_combine_push(p, m_base + lane, n0, v);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (p.tma_epi && lane == 0) bulk_wait_group0();  // every bulk store / reduce has landed
    __syncwarp();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// Launch one instantiation (defined in gemm_inst_*.cu).
template <int BN, bool A_MN, bool B_MN, int EPI>
void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const CUtensorMap& tx,
                 const GemmParams& p, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN, EPI>;
  static bool attr_set[64] = {};
  const int dev = current_device();
  if (!attr_set[dev]) {
    HB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    attr_set[dev] = true;
  }
  const int num_tiles =
      ((p.M + 127) / 128) * ((p.N + BN - 1) / BN) * p.splits * (p.grp_mode == 2 ? p.grp_n : 1);
  const int grid = num_tiles < num_sms(dev) ? num_tiles : num_sms(dev);
  kern<<<grid, kGemmThreads, Cfg::SMEM_BYTES, stream>>>(ta, tb, tc, tx, p);
  HB_CUDA_CHECK(cudaGetLastError());
}

// Dispatch over epilogues for one (BN, majors) combination.
template <int BN, bool A_MN, bool B_MN>
void gemm_dispatch_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                       const CUtensorMap& tx, const GemmParams& p, cudaStream_t s) {
  switch (epi) {
    case kEpiBf16: return launch_gemm<BN, A_MN, B_MN, kEpiBf16>(ta, tb, tc, tx, p, s);
    case kEpiBf16Gelu: return launch_gemm<BN, A_MN, B_MN, kEpiBf16Gelu>(ta, tb, tc, tx, p, s);
    case kEpiF32: return launch_gemm<BN, A_MN, B_MN, kEpiF32>(ta, tb, tc, tx, p, s);
    case kEpiF32Acc: return launch_gemm<BN, A_MN, B_MN, kEpiF32Acc>(ta, tb, tc, tx, p, s);
    case kEpiF32Resid: return launch_gemm<BN, A_MN, B_MN, kEpiF32Resid>(ta, tb, tc, tx, p, s);
    case kEpiBf16Dgelu: return launch_gemm<BN, A_MN, B_MN, kEpiBf16Dgelu>(ta, tb, tc, tx, p, s);
    case kEpiF32Atomic: return launch_gemm<BN, A_MN, B_MN, kEpiF32Atomic>(ta, tb, tc, tx, p, s);
    default: throw std::runtime_error("gemm: unknown epilogue");
  }
}

}  // namespace hb
