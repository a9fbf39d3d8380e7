#pragma once
// Pieces shared by the causal attention kernels of every head width
// (attention.cu: head_dim 64, attention_d128.cu: head_dim 128).
#include <cuda_bf16.h>

#include "common.cuh"
#include "dropout.cuh"

namespace hb {

struct AttnParams {
  int B, T, nh, Hs;         // Hs = nh * head_dim (this rank's heads)
  __nv_bfloat16* out;       // forward: y [B*T, ld_out]; backward: dqkv [B*T, ld_out]
  long ld_out;
  float* lse;               // [B, nh, Tpad] NEGATED log2-domain LSE of the scaled scores (-lse, the
                            // form the backward's fma consumes)
  int Tpad;
  const float* dvec;        // backward: -scale * D, D = rowsum(dO * O) [B, nh, Tpad]
  float* dq_acc;            // backward: fp32 dQ accumulator [B*T, Hs]
  float scale;              // softmax scale (1/sqrt(head_dim) unless the caller says otherwise)
  float scale_log2;         // scale * log2(e)
  int* status;
  uint64_t* trace;          // optional phase timestamps [grid][kTraceSlots] (nullptr: off)
  // Dropout on the attention probabilities (DROP instantiations only): mask
  // element ((b * nh_total + h0 + h) * T + q) * T + k.
  DropoutArgs drop;
  int h0, nh_total;
  // Forward softmax with O in registers (head_dim 64, the dropout path): share of the
  // exponentials evaluated on the FMA pipe (exp2_fma) instead of the transcendental
  // unit: 0 none, 1 one in eight (the default: 51.2 vs 53.2 us at B 8, T 1024, 12
  // heads), 2 one in four (53.2 us). The O-in-TMEM form always uses one in eight.
  int exp_fma;
};

// Phase tracing: with a trace buffer set, the kernels stamp %globaltimer at
// their pipeline hand-offs (slot layout documented at each kernel), which
// turns "where does a tile's time go" into a measurement. Off by default;
// one predicated branch per hand-off when off.
constexpr int kTraceSlots = 80;
#define HB_TRACE(slot)                                                                \
  do {                                                                                \
    if (p.trace != nullptr && (slot) < kTraceSlots)                                   \
      p.trace[(long)blockIdx.x * kTraceSlots + (slot)] = globaltimer_ns();            \
  } while (0)

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Byte offset of 16-byte chunk `c16` (0..15 over 128 bf16 columns) of row `r`
// in a K-major 128-byte-swizzled tile of 128-byte rows, laid out as 16 KB
// atoms of 64 columns (chunks 8..15 live in the second atom).
__device__ __forceinline__ uint32_t sw128_off(int r, int c16) {
  return (c16 >> 3) * 16384 + r * 128 + (((c16 & 7) ^ (r & 7)) << 4);
}

constexpr int kTile = 128;  // keys per key tile, queries per query tile

// exp2 on the special-function unit (PTX ex2.approx, flush-to-zero).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Tensor map over [B, T, cols] bf16 (row stride ld elements) with a box of
// 64 columns x `box_rows` rows, 128-byte swizzle: a box never crosses into
// the next sequence, and rows >= T read as zeros.
CUtensorMap attn_seq_map(const void* base, int B, int T, long ld, int cols, int box_rows);

}  // namespace hb
