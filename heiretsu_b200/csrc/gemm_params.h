// Parameters and epilogue codes of the tcgen05 GEMM (shared by host and device code).
#pragma once

#include "dropout_args.h"

namespace hb {

enum GemmEpi : int {
  // "Bf16" epilogues write the 16-bit format of the operands (bf16 or fp16, GemmParams::f16).
  kEpiBf16 = 0,       // C bf16 = acc (+ bias)
  kEpiBf16Gelu = 1,   // AUX bf16 = acc + bias ; C bf16 = gelu(acc + bias)
  kEpiF32 = 2,        // C f32 = acc (+ bias)
  kEpiF32Acc = 3,     // C f32 += acc
  kEpiF32Resid = 4,   // C f32 = R f32 + dropout(acc (+ bias))     (C may alias R; dropout optional)
  kEpiBf16Dgelu = 5,  // C bf16 = acc * gelu'(AUX)
  kEpiF32Atomic = 6,  // C f32 += acc with vector atomics (split-K partial sums)
};

struct GemmParams {
  int M, N, K;
  void* C;
  long ldc;
  const float* bias;  // [N] fp32 or nullptr
  void* aux;          // bf16 [M, ldaux]
  long ldaux;
  const float* resid;  // fp32 [M, ldr]
  long ldr;
  int* status;
  int splits;          // split-K factor (>= 1); tiles are (split, m-block, n-block)
  int kb_per_split;    // K blocks handled by one split
  int raster_n;        // 1: n-block fastest (CTAs in flight share A), 0: m-block fastest

  // All-gather prologue (tensor parallelism): A is the token-gathered matrix
  // [world * ag_rows, K] in local memory; rows [r * ag_rows, (r+1) * ag_rows)
  // are copied from rank r's shard (ag_src[r], row stride K) by the
  // epilogue warps at kernel start, and ag_flags[m-block] counts the 16-row
  // units delivered. 0 = off.
  int ag_world;
  int ag_rank;
  int ag_rows;
  const void* ag_src[8];
  void* ag_dst;
  int* ag_flags;

  // Reduce-scatter epilogue: the output tile of rows [m, m+128) belongs to
  // rank m / rs_rows; it is stored (not reduced) into slot rs_rank of that
  // rank's receive buffer rs_dst[owner] = [world][rs_rows][ldc]. 0 = off.
  int rs_world;
  int rs_rank;
  int rs_rows;
  void* rs_dst[8];

  // Expert-grouped GEMMs (mixture of experts). The rows of the permuted
  // activations are grouped by expert in segments padded to 128 rows;
  // grp_off[e] (device memory, grp_n + 1 entries) is the first row of expert e.
  //   grp_mode 1, row-grouped (forward / dgrad): the m-block's expert e selects
  //     the weights: B's row (K-major B) or k (MN-major B) coordinate is
  //     offset by e * grp_b_off. The m-block count is read on the device.
  //   grp_mode 2, reduction-grouped (weight gradients): tile (e, m, n) reduces
  //     over the rows of expert e into C rows offset by e * grp_c_off.
  int grp_mode;
  int grp_n;
  const int* grp_off;
  int grp_b_off;
  int grp_c_off;

  // Epilogue output through TMA: each 32x32 chunk leaves the swizzled staging
  // tile with one bulk tensor store (or an fp32 bulk reduce-add for the
  // accumulating epilogues) through the C / AUX tensor maps. 0 = per-lane
  // global stores (always the case for reduce-scatter peer outputs).
  int tma_epi;

  // 16-bit format of A, B and of the 16-bit outputs / AUX: 0 bf16, 1 fp16.
  int f16;

  // GELU / GELU' evaluation in the activation epilogues: 0 sigmoid form, one
  // ex2.approx per element; 1 the same with every other exponential on the FMA
  // pipe; 2 tanh.approx (the default).
  int gelu_mode;

  // Expert-parallel combine epilogue (row-grouped GEMM with a 16-bit output;
  // cmb_world = 0: off). Output row p of this rank's expert window holds the
  // expert output of routing slot cmb_inv[p] = t * cmb_K + k (-1: padding row).
  // Besides C, the epilogue stores 16-bit(cmb_w[t * cmb_K + k] * row) into row
  // t of slot k of every EP rank's receive buffer cmb_dst[r] = [cmb_K][cmb_N][N]
  // (peer stores over NVLink). Each (t, k) belongs to exactly one rank's
  // experts, so every slot row is written once per call.
  int cmb_world;
  int cmb_K;
  int cmb_N;
  const int* cmb_inv;
  const float* cmb_w;
  void* cmb_dst[8];

  // Residual dropout of the F32Resid epilogue (thresh 0 = off):
  // C = R + mask * (acc + bias), mask element (drop.row0 + row) * N + col.
  DropoutArgs drop;
};

}  // namespace hb
