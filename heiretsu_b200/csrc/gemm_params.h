// Parameters and epilogue codes of the tcgen05 GEMM (shared by host and device code).
#pragma once

namespace hb {

enum GemmEpi : int {
  kEpiBf16 = 0,       // C bf16 = acc (+ bias)
  kEpiBf16Gelu = 1,   // AUX bf16 = acc + bias ; C bf16 = gelu(acc + bias)
  kEpiF32 = 2,        // C f32 = acc (+ bias)
  kEpiF32Acc = 3,     // C f32 += acc
  kEpiF32Resid = 4,   // C f32 = R f32 + acc (+ bias)     (C may alias R)
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
};

}  // namespace hb
