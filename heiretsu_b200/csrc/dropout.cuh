#pragma once
// Counter-based dropout masks.
//
// A mask bit is a pure function of (seed, site, element index), so forward
// and backward recompute it instead of storing it, and a CUDA graph replay
// draws a fresh mask as long as the seed (read from device memory) changes.
// One 32-bit hash covers an element pair: its low and high 16 bits are two
// uniforms in [0, 65536); an element is kept when its uniform >= thresh,
// thresh = round(p * 65536), and kept values are scaled by 1 / (1 - p).
//
// The mixing function is "lowbias32" from Chris Wellons' Hash Prospector
// (public domain): x ^= x >> 16; x *= 0x7feb352d; x ^= x >> 15;
// x *= 0x846ca68b; x ^= x >> 16. The per-site key mixes the seed and the
// site id once; the high half of a 64-bit pair index is folded in per pair.
// heiretsu_b200/ops/dropout_ref.py restates the same arithmetic in PyTorch
// (the tests rebuild masks with it).
#include <cstdint>

#include "dropout_args.h"

namespace hb {


__host__ __device__ __forceinline__ uint32_t lowbias32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

// Key of one site under one seed (computed once per thread).
__device__ __forceinline__ uint32_t dropout_key(uint32_t seed, uint32_t site) {
  return lowbias32(seed ^ lowbias32(site * 0x9E3779B9u + 0x85EBCA6Bu));
}

// 32 random bits for element pair `pair` (= element index / 2) under `key`.
__device__ __forceinline__ uint32_t dropout_bits(uint32_t key, uint64_t pair) {
  return lowbias32(static_cast<uint32_t>(pair) ^ key ^ (static_cast<uint32_t>(pair >> 32) * 0xC2B2AE35u));
}

// Multipliers (0 or scale) of the element pair (2i, 2i+1).
__device__ __forceinline__ void dropout_pair(uint32_t bits, uint32_t thresh, float scale, float& m0, float& m1) {
  m0 = (bits & 0xFFFFu) >= thresh ? scale : 0.f;
  m1 = (bits >> 16) >= thresh ? scale : 0.f;
}

}  // namespace hb
