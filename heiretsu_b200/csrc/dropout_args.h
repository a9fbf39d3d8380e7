// Arguments of a counter-based dropout site (plain struct shared by host
// and device code; the mask arithmetic is in dropout.cuh).
#pragma once
#include <cstdint>

namespace hb {

struct DropoutArgs {
  const uint32_t* seed;  // device scalar, a per-forward snapshot of the step's seed; nullptr = off
  uint32_t site;         // distinct per dropout site (layer, position)
  uint32_t thresh;       // round(p * 65536); 0 = off
  float scale;           // 1 / (1 - p)
  long row0;             // first global row of this rank's rows (token shards)
};

}  // namespace hb
