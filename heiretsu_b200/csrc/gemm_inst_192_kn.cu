// Instantiations of the tcgen05 GEMM for BN=192, A_MN=false, B_MN=true (split
// across files so the build compiles them in parallel).
#include "gemm_kernel.cuh"

namespace hb {
void gemm_launch_192_kn(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                        const CUtensorMap& tx, const GemmParams& p, cudaStream_t s) {
  gemm_dispatch_epi<192, false, true>(epi, ta, tb, tc, tx, p, s);
}
}  // namespace hb
