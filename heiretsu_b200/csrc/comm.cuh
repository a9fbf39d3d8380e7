#pragma once
// Peer-memory primitives shared by the NVLink kernels (comm.cu, moe.cu):
// peer pointer table, release/acquire flag accessors and the bounded,
// epoch-tagged per-block group barrier.
#include <cuda_runtime.h>

#include "common.cuh"

namespace hb {

constexpr int kMaxRanks = 8;
constexpr int kMaxSignalBlocks = 1024;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct PeerTable {
  uint64_t data[kMaxRanks];    // peer data buffers (index = group rank)
  uint64_t signal[kMaxRanks];  // peer signal pads, uint32 [kMaxRanks][kMaxSignalBlocks]
};

// Per-block barrier across the group. Called by all threads of the block.
// `counter` is this rank's per-block epoch array (device memory, local).
// Returns false (after recording an error) if a peer did not arrive in time.
//
// The block-wide __syncthreads() before thread 0's system fence is what
// makes the release cover the stores of EVERY warp of the block (the fence
// is cumulative over what the CTA barrier ordered before it), not only
// thread 0's own: a barrier that follows a data phase ("results delivered")
// must not signal while other warps are still writing into peers' buffers.
__device__ __forceinline__ bool group_barrier(const PeerTable& pt, int rank, int world, uint32_t* counter,
                                              uint32_t phase_tag, int* status) {
  __shared__ int ok_sh;
  __syncthreads();
  if (threadIdx.x == 0) {
    ok_sh = 1;
    const uint32_t epoch = counter[blockIdx.x] + 1;  // advanced once per call, after both barriers
    const uint32_t val = epoch * 4u + phase_tag;
    __threadfence_system();
    for (int p = 0; p < world; ++p) {
      if (p == rank) continue;
      uint32_t* slot = reinterpret_cast<uint32_t*>(pt.signal[p]) + rank * kMaxSignalBlocks + blockIdx.x;
      st_release_sys(slot, val);
    }
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(pt.signal[rank]);
    const uint64_t t0 = globaltimer_ns();
    for (int p = 0; p < world && ok_sh; ++p) {
      if (p == rank) continue;
      const uint32_t* slot = mine + p * kMaxSignalBlocks + blockIdx.x;
      int spins = 0;
      while (static_cast<int32_t>(ld_acquire_sys(slot) - val) < 0) {
        // Back off after a short spin: a rank that is ahead waits here while its
        // peers finish their compute, and a tight poll in every CTA would take
        // issue slots from the kernels that share the SMs (the overlapped DP
        // reduction runs beside backward GEMMs and attention).
        if (spins > 32) __nanosleep(128);
        if (((++spins) & 255) == 0 && globaltimer_ns() - t0 > HB_WAIT_TIMEOUT_NS) {
          record_error(status, kPeerTimeout, 100 + p);
          ok_sh = 0;
          break;
        }
      }
      // A peer is at most one call ahead (same call sequence on every rank);
      // further ahead means the ranks issued different collectives.
      if (ok_sh && !HB_DCHECK(static_cast<int32_t>(ld_acquire_sys(slot) - val) < 8, status, 200 + p)) ok_sh = 0;
    }
  }
  __syncthreads();
  return ok_sh != 0;
}

}  // namespace hb
