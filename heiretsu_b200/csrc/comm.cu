// NVLink peer-memory runtime and the fused data-parallel gradient reduction.
//
// Symmetric buffers: every rank of a group allocates the same number of
// bytes with cudaMalloc, exports a CUDA IPC handle, and opens the handles of
// its peers (handles travel over torch.distributed). A kernel then holds a
// device pointer to every peer's buffer and moves data with plain loads and
// stores over NVLink -- no staging copies, no library kernel touching peer
// memory, no TMA multicast.
//
// Signal pads: a small symmetric uint32 array per group. Slot
// [src_rank][block] on rank p is written (st.release.sys) by block `block`
// of rank src_rank and polled (ld.acquire.sys) by block `block` of rank p.
// Values are epoch-tagged and monotonic, and the epoch counter lives in
// device memory (per block), so captured CUDA graphs replay correctly.
// Every wait is bounded: on timeout the kernel records kPeerTimeout in the
// device status word and returns (the host raises CommTimeoutError).
//
// Fused DP all-reduce (replaces reference dp.py:13-26): rank r owns chunk r
// of the flat fp32 gradient buffer. Each block, for its part of chunk r,
// loads the chunk from all peers (vector P2P loads issued back to back),
// sums in a fixed rank order, multiplies by 1/world, and stores the result
// into the same chunk of every peer's buffer (push all-gather). Two
// per-block barriers bracket the data phase: "all inputs ready" and "all
// results delivered". Every rank moves (world-1)/world of the buffer in each
// direction over NVLink, once.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "comm.cuh"
#include "common.cuh"
#include "host_utils.h"

namespace hb {

__global__ void __launch_bounds__(512) dp_allreduce_kernel(PeerTable pt, int rank, int world, long n4, long chunk4,
                                                           float scale, uint32_t* counter, int* status) {
  if (!group_barrier(pt, rank, world, counter, 1, status)) return;
  const long begin = (long)rank * chunk4;
  const long end = min(n4, begin + chunk4);
  for (long i = begin + (long)blockIdx.x * blockDim.x + threadIdx.x; i < end; i += (long)gridDim.x * blockDim.x) {
    float4 v[kMaxRanks];
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p)
      if (p < world) v[p] = reinterpret_cast<const float4*>(pt.data[p])[i];
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p) {
      if (p < world) {
        s.x += v[p].x;
        s.y += v[p].y;
        s.z += v[p].z;
        s.w += v[p].w;
      }
    }
    s.x *= scale;
    s.y *= scale;
    s.z *= scale;
    s.w *= scale;
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p)
      if (p < world) reinterpret_cast<float4*>(pt.data[p])[i] = s;
  }
  if (!group_barrier(pt, rank, world, counter, 2, status)) return;
  if (threadIdx.x == 0) counter[blockIdx.x] += 1;
}

// Sum of peer partials (expert-parallel combine and its backward):
//   dst[i] = addend[i] (or 0) + sum_{r = 0 .. world-1} data_r[i]
// after one bounded barrier ("every rank's partial is written"). Every rank
// computes the whole sum in the same rank order, so all replicas hold
// bitwise-identical results. One barrier per call is enough when each call
// site owns its buffer: a rank writes that buffer again only after a later
// barrier, which its peers reach only after finishing this read.
__global__ void __launch_bounds__(512) peer_sum_kernel(PeerTable pt, int rank, int world, const float* addend,
                                                        float* dst, long n4, uint32_t* counter, int* status) {
  if (!group_barrier(pt, rank, world, counter, 1, status)) return;
  const float4* add4 = reinterpret_cast<const float4*>(addend);
  float4* dst4 = reinterpret_cast<float4*>(dst);
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    float4 v[kMaxRanks];
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p)
      if (p < world) v[p] = reinterpret_cast<const float4*>(pt.data[p])[i];
    float4 s = add4 ? add4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p) {
      if (p < world) {
        s.x += v[p].x;
        s.y += v[p].y;
        s.z += v[p].z;
        s.w += v[p].w;
      }
    }
    dst4[i] = s;
  }
  if (threadIdx.x == 0) counter[blockIdx.x] += 1;
}

// Bounded barrier kernel (also used by the tests' "peer never arrives" case).
__global__ void group_barrier_kernel(PeerTable pt, int rank, int world, uint32_t* counter, int* status) {
  if (!group_barrier(pt, rank, world, counter, 3, status)) return;
  if (threadIdx.x == 0) counter[blockIdx.x] += 1;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static std::mutex g_ipc_mu;

std::vector<uint8_t> ipc_handle(uint64_t ptr) {
  cudaIpcMemHandle_t h;
  HB_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  std::vector<uint8_t> out(sizeof(h));
  std::memcpy(out.data(), &h, sizeof(h));
  return out;
}

uint64_t ipc_open(const std::vector<uint8_t>& handle) {
  if (handle.size() != sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("ipc_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  std::lock_guard<std::mutex> lk(g_ipc_mu);
  HB_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<uint64_t>(p);
}

void ipc_close(uint64_t ptr) { HB_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

static PeerTable make_table(const std::vector<uint64_t>& data, const std::vector<uint64_t>& signal) {
  if (data.size() > kMaxRanks || signal.size() != data.size())
    throw std::runtime_error("peer table: at most 8 ranks, one signal pad per rank");
  PeerTable t{};
  for (size_t i = 0; i < data.size(); ++i) {
    t.data[i] = data[i];
    t.signal[i] = signal[i];
  }
  return t;
}

int dp_allreduce_blocks(int device) { return num_sms(device); }

void dp_allreduce_launch(const std::vector<uint64_t>& data, const std::vector<uint64_t>& signal, int rank,
                         long n, float scale, uint32_t* counter, int* status, int threads, int blocks_req,
                         cudaStream_t s) {
  const int world = static_cast<int>(data.size());
  if (n % 4 != 0) throw std::runtime_error("dp_allreduce: element count must be a multiple of 4");
  // float4 peer loads and stores: an unaligned range start would fault the GPU.
  for (uint64_t ptr : data)
    if (ptr % 16) throw std::runtime_error("dp_allreduce: peer ranges must start 16-byte aligned");
  const PeerTable t = make_table(data, signal);
  const long n4 = n / 4;
  const long chunk4 = (n4 + world - 1) / world;
  // blocks_req = 0: one CTA per SM. Every rank must pass the same block count
  // for the same call (the barrier epochs are per block index).
  const int blocks = std::min(blocks_req > 0 ? blocks_req : dp_allreduce_blocks(current_device()), kMaxSignalBlocks);
  // threads = 512: the whole GPU moves the data (reduction after backward).
  // threads = 64: a footprint of 2 warps and ~3K registers per SM, small
  // enough to sit beside a persistent GEMM / attention CTA, so the reduction
  // runs underneath backward compute; with few blocks it also stays off most SMs.
  if (threads != 512 && threads != 256 && threads != 128 && threads != 64)
    throw std::runtime_error("dp_allreduce: threads must be 64, 128, 256 or 512");
  dp_allreduce_kernel<<<blocks, threads, 0, s>>>(t, rank, world, n4, chunk4, scale, counter, status);
  HB_CUDA_CHECK(cudaGetLastError());
}

void peer_sum_launch(const std::vector<uint64_t>& data, const std::vector<uint64_t>& signal, int rank,
                     const float* addend, float* dst, long n, uint32_t* counter, int* status, cudaStream_t s) {
  const int world = static_cast<int>(data.size());
  if (n % 4 != 0) throw std::runtime_error("peer_sum: element count must be a multiple of 4");
  for (uint64_t ptr : data)
    if (ptr % 16) throw std::runtime_error("peer_sum: peer buffers must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(addend)) % 16)
    throw std::runtime_error("peer_sum: dst / addend must be 16-byte aligned");
  const PeerTable t = make_table(data, signal);
  const int blocks = std::min(num_sms(current_device()), kMaxSignalBlocks);
  peer_sum_kernel<<<blocks, 512, 0, s>>>(t, rank, world, addend, dst, n / 4, counter, status);
  HB_CUDA_CHECK(cudaGetLastError());
}

void group_barrier_launch(const std::vector<uint64_t>& data, const std::vector<uint64_t>& signal, int rank,
                          uint32_t* counter, int* status, cudaStream_t s) {
  const PeerTable t = make_table(data, signal);
  group_barrier_kernel<<<1, 32, 0, s>>>(t, rank, static_cast<int>(data.size()), counter, status);
  HB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace hb
