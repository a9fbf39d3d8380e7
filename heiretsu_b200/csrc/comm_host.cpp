// Torch-facing entry points of the peer-memory runtime (comm.cu):
// raw device allocations for symmetric buffers, CUDA IPC handle export /
// import, and the fused DP all-reduce and barrier launches.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "host_utils.h"
#include "ops.h"

namespace hb {

std::vector<uint8_t> ipc_handle(uint64_t ptr);
uint64_t ipc_open(const std::vector<uint8_t>& handle);
void ipc_close(uint64_t ptr);
void dp_allreduce_launch(const std::vector<uint64_t>& data, const std::vector<uint64_t>& signal, int rank, long n,
                         float scale, uint32_t* counter, int* status, int threads, int blocks, cudaStream_t s);
void group_barrier_launch(const std::vector<uint64_t>& data, const std::vector<uint64_t>& signal, int rank,
                          uint32_t* counter, int* status, cudaStream_t s);
void peer_sum_launch(const std::vector<uint64_t>& data, const std::vector<uint64_t>& signal, int rank,
                     const float* addend, float* dst, long n, uint32_t* counter, int* status, cudaStream_t s);

uint64_t raw_malloc(int64_t bytes) {
  void* p = nullptr;
  HB_CUDA_CHECK(cudaMalloc(&p, static_cast<size_t>(bytes)));
  HB_CUDA_CHECK(cudaMemset(p, 0, static_cast<size_t>(bytes)));
  HB_CUDA_CHECK(cudaDeviceSynchronize());
  return reinterpret_cast<uint64_t>(p);
}

void raw_free(uint64_t ptr) { HB_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

at::Tensor tensor_from_ptr(uint64_t ptr, int64_t numel, at::ScalarType dtype, int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, device);
  return at::from_blob(reinterpret_cast<void*>(ptr), {numel}, [](void*) {}, opts);
}

py::bytes ipc_handle_py(uint64_t ptr) {
  auto v = ipc_handle(ptr);
  return py::bytes(reinterpret_cast<const char*>(v.data()), v.size());
}

uint64_t ipc_open_py(py::bytes handle) {
  std::string s = handle;
  std::vector<uint8_t> v(s.begin(), s.end());
  return ipc_open(v);
}

void dp_allreduce(const std::vector<uint64_t>& data, const std::vector<uint64_t>& signal, int64_t rank, int64_t n,
                  double scale, const at::Tensor& counter, int64_t threads, int64_t blocks) {
  TORCH_CHECK(counter.is_cuda() && counter.scalar_type() == at::kInt && counter.numel() >= 1024,
              "dp_allreduce: counter must be int32 [>=1024] on the device");
  c10::cuda::CUDAGuard g(counter.device());
  dp_allreduce_launch(data, signal, static_cast<int>(rank), n, static_cast<float>(scale),
                      reinterpret_cast<uint32_t*>(counter.data_ptr()), device_status_ptr(counter.get_device()),
                      static_cast<int>(threads), static_cast<int>(blocks), at::cuda::getCurrentCUDAStream());
}

void group_barrier(const std::vector<uint64_t>& data, const std::vector<uint64_t>& signal, int64_t rank,
                   const at::Tensor& counter) {
  c10::cuda::CUDAGuard g(counter.device());
  group_barrier_launch(data, signal, static_cast<int>(rank), reinterpret_cast<uint32_t*>(counter.data_ptr()),
                       device_status_ptr(counter.get_device()), at::cuda::getCurrentCUDAStream());
}

void peer_sum(const std::vector<uint64_t>& data, const std::vector<uint64_t>& signal, int64_t rank,
              const c10::optional<at::Tensor>& addend, const at::Tensor& dst, int64_t n, const at::Tensor& counter) {
  TORCH_CHECK(counter.is_cuda() && counter.scalar_type() == at::kInt && counter.numel() >= 1024,
              "peer_sum: counter must be int32 [>=1024] on the device");
  TORCH_CHECK(dst.is_cuda() && dst.scalar_type() == at::kFloat && dst.is_contiguous() && dst.numel() >= n,
              "peer_sum: dst must be contiguous fp32 with >= n elements");
  const float* add = nullptr;
  if (addend && addend->defined()) {
    TORCH_CHECK(addend->scalar_type() == at::kFloat && addend->is_contiguous() && addend->numel() >= n,
                "peer_sum: addend must be contiguous fp32 with >= n elements");
    add = addend->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(counter.device());
  peer_sum_launch(data, signal, static_cast<int>(rank), add, dst.data_ptr<float>(), n,
                  reinterpret_cast<uint32_t*>(counter.data_ptr()), device_status_ptr(counter.get_device()),
                  at::cuda::getCurrentCUDAStream());
}

}  // namespace hb
