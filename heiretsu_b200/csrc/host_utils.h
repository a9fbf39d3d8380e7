// Host-side helpers shared by the extension's .cu files: error checks,
// device properties, the per-device status word and TMA descriptor encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

#define HB_CUDA_CHECK(expr)                                                                   \
  do {                                                                                        \
    cudaError_t _e = (expr);                                                                  \
    if (_e != cudaSuccess) {                                                                  \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(_e) + " at " + \
                               __FILE__ + ":" + std::to_string(__LINE__));                    \
    }                                                                                         \
  } while (0)

namespace hb {

int current_device();
int num_sms(int device);

// Per-device int32 written by kernels whose bounded waits expired (see
// common.cuh StatusCode). Allocated on first use; never freed.
int* device_status_ptr(int device);

// 2-D bf16 tensor map with 128-byte swizzle: `inner` contiguous elements per
// row, `outer` rows, `row_stride_bytes` between rows; box = box_inner x box_outer.
CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                              uint32_t box_inner, uint32_t box_outer);

// Tensor map of any element type with a chosen swizzle.
CUtensorMap make_tmap(CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

// Generic 2-D/3-D tensor map (any 2-byte dtype) with a chosen swizzle.
CUtensorMap make_tmap_bf16(int rank, const void* base, const uint64_t* dims, const uint64_t* strides_bytes,
                           const uint32_t* box, CUtensorMapSwizzle swizzle);

}  // namespace hb
