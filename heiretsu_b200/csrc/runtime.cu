// Host runtime pieces of the extension: device properties, the per-device
// status word that bounded device-side waits report into, and TMA tensor-map
// encoding through the driver entry point (no link-time libcuda dependency).
#include <mutex>
#include <vector>

#include "host_utils.h"

namespace hb {

int current_device() {
  int d = 0;
  HB_CUDA_CHECK(cudaGetDevice(&d));
  return d;
}

int num_sms(int device) {
  static int cache[64] = {};
  if (cache[device] == 0) {
    HB_CUDA_CHECK(cudaDeviceGetAttribute(&cache[device], cudaDevAttrMultiProcessorCount, device));
  }
  return cache[device];
}

static std::mutex g_status_mu;
static int* g_status[64] = {};

int* device_status_ptr(int device) {
  if (g_status[device] != nullptr) return g_status[device];
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (g_status[device] == nullptr) {
    int prev = current_device();
    HB_CUDA_CHECK(cudaSetDevice(device));
    int* p = nullptr;
    HB_CUDA_CHECK(cudaMalloc(&p, sizeof(int)));
    HB_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
    HB_CUDA_CHECK(cudaDeviceSynchronize());
    g_status[device] = p;
    HB_CUDA_CHECK(cudaSetDevice(prev));
  }
  return g_status[device];
}

// Returns the status word of `device` and clears it (synchronises the device).
int64_t read_and_clear_status(int64_t device) {
  int* p = device_status_ptr(static_cast<int>(device));
  int prev = current_device();
  HB_CUDA_CHECK(cudaSetDevice(static_cast<int>(device)));
  int v = 0;
  HB_CUDA_CHECK(cudaDeviceSynchronize());
  HB_CUDA_CHECK(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
  HB_CUDA_CHECK(cudaMemset(p, 0, sizeof(int)));
  HB_CUDA_CHECK(cudaSetDevice(prev));
  return v;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    HB_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || ptr == nullptr) {
      throw std::runtime_error("cuTensorMapEncodeTiled entry point not found");
    }
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

CUtensorMap make_tmap(CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                      const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  CUtensorMap m;
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) {
    if (strides_bytes[i] % 16 != 0) throw std::runtime_error("tensor map stride must be a multiple of 16 bytes");
    gstride[i] = strides_bytes[i];
  }
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) throw std::runtime_error("tensor map base must be 16B aligned");
  CUresult r = get_encode_fn()(&m, dtype, rank, const_cast<void*>(base), gdim, gstride, bdim, estride,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    throw std::runtime_error("cuTensorMapEncodeTiled failed with code " + std::to_string(static_cast<int>(r)));
  }
  return m;
}

CUtensorMap make_tmap_bf16(int rank, const void* base, const uint64_t* dims, const uint64_t* strides_bytes,
                           const uint32_t* box, CUtensorMapSwizzle swizzle) {
  return make_tmap(CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, base, dims, strides_bytes, box, swizzle);
}

CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                              uint32_t box_inner, uint32_t box_outer) {
  const uint64_t dims[2] = {inner, outer};
  const uint64_t strides[1] = {row_stride_bytes};
  const uint32_t box[2] = {box_inner, box_outer};
  return make_tmap_bf16(2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace hb
