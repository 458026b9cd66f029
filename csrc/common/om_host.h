// Host helpers shared by the extension's .cu files: error checks, SM count,
// TMA tensor-map encoding through the driver entry point (so the extension
// does not link libcuda directly and still imports on a machine without a GPU).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <atomic>
#include <mutex>

#define OM_CUDA_CHECK(x)                                                                   \
  do {                                                                                     \
    cudaError_t _e = (x);                                                                  \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error ", cudaGetErrorString(_e), " at ", __FILE__, \
                ":", __LINE__);                                                            \
  } while (0)

// Check the last launch and count it.
#define OM_LAUNCH_CHECK()                  \
  do {                                     \
    OM_CUDA_CHECK(cudaGetLastError());     \
    om::g_launches.fetch_add(1);           \
  } while (0)

namespace om {

// Host-side count of kernel launches issued by this library (also counts
// launches recorded into a CUDA graph during capture).
inline std::atomic<long long> g_launches{0};

inline int num_sms(int dev = -1) {
  static int cache[64] = {0};
  if (dev < 0) OM_CUDA_CHECK(cudaGetDevice(&dev));
  if (cache[dev] == 0) OM_CUDA_CHECK(cudaDeviceGetAttribute(&cache[dev], cudaDevAttrMultiProcessorCount, dev));
  return cache[dev];
}

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    OM_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Row-major 2-D tensor [outer, inner] with row stride `ld` elements.
inline CUtensorMap make_tmap_2d(const void* ptr, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                                uint64_t outer, uint64_t ld, uint32_t box_inner, uint32_t box_outer,
                                CUtensorMapSwizzle sw) {
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((strides[0] & 15) == 0, "TMA row stride must be a multiple of 16 bytes");
  CUresult r = encode_fn()(&m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

// 3-D tensor [d2, d1, d0] (d0 innermost) with strides s1, s2 in elements.
inline CUtensorMap make_tmap_3d(const void* ptr, CUtensorMapDataType dt, int elem_bytes, uint64_t d0, uint64_t d1,
                                uint64_t d2, uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, uint32_t b2,
                                CUtensorMapSwizzle sw) {
  CUtensorMap m;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1 * (uint64_t)elem_bytes, s2 * (uint64_t)elem_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((strides[0] & 15) == 0 && (strides[1] & 15) == 0, "TMA strides must be multiples of 16 bytes");
  CUresult r = encode_fn()(&m, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3d) failed: ", (int)r);
  return m;
}

}  // namespace om
