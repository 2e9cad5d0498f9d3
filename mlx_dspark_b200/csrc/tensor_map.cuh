// Host helpers shared by the TMA-fed kernels: the driver's tensor-map encoder (reached through
// cudaGetDriverEntryPoint, so the library links without libcuda), 2-D tiled map encoding with
// the 16-byte alignment rules checked, and the device's SM count.
#pragma once

#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace dspark {

inline PFN_cuTensorMapEncodeTiled_v12000 get_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

inline int make_map_2d(CUtensorMap* map, CUtensorMapDataType dt, int elem_bytes, const void* ptr,
                       uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
                       uint32_t box_outer, CUtensorMapSwizzle swz) {
  auto enc = get_encoder();
  if (!enc) return set_error(DSPARK_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0 || (row_bytes & 15u) != 0)
    return set_error(DSPARK_ERR_ALIGN, "tensor map base/stride not 16-byte aligned");
  if ((box_inner * (uint32_t)elem_bytes) % 16u != 0)
    return set_error(DSPARK_ERR_ALIGN, "tensor map box inner extent not a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DSPARK_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DSPARK_OK;
}

inline int sm_count() {
  static int cached = 0;
  if (cached) return cached;
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (n > 0) cached = n;
  return n > 0 ? n : 148;
}

}  // namespace dspark
