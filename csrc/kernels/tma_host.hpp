// Host-side creation of TMA tensor maps (cuTensorMapEncodeTiled reached through
// the runtime's driver entry point, so nothing links libcuda directly).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <stdexcept>
#include <string>

namespace mgfa::host {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                                     cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point not available");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 16-bit (bf16 by default, or `dtype`) tensor map with `rank` dims (innermost first),
// byte strides of dims 1..rank-1,
// a box of `box` elements per dim and 128-byte swizzle. The innermost box extent
// must be 64 elements (128 bytes).
inline CUtensorMap make_bf16_map(const void* base, int rank, const uint64_t* dims,
                                 const uint64_t* byte_strides, const uint32_t* box,
                                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B,
                                 CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    throw std::invalid_argument("TMA base address must be 16-byte aligned");
  for (int i = 0; i < rank - 1; ++i)
    if (byte_strides[i] % 16 != 0)
      throw std::invalid_argument("TMA strides must be multiples of 16 bytes");
  CUtensorMap m;
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = tensor_map_encoder()(
      &m, dtype, cuuint32_t(rank), const_cast<void*>(base),
      reinterpret_cast<const cuuint64_t*>(dims), reinterpret_cast<const cuuint64_t*>(byte_strides),
      reinterpret_cast<const cuuint32_t*>(box), elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
      swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
  return m;
}

}  // namespace mgfa::host
