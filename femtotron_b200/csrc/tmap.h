// Host-side helpers to build TMA tensor maps (CUtensorMap) without linking libcuda directly:
// the driver entry point is fetched once through the runtime.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdexcept>
#include <string>

namespace ft {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("femtotron_b200: cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D row-major tensor [outer, inner] with `row_stride_elems` elements between rows.
// The box is [box_outer, box_inner]; `swizzle128` selects the 128-byte swizzle used by the
// UMMA shared-memory descriptors (box_inner * elem_bytes must then be 128).
inline CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, int elem_bytes,
                                uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                                uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * static_cast<uint64_t>(elem_bytes)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0)
    throw std::runtime_error("femtotron_b200: TMA base address must be 16-byte aligned");
  if (strides[0] % 16 != 0)
    throw std::runtime_error("femtotron_b200: TMA row stride must be a multiple of 16 bytes");
  CUresult r = encode_tiled_fn()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("femtotron_b200: cuTensorMapEncodeTiled failed with code " +
                             std::to_string(static_cast<int>(r)));
  return m;
}

}  // namespace ft
