// Host-side encoding of TMA tensor maps (cuTensorMapEncodeTiled, reached through the
// runtime's driver entry-point query so the library needs no link against libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace p3d {

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// A tiled map with zero fill outside the tensor.  dims / box innermost first; strides
// (bytes) for dims 1..rank-1.
inline int encode_tiled(CUtensorMap *map, CUtensorMapDataType type, const void *ptr, int rank, const uint64_t *dims,
                        const uint64_t *strides, const uint32_t *box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return fail(P3D_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint32_t elem[5] = {1, 1, 1, 1, 1};
  const CUresult r = fn(map, type, rank, const_cast<void *>(ptr), dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(P3D_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return P3D_OK;
}

// 16-bit operand tiles for the tensor cores: boxes of 16 channels (32 bytes), SWIZZLE_32B.
inline int encode_operand(CUtensorMap *map, int dtype, const void *ptr, int rank, const uint64_t *dims,
                          const uint64_t *strides, const uint32_t *box) {
  return encode_tiled(map, dtype == P3D_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ptr,
                      rank, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_32B);
}

// 16-bit operand tiles with 64-channel (128-byte) rows, SWIZZLE_128B.
inline int encode_operand_sw128(CUtensorMap *map, int dtype, const void *ptr, int rank, const uint64_t *dims,
                                const uint64_t *strides, const uint32_t *box) {
  return encode_tiled(map, dtype == P3D_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ptr,
                      rank, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

// fp32 per-row values (logsumexp, Delta), no swizzle.
inline int encode_rows_f32(CUtensorMap *map, const float *ptr, int rank, const uint64_t *dims, const uint64_t *strides,
                           const uint32_t *box) {
  return encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ptr, rank, dims, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
}

}  // namespace p3d
