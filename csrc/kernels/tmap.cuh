// Host-side TMA tensor-map encoding through the driver entry point (no link against libcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace foa {

inline PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

// A K-major matrix of `rows` x `cols` elements of `dtype` (row stride `ld` elements), loaded in
// boxes of `box_rows` rows x `box_cols` elements with the given swizzle. Out-of-range rows and
// columns read as zero.
inline bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes,
                           const void* base, long rows, long cols, long ld, int box_rows,
                           int box_cols, CUtensorMapSwizzle swizzle) {
  auto fn = tmap_encoder();
  if (fn == nullptr) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return false;
  if ((ld * elem_bytes) % 16 != 0) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * elem_bytes)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// BF16 K-major operand in 64-element (128-byte) swizzled rows, as the GEMMs stage it.
inline bool encode_tmap_bf16_kmajor(CUtensorMap* map, const void* base, long rows, long k,
                                    long ld, int box_rows) {
  return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, rows, k, ld, box_rows, 64,
                        CU_TENSOR_MAP_SWIZZLE_128B);
}

// One-byte (FP8) K-major operand in 128-element (128-byte) swizzled rows.
inline bool encode_tmap_u8_kmajor(CUtensorMap* map, const void* base, long rows, long k, long ld,
                                  int box_rows) {
  return encode_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, base, rows, k, ld, box_rows, 128,
                        CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace foa
