// Host-side creation of TMA tensor maps (CUtensorMap) for 2-D row-major operands. The driver
// entry point is looked up through the runtime, so the library does not link libcuda.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mrn {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// A K-major operand [rows, k] (row stride = `row_elems` elements, k when 0) read in boxes of
// `box_rows` rows x 128 bytes with 128-byte swizzling. `elem_bytes` is 2 (bf16) or 1 (e4m3).
// Rows and columns outside the tensor read as zero. Returns false on failure.
inline bool make_kmajor_map(CUtensorMap* map, const void* base, int elem_bytes, uint64_t rows, uint64_t k,
                            uint32_t box_rows, uint64_t row_elems = 0) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  if (row_elems == 0) row_elems = k;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (row_elems * elem_bytes) % 16 != 0 || row_elems < k)
    return false;
  const cuuint64_t dims[2] = {k, rows};
  const cuuint64_t strides[1] = {row_elems * static_cast<uint64_t>(elem_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / elem_bytes), box_rows};
  const cuuint32_t estrides[2] = {1, 1};
  const CUtensorMapDataType dt = elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estrides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// A row-major output [rows, cols] (row stride `ld` elements) written in 32 x 32 blocks whose
// rows are 32 * elem_bytes bytes, with the matching swizzle (128, 64 or 32 bytes).
inline bool make_store_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t rows,
                           uint64_t cols, uint64_t ld) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (ld * elem_bytes) % 16 != 0) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * static_cast<uint64_t>(elem_bytes)};
  const cuuint32_t box[2] = {32, 32};
  const cuuint32_t estrides[2] = {1, 1};
  const CUtensorMapSwizzle sw = elem_bytes == 4   ? CU_TENSOR_MAP_SWIZZLE_128B
                                : elem_bytes == 2 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                  : CU_TENSOR_MAP_SWIZZLE_32B;
  const CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estrides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace mrn
