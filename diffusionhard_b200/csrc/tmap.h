// tmap.h -- host-side creation of TMA tensor maps (cuTensorMapEncodeTiled is
// reached through cudaGetDriverEntryPoint, so the library needs no direct
// libcuda symbol binding).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dh {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D row-major matrix [rows, cols] of `elem_bytes` elements with row stride
// `row_stride_bytes`; box [box_rows, box_cols] with 128-byte swizzle
// (box_cols * elem_bytes must be 128).  Out-of-range elements read as zero.
inline bool make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                         uint32_t elem_bytes, uint64_t rows, uint64_t cols,
                         uint64_t row_stride_bytes, uint32_t box_rows, uint32_t box_cols) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (row_stride_bytes & 15u) != 0) return false;
    if (box_cols * elem_bytes != 128 || box_rows == 0 || box_rows > 256) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Same, for a box whose rows are 64 bytes, with 64-byte swizzle: 16-byte
// piece c of box row r sits at piece c ^ ((r >> 1) & 3) of that row -- the
// layout of a TMA store source staged row by row without bank conflicts.
inline bool make_tmap_2d_sw64(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                              uint32_t elem_bytes, uint64_t rows, uint64_t cols,
                              uint64_t row_stride_bytes, uint32_t box_rows, uint32_t box_cols) {
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (row_stride_bytes & 15u) != 0) return false;
    if (box_cols * elem_bytes != 64 || box_rows == 0 || box_rows > 256) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                    CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace dh
