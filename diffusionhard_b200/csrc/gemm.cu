// gemm.cu -- W8A8 GEMM entry points on the tcgen05 kernel (gemm_tc.cuh).
//
// dh_gemm_i8_s32 exposes the raw int32 accumulators: the tensor-engine
// contract of the reference (torch._int_mm in fixed_mlp._integer_matmul,
// src/diffusion_accel/fixed_mlp.py:55-62; the 4x8x32 HLS MAC tile,
// hls/tensor_engine/int8_mac_tile.cpp:7-41) -- bit-exact by construction.
#include "gemm_tc.cuh"
#include "tmap.h"

namespace dh {
namespace {

struct EpiStoreI32 {
    static constexpr uint32_t kChunk = 32;
    struct Params {
        int32_t* c;
        uint64_t ldc;
        uint32_t n;
    };
    struct TileState {};
    static DH_DEVINL void tile_begin(const Params&, TileState&, uint32_t, bool, uint32_t) {}
    static DH_DEVINL void chunk(const Params& p, TileState&, uint32_t row, bool ok, uint32_t col0,
                                const uint32_t* v) {
        if (!ok) return;
        int32_t* dst = p.c + static_cast<uint64_t>(row) * p.ldc + col0;
        if (col0 + 32 <= p.n && (p.ldc & 3u) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
#pragma unroll
            for (uint32_t j = 0; j < 32; j += 4)
                *reinterpret_cast<int4*>(dst + j) = make_int4(static_cast<int32_t>(v[j]),
                                                              static_cast<int32_t>(v[j + 1]),
                                                              static_cast<int32_t>(v[j + 2]),
                                                              static_cast<int32_t>(v[j + 3]));
        } else {
#pragma unroll
            for (uint32_t j = 0; j < 32; ++j)
                if (col0 + j < p.n) dst[j] = static_cast<int32_t>(v[j]);
        }
    }
    static DH_DEVINL void tile_end(const Params&, TileState&, uint32_t, bool) {}
};

}  // namespace

// Shared validation + tensor maps for an int8 K-major operand pair.
uint32_t make_i8_operand_maps(CUtensorMap* ta, CUtensorMap* tb, const int8_t* a, uint64_t lda,
                              const int8_t* w, uint64_t ldw, uint32_t m, uint32_t n, uint32_t k,
                              uint32_t bn) {
    if (!a || !w) return DH_ERR_NULL_POINTER;
    if (m == 0 || n == 0 || k == 0) return DH_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(a) & 15u) || (reinterpret_cast<uintptr_t>(w) & 15u) ||
        (lda & 15u) || (ldw & 15u))
        return DH_ERR_ALIGNMENT;
    if (lda < k || ldw < k) return DH_ERR_INVALID_ARGUMENT;
    if (!make_tmap_2d(ta, a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, m, k, lda, 128, 128))
        return DH_ERR_CUDA;
    if (!make_tmap_2d(tb, w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, n, k, ldw, bn, 128))
        return DH_ERR_CUDA;
    return DH_OK;
}

}  // namespace dh

using namespace dh;

extern "C" uint32_t dh_gemm_i8_s32(const int8_t* a, uint64_t lda, const int8_t* w, uint64_t ldw,
                                   int32_t* c, uint64_t ldc, uint32_t m, uint32_t n, uint32_t k,
                                   void* stream) {
    if (!c) return DH_ERR_NULL_POINTER;
    if (ldc < n) return DH_ERR_INVALID_ARGUMENT;
    CUtensorMap ta, tb;
    uint32_t st = make_i8_operand_maps(&ta, &tb, a, lda, w, ldw, m, n, k, 256);
    if (st != DH_OK) return st;
    EpiStoreI32::Params p{c, ldc, n};
    GemmShape shape{m, n, k, nullptr};
    const uint32_t tiles = ((m + 127) / 128) * ((n + 255) / 256);
    if (launch_gemm_i8<256, EpiStoreI32>(ta, tb, shape, p, tiles,
                                         static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return DH_ERR_CUDA;
    return DH_OK;
}
