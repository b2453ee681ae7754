// gemm.cu -- W8A8 GEMM entry points on the tcgen05 kernel (gemm_tc.cuh).
//
// dh_gemm_i8_s32 exposes the raw int32 accumulators: the tensor-engine
// contract of the reference (torch._int_mm in fixed_mlp._integer_matmul,
// src/diffusion_accel/fixed_mlp.py:55-62; the 4x8x32 HLS MAC tile,
// hls/tensor_engine/int8_mac_tile.cpp:7-41) -- bit-exact by construction.
#include <cuda_bf16.h>

#include "gemm_tc.cuh"
#include "tmap.h"

namespace dh {
namespace {

struct EpiStoreI32 : EpiBase {
    static constexpr uint32_t kChunk = 32;
    struct Params {
        int32_t* c;
        uint64_t ldc;
        uint32_t n;
    };
    struct TileState {};
    static DH_DEVINL void tile_begin(const Params&, TileState&, uint32_t, bool, uint32_t, uint8_t*) {}
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

// y = acc * (a_scale[row] * w_scale[col]) + bias[col]   (fp32)
DH_DEVINL float dequant(uint32_t acc, float ab, float w, float b) {
    return __fmaf_rn(static_cast<float>(static_cast<int32_t>(acc)), ab * w, b);
}

// QKV projection (N = 3 * 768): dequant + rotary on q and k (rotate-half,
// mlx_mdlm.py:316-329 / mdlm.py:399-410), then scatter to the attention
// layouts: Q, K as [B, H, len, 64] and V transposed as [B, H, 64, kv_len], all
// bf16.  A chunk is 64 columns = one head of one of q / k / v.
struct EpiQKV : EpiBase {
    static constexpr uint32_t kChunk = 64;
    struct Params {
        const float* a_scale;
        const float* w_scale;
        const float* bias;
        const float* rope_cos;  // [max_pos, 32]
        const float* rope_sin;
        uint32_t seq_len;       // rows per sequence in this forward
        uint32_t pos_offset;    // rotary position of the first row of a sequence
        uint32_t kv_stride;     // rows per (sequence, head) in the K / V buffers
        uint32_t kv_offset;     // where this forward's rows go in K / V
        __nv_bfloat16* q;
        __nv_bfloat16* k;
        __nv_bfloat16* vt;
    };
    struct TileState {};
    static DH_DEVINL void tile_begin(const Params&, TileState&, uint32_t, bool, uint32_t, uint8_t*) {}
    static DH_DEVINL void chunk(const Params& p, TileState&, uint32_t row, bool ok, uint32_t col0,
                                const uint32_t* v) {
        if (!ok) return;
        const float ab = p.a_scale[row];
        const uint32_t which = col0 / 768u;
        const uint32_t h = (col0 % 768u) / 64u;
        const uint32_t b = row / p.seq_len;
        const uint32_t t = row % p.seq_len;
        float y[64];
#pragma unroll
        for (uint32_t j = 0; j < 64; ++j)
            y[j] = dequant(v[j], ab, __ldg(p.w_scale + col0 + j), __ldg(p.bias + col0 + j));
        const uint32_t heads = 12;
        if (which < 2) {
            const float* cs = p.rope_cos + static_cast<uint64_t>(t + p.pos_offset) * 32;
            const float* sn = p.rope_sin + static_cast<uint64_t>(t + p.pos_offset) * 32;
#pragma unroll
            for (uint32_t i = 0; i < 32; ++i) {
                const float c = __ldg(cs + i), s = __ldg(sn + i);
                const float x1 = y[i], x2 = y[i + 32];
                y[i] = x1 * c - x2 * s;
                y[i + 32] = x2 * c + x1 * s;
            }
            const uint32_t len = which == 0 ? p.seq_len : p.kv_stride;
            const uint32_t pos = which == 0 ? t : t + p.kv_offset;
            __nv_bfloat16* dst = (which == 0 ? p.q : p.k) +
                                 ((static_cast<uint64_t>(b) * heads + h) * len + pos) * 64;
#pragma unroll
            for (uint32_t j = 0; j < 64; j += 8) {
                uint4 pk;
                __nv_bfloat162* hp = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                for (uint32_t e = 0; e < 4; ++e) hp[e] = __floats2bfloat162_rn(y[j + 2 * e], y[j + 2 * e + 1]);
                *reinterpret_cast<uint4*>(dst + j) = pk;
            }
        } else {
            __nv_bfloat16* dst = p.vt + (static_cast<uint64_t>(b) * heads + h) * 64 * p.kv_stride +
                                 t + p.kv_offset;
#pragma unroll
            for (uint32_t j = 0; j < 64; ++j) dst[static_cast<uint64_t>(j) * p.kv_stride] = __float2bfloat16_rn(y[j]);
        }
    }
    static DH_DEVINL void tile_end(const Params&, TileState&, uint32_t, bool) {}
};

// x[row, col] += acc * (a_scale * w_scale) + bias  (attention out, MLP down).
struct EpiResidual : EpiBase {
    static constexpr uint32_t kChunk = 32;
    struct Params {
        const float* a_scale;
        const float* w_scale;
        const float* bias;  // may be null
        float* x;
        uint32_t n;
    };
    struct TileState {};
    static DH_DEVINL void tile_begin(const Params&, TileState&, uint32_t, bool, uint32_t, uint8_t*) {}
    static DH_DEVINL void chunk(const Params& p, TileState&, uint32_t row, bool ok, uint32_t col0,
                                const uint32_t* v) {
        if (!ok) return;
        const float ab = p.a_scale[row];
        float4* dst = reinterpret_cast<float4*>(p.x + static_cast<uint64_t>(row) * p.n + col0);
#pragma unroll
        for (uint32_t j = 0; j < 32; j += 4) {
            float4 o = dst[j / 4];
            const float4 w = __ldg(reinterpret_cast<const float4*>(p.w_scale + col0 + j));
            float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
            if (p.bias) b = __ldg(reinterpret_cast<const float4*>(p.bias + col0 + j));
            o.x += dequant(v[j], ab, w.x, b.x);
            o.y += dequant(v[j + 1], ab, w.y, b.y);
            o.z += dequant(v[j + 2], ab, w.z, b.z);
            o.w += dequant(v[j + 3], ab, w.w, b.w);
            dst[j / 4] = o;
        }
    }
    static DH_DEVINL void tile_end(const Params&, TileState&, uint32_t, bool) {}
};

DH_DEVINL float gelu_tanh(float x) {
    // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))   (nn.GELU(approx="tanh"))
    const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
    return 0.5f * x * (1.0f + t);
}

// out[row, col] = bf16(gelu_tanh(acc * (a_scale * w_scale) + bias))  (MLP up).
struct EpiGelu : EpiBase {
    static constexpr uint32_t kChunk = 32;
    struct Params {
        const float* a_scale;
        const float* w_scale;
        const float* bias;
        __nv_bfloat16* out;
        uint32_t n;
    };
    struct TileState {};
    static DH_DEVINL void tile_begin(const Params&, TileState&, uint32_t, bool, uint32_t, uint8_t*) {}
    static DH_DEVINL void chunk(const Params& p, TileState&, uint32_t row, bool ok, uint32_t col0,
                                const uint32_t* v) {
        if (!ok) return;
        const float ab = p.a_scale[row];
        __nv_bfloat16* dst = p.out + static_cast<uint64_t>(row) * p.n + col0;
#pragma unroll
        for (uint32_t j = 0; j < 32; j += 8) {
            uint4 pk;
            __nv_bfloat162* hp = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
            for (uint32_t e = 0; e < 4; ++e) {
                const uint32_t c = j + 2 * e;
                const float a0 = gelu_tanh(dequant(v[c], ab, __ldg(p.w_scale + col0 + c), __ldg(p.bias + col0 + c)));
                const float a1 = gelu_tanh(dequant(v[c + 1], ab, __ldg(p.w_scale + col0 + c + 1), __ldg(p.bias + col0 + c + 1)));
                hp[e] = __floats2bfloat162_rn(a0, a1);
            }
            *reinterpret_cast<uint4*>(dst + j) = pk;
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

extern "C" uint32_t dh_gemm_qkv_rope(const int8_t* a, const float* a_scale, const int8_t* w,
                                     const float* w_scale, const float* bias, const float* rope_cos,
                                     const float* rope_sin, uint32_t m, uint32_t seq_len,
                                     uint32_t pos_offset, uint32_t kv_stride, uint32_t kv_offset,
                                     void* q, void* k, void* vt, const uint32_t* run_rows,
                                     void* stream) {
    if (!a_scale || !w_scale || !bias || !rope_cos || !rope_sin || !q || !k || !vt)
        return DH_ERR_NULL_POINTER;
    if (seq_len == 0 || m % seq_len != 0 || kv_offset + seq_len > kv_stride)
        return DH_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k)) & 15u) return DH_ERR_ALIGNMENT;
    CUtensorMap ta, tb;
    uint32_t st = make_i8_operand_maps(&ta, &tb, a, 768, w, 768, m, 2304, 768, 256);
    if (st != DH_OK) return st;
    EpiQKV::Params p{a_scale, w_scale, bias, rope_cos, rope_sin, seq_len, pos_offset, kv_stride,
                     kv_offset, static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k),
                     static_cast<__nv_bfloat16*>(vt)};
    GemmShape shape{m, 2304, 768, run_rows};
    const uint32_t tiles = ((m + 127) / 128) * 9;
    if (launch_gemm_i8<256, EpiQKV>(ta, tb, shape, p, tiles, static_cast<cudaStream_t>(stream)) !=
        cudaSuccess)
        return DH_ERR_CUDA;
    return DH_OK;
}

extern "C" uint32_t dh_gemm_residual(const int8_t* a, const float* a_scale, const int8_t* w,
                                     const float* w_scale, const float* bias, float* x, uint32_t m,
                                     uint32_t n, uint32_t k, const uint32_t* run_rows,
                                     void* stream) {
    if (!a_scale || !w_scale || !x) return DH_ERR_NULL_POINTER;
    if (n % 256 != 0) return DH_ERR_UNSUPPORTED_SHAPE;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w_scale) |
         reinterpret_cast<uintptr_t>(bias)) & 15u)
        return DH_ERR_ALIGNMENT;
    CUtensorMap ta, tb;
    uint32_t st = make_i8_operand_maps(&ta, &tb, a, k, w, k, m, n, k, 256);
    if (st != DH_OK) return st;
    EpiResidual::Params p{a_scale, w_scale, bias, x, n};
    GemmShape shape{m, n, k, run_rows};
    const uint32_t tiles = ((m + 127) / 128) * (n / 256);
    if (launch_gemm_i8<256, EpiResidual>(ta, tb, shape, p, tiles,
                                         static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return DH_ERR_CUDA;
    return DH_OK;
}

extern "C" uint32_t dh_gemm_gelu(const int8_t* a, const float* a_scale, const int8_t* w,
                                 const float* w_scale, const float* bias, void* out, uint32_t m,
                                 uint32_t n, uint32_t k, const uint32_t* run_rows, void* stream) {
    if (!a_scale || !w_scale || !bias || !out) return DH_ERR_NULL_POINTER;
    if (n % 256 != 0) return DH_ERR_UNSUPPORTED_SHAPE;
    if (reinterpret_cast<uintptr_t>(out) & 15u) return DH_ERR_ALIGNMENT;
    CUtensorMap ta, tb;
    uint32_t st = make_i8_operand_maps(&ta, &tb, a, k, w, k, m, n, k, 256);
    if (st != DH_OK) return st;
    EpiGelu::Params p{a_scale, w_scale, bias, static_cast<__nv_bfloat16*>(out), n};
    GemmShape shape{m, n, k, run_rows};
    const uint32_t tiles = ((m + 127) / 128) * (n / 256);
    if (launch_gemm_i8<256, EpiGelu>(ta, tb, shape, p, tiles, static_cast<cudaStream_t>(stream)) !=
        cudaSuccess)
        return DH_ERR_CUDA;
    return DH_OK;
}
