// norm_quant.cu -- HBM-bound row kernels of the DDiT forward:
//   K10 embed_gather       x[r] = embedding[token[r]]                  (mlx_mdlm.py:262-268)
//   K3  ln_smooth_quant    LayerNorm (no affine, eps 1e-5; the adaLN affine is
//                          folded into the next linear, model_specialization.py:10-29)
//                          -> divide by the SmoothQuant scale -> per-token
//                          symmetric int8 + row scale      (fixed_mlp.py:11-35, 82-90)
//   K3' quant_rows_bf16    same quantiser for bf16 activations (attention
//                          output, GELU output)
// The quantiser (row_quant.cuh) divides as the reference does and gives the
// same bytes and row scale as fixed_mlp._quantize_symmetric.
// One warp per row; rows are read once (float4 / 16-byte vector loads) and
// kept in registers between the statistics and the quantisation pass.
#include <cuda_bf16.h>

#include "row_quant.cuh"

namespace dh {
namespace {

constexpr uint32_t kD = 768;
// Rows per CTA (one warp each).  Small CTAs measured faster on these
// HBM-bound kernels (finer-grained scheduling of the last waves): 2 rows for
// the 768-wide kernels (LN 30.7 -> 28.9 us, requant 20.8 -> 18.7 us at 32,768
// rows) and 1 for the two-pass 3072-wide requant (61.0 -> 57.0 us).
constexpr uint32_t kRowWarps = 2;
constexpr uint32_t kWideRowWarps = 1;

// Rows processed by a launch: all `rows`, or the first *run_rows of them
// when the caller gives that device word (0 = none: a captured graph skips
// the work of a transition that needs no forward).
DH_DEVINL uint32_t live_rows(uint32_t rows, const uint32_t* run_rows) {
    return run_rows ? min(rows, *run_rows) : rows;
}

// x[r] = embedding[tokens[src(r)]]: src(r) = r, or, with a sequence list,
// the position r % positions of sequence seq_list[r / positions] (the
// forward over the sequences that need one, packed together).
__global__ void __launch_bounds__(kRowWarps * 32)
embed_gather_kernel(const int32_t* __restrict__ tokens, const float* __restrict__ embed,
                    float* __restrict__ x, uint32_t rows, uint32_t vocab,
                    const uint32_t* __restrict__ run_flag, const uint32_t* __restrict__ seq_list,
                    uint32_t positions) {
    const uint32_t r = blockIdx.x * kRowWarps + warp_id();
    if (r >= live_rows(rows, run_flag)) return;
    const uint32_t tr = seq_list ? seq_list[r / positions] * positions + r % positions : r;
    uint32_t t = static_cast<uint32_t>(tokens[tr]);
    if (t >= vocab) t = vocab - 1;
    const float4* src = reinterpret_cast<const float4*>(embed + static_cast<uint64_t>(t) * kD);
    float4* dst = reinterpret_cast<float4*>(x + static_cast<uint64_t>(r) * kD);
#pragma unroll
    for (uint32_t j = 0; j < kD / 128; ++j) dst[lane_id() + 32 * j] = __ldg(src + lane_id() + 32 * j);
}

// LayerNorm + SmoothQuant + int8.  Optional row gather: output row i reads
// input row rows_index[i] (used to project only selected rows).
__global__ void __launch_bounds__(kRowWarps * 32)
ln_quant_kernel(const float* __restrict__ x, const float* __restrict__ smooth,
                const float* __restrict__ inv_smooth, int8_t* __restrict__ out, float* __restrict__ scale, uint32_t rows,
                const uint32_t* __restrict__ rows_index, const uint32_t* __restrict__ rows_count,
                const uint32_t* __restrict__ run_flag, const uint32_t* __restrict__ seq_list,
                uint32_t positions) {
    const uint32_t i = blockIdx.x * kRowWarps + warp_id();
    uint32_t n = live_rows(rows, run_flag);
    if (rows_count) n = min(n, *rows_count);
    if (i >= n) return;
    const uint32_t r = rows_index ? rows_index[i] : i;
    // output row: i, or scattered to the sequence's own rows
    const uint32_t o = seq_list ? seq_list[i / positions] * positions + i % positions : i;
    ln_smooth_quant_row(x + static_cast<uint64_t>(r) * kD, smooth, inv_smooth, out + static_cast<uint64_t>(o) * kD,
                        scale + o, lane_id());
}

// bf16 rows of C = 768 or 3072 columns -> per-token int8 + row scale.  The
// SmoothQuant division is already applied by the producer (the attention
// output inherits it from V, the GELU output from the MLP-up epilogue), or
// here when `smooth` is given: then a = fp32(x) / s is kept in fp32 registers
// (never rounded back to bf16) for the amax and the quantisation, as the
// reference divides fp32 activations.  Without it the row amax is taken in
// packed bf16x2 (exact) and the quantisation in fp32.
template <uint32_t C, bool kSmooth>
__global__ void __launch_bounds__(kRowWarps * 32)
quant_rows_bf16_kernel(const __nv_bfloat16* __restrict__ in, const float* __restrict__ smooth,
                       const float* __restrict__ inv_smooth, int8_t* __restrict__ out, float* __restrict__ scale, uint32_t rows,
                       const uint32_t* __restrict__ run_flag) {
    const uint32_t r = blockIdx.x * kRowWarps + warp_id();
    if (r >= live_rows(rows, run_flag)) return;
    constexpr uint32_t kVec = C / 256;  // 8-element (16-byte) vectors per lane
    const uint4* src = reinterpret_cast<const uint4*>(in + static_cast<uint64_t>(r) * C);
    uint4 raw[kVec];
#pragma unroll
    for (uint32_t j = 0; j < kVec; ++j) raw[j] = __ldcs(src + lane_id() + 32 * j);
    uint2* dst = reinterpret_cast<uint2*>(out + static_cast<uint64_t>(r) * C);
    if (kSmooth) {
        const float4* sm = reinterpret_cast<const float4*>(smooth);
        float a[kVec][8];
        float amax = 0.f;
#pragma unroll
        for (uint32_t j = 0; j < kVec; ++j) {
            const uint32_t c4 = (lane_id() + 32 * j) * 2;
            const float4 s0 = __ldg(sm + c4), s1 = __ldg(sm + c4 + 1);
            const float4* iv = reinterpret_cast<const float4*>(inv_smooth);
            const float4 r0 = column_reciprocals(s0, iv, c4), r1 = column_reciprocals(s1, iv, c4 + 1);
            const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
            const float rv[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[j]);
#pragma unroll
            for (uint32_t e = 0; e < 4; ++e) {
                const float2 f = __bfloat1622float2(h[e]);
                a[j][2 * e] = divide(f.x, {sv[2 * e], rv[2 * e]});
                a[j][2 * e + 1] = divide(f.y, {sv[2 * e + 1], rv[2 * e + 1]});
                amax = fmaxf(amax, fmaxf(fabsf(a[j][2 * e]), fabsf(a[j][2 * e + 1])));
            }
        }
        const float sc = row_scale(warp_max_f32(amax));
        const Divisor d = make_divisor(sc);
#pragma unroll
        for (uint32_t j = 0; j < kVec; ++j)
            dst[lane_id() + 32 * j] =
                make_uint2(pack4_i8(q8_div_bits(a[j][0], d), q8_div_bits(a[j][1], d), q8_div_bits(a[j][2], d),
                                    q8_div_bits(a[j][3], d)),
                           pack4_i8(q8_div_bits(a[j][4], d), q8_div_bits(a[j][5], d), q8_div_bits(a[j][6], d),
                                    q8_div_bits(a[j][7], d)));
        if (lane_id() == 0) scale[r] = sc;
        return;
    }
    __nv_bfloat162 m2 = __float2bfloat162_rn(0.f);
#pragma unroll
    for (uint32_t j = 0; j < kVec; ++j) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[j]);
#pragma unroll
        for (uint32_t e = 0; e < 4; ++e) m2 = __hmax2(m2, __habs2(h[e]));
    }
    const float sc = row_scale(warp_max_f32(fmaxf(__low2float(m2), __high2float(m2))));
    const Divisor d = make_divisor(sc);
#pragma unroll
    for (uint32_t j = 0; j < kVec; ++j) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw[j]);
        uint32_t packed[2];
#pragma unroll
        for (uint32_t e = 0; e < 4; e += 2) {
            const float2 f0 = __bfloat1622float2(h[e]), f1 = __bfloat1622float2(h[e + 1]);
            packed[e >> 1] = pack4_i8(q8_div_bits(f0.x, d), q8_div_bits(f0.y, d), q8_div_bits(f1.x, d),
                                      q8_div_bits(f1.y, d));
        }
        dst[lane_id() + 32 * j] = make_uint2(packed[0], packed[1]);
    }
    if (lane_id() == 0) scale[r] = sc;
}

// Wide rows (3072): two streaming passes instead of holding the row in
// registers -- pass 1 takes the row amax, pass 2 re-reads the row (L1 / L2
// resident, just read by this warp) and quantises.  Few registers, so many
// rows are in flight per SM.
__global__ void __launch_bounds__(kWideRowWarps * 32)
quant_rows_bf16_wide_kernel(const __nv_bfloat16* __restrict__ in, int8_t* __restrict__ out,
                            float* __restrict__ scale, uint32_t rows, uint32_t cols,
                            const uint32_t* __restrict__ run_flag) {
    const uint32_t r = blockIdx.x * kWideRowWarps + warp_id();
    if (r >= live_rows(rows, run_flag)) return;
    const uint32_t nvec = cols / 8;
    const uint4* src = reinterpret_cast<const uint4*>(in + static_cast<uint64_t>(r) * cols);
    __nv_bfloat162 m2 = __float2bfloat162_rn(0.f);
#pragma unroll 4
    for (uint32_t j = lane_id(); j < nvec; j += 32) {
        const uint4 raw = src[j];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (uint32_t e = 0; e < 4; ++e) m2 = __hmax2(m2, __habs2(h[e]));
    }
    const float sc = row_scale(warp_max_f32(fmaxf(__low2float(m2), __high2float(m2))));
    const Divisor d = make_divisor(sc);
    uint2* dst = reinterpret_cast<uint2*>(out + static_cast<uint64_t>(r) * cols);
#pragma unroll 4
    for (uint32_t j = lane_id(); j < nvec; j += 32) {
        const uint4 raw = __ldcs(src + j);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
        uint32_t packed[2];
#pragma unroll
        for (uint32_t e = 0; e < 4; e += 2) {
            const float2 f0 = __bfloat1622float2(h[e]), f1 = __bfloat1622float2(h[e + 1]);
            packed[e >> 1] = pack4_i8(q8_div_bits(f0.x, d), q8_div_bits(f0.y, d), q8_div_bits(f1.x, d),
                                      q8_div_bits(f1.y, d));
        }
        dst[j] = make_uint2(packed[0], packed[1]);
    }
    if (lane_id() == 0) scale[r] = sc;
}

// bf16 rows whose amax the producer already merged into row_amax (bits of a
// non-negative float, see dh_gemm_gelu): one streaming pass quantises the
// row with scale = amax / 127, then the word is cleared for the producer's
// next launch.  Same bytes and scales as quant_rows_bf16_wide_kernel.
__global__ void __launch_bounds__(kRowWarps * 32)
quant_rows_bf16_amax_kernel(const __nv_bfloat16* __restrict__ in, uint32_t* __restrict__ row_amax,
                            int8_t* __restrict__ out, float* __restrict__ scale, uint32_t rows, uint32_t cols,
                            const uint32_t* __restrict__ run_flag) {
    const uint32_t r = blockIdx.x * kRowWarps + warp_id();
    if (r >= live_rows(rows, run_flag)) return;
    const float sc = row_scale(__uint_as_float(row_amax[r]));
    const Divisor d = make_divisor(sc);
    const uint32_t nvec = cols / 8;
    const uint4* src = reinterpret_cast<const uint4*>(in + static_cast<uint64_t>(r) * cols);
    uint2* dst = reinterpret_cast<uint2*>(out + static_cast<uint64_t>(r) * cols);
#pragma unroll 4
    for (uint32_t j = lane_id(); j < nvec; j += 32) {
        const uint4 raw = __ldcs(src + j);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
        uint32_t packed[2];
#pragma unroll
        for (uint32_t e = 0; e < 4; e += 2) {
            const float2 f0 = __bfloat1622float2(h[e]), f1 = __bfloat1622float2(h[e + 1]);
            packed[e >> 1] = pack4_i8(q8_div_bits(f0.x, d), q8_div_bits(f0.y, d), q8_div_bits(f1.x, d),
                                      q8_div_bits(f1.y, d));
        }
        dst[j] = make_uint2(packed[0], packed[1]);
    }
    __syncwarp();
    if (lane_id() == 0) {
        scale[r] = sc;
        row_amax[r] = 0u;
    }
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" {

uint32_t dh_embed_gather(const int32_t* tokens, const float* embedding, float* x, uint32_t rows,
                         uint32_t vocabulary_size, const uint32_t* run_flag, void* stream) {
    if (!tokens || !embedding || !x) return DH_ERR_NULL_POINTER;
    if (rows == 0) return DH_OK;
    if ((reinterpret_cast<uintptr_t>(embedding) | reinterpret_cast<uintptr_t>(x)) & 15u)
        return DH_ERR_ALIGNMENT;
    embed_gather_kernel<<<(rows + kRowWarps - 1) / kRowWarps, kRowWarps * 32, 0,
                          static_cast<cudaStream_t>(stream)>>>(tokens, embedding, x, rows,
                                                               vocabulary_size, run_flag, nullptr, 1);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_embed_gather_seqs(const int32_t* tokens, const uint32_t* seq_list, uint32_t positions,
                              const float* embedding, float* x, uint32_t rows, uint32_t vocabulary_size,
                              const uint32_t* run_rows, void* stream) {
    if (!tokens || !seq_list || !embedding || !x) return DH_ERR_NULL_POINTER;
    if (rows == 0) return DH_OK;
    if (positions == 0) return DH_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(embedding) | reinterpret_cast<uintptr_t>(x)) & 15u)
        return DH_ERR_ALIGNMENT;
    embed_gather_kernel<<<(rows + kRowWarps - 1) / kRowWarps, kRowWarps * 32, 0,
                          static_cast<cudaStream_t>(stream)>>>(tokens, embedding, x, rows, vocabulary_size,
                                                               run_rows, seq_list, positions);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_ln_smooth_quant(const float* x, const float* smooth, const float* inv_smooth, int8_t* out, float* scale,
                            uint32_t rows, const uint32_t* rows_index, const uint32_t* rows_count,
                            const uint32_t* run_flag, void* stream) {
    if (!x || !smooth || !out || !scale) return DH_ERR_NULL_POINTER;
    if (rows == 0) return DH_OK;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(smooth) | reinterpret_cast<uintptr_t>(inv_smooth) |
         reinterpret_cast<uintptr_t>(out)) & 15u)
        return DH_ERR_ALIGNMENT;
    ln_quant_kernel<<<(rows + kRowWarps - 1) / kRowWarps, kRowWarps * 32, 0,
                      static_cast<cudaStream_t>(stream)>>>(x, smooth, inv_smooth, out, scale, rows,
                                                           rows_index, rows_count, run_flag, nullptr, 1);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_ln_smooth_quant_scatter(const float* x, const float* smooth, const float* inv_smooth, int8_t* out,
                                    float* scale, uint32_t rows, const uint32_t* seq_list, uint32_t positions,
                                    const uint32_t* run_rows, void* stream) {
    if (!x || !smooth || !out || !scale || !seq_list) return DH_ERR_NULL_POINTER;
    if (rows == 0) return DH_OK;
    if (positions == 0) return DH_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(smooth) | reinterpret_cast<uintptr_t>(inv_smooth) |
         reinterpret_cast<uintptr_t>(out)) & 15u)
        return DH_ERR_ALIGNMENT;
    ln_quant_kernel<<<(rows + kRowWarps - 1) / kRowWarps, kRowWarps * 32, 0,
                      static_cast<cudaStream_t>(stream)>>>(x, smooth, inv_smooth, out, scale, rows, nullptr,
                                                           nullptr, run_rows, seq_list, positions);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

// dst row i = src row rows_index[i] (768 int8 + its fp32 scale), i < *rows_count.
__global__ void gather_rows_i8_kernel(const int8_t* __restrict__ src, const float* __restrict__ src_scale,
                                      const uint32_t* __restrict__ rows_index, const uint32_t* __restrict__ rows_count,
                                      uint32_t rows, int8_t* __restrict__ dst, float* __restrict__ dst_scale) {
    const uint32_t i = blockIdx.x * (blockDim.x / 32) + warp_id();
    if (i >= min(rows, *rows_count)) return;
    const uint32_t r = rows_index[i];
    const uint2* s = reinterpret_cast<const uint2*>(src + static_cast<uint64_t>(r) * kD);
    uint2* d = reinterpret_cast<uint2*>(dst + static_cast<uint64_t>(i) * kD);
#pragma unroll
    for (uint32_t j = 0; j < kD / 256; ++j) d[lane_id() + 32 * j] = s[lane_id() + 32 * j];
    if (lane_id() == 0) dst_scale[i] = src_scale[r];
}

uint32_t dh_gather_rows_i8(const int8_t* src, const float* src_scale, const uint32_t* rows_index,
                           const uint32_t* rows_count, uint32_t rows, int8_t* dst, float* dst_scale, void* stream) {
    if (!src || !src_scale || !rows_index || !rows_count || !dst || !dst_scale) return DH_ERR_NULL_POINTER;
    if (rows == 0) return DH_OK;
    if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 7u) return DH_ERR_ALIGNMENT;
    gather_rows_i8_kernel<<<(rows + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        src, src_scale, rows_index, rows_count, rows, dst, dst_scale);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

// dst row i = src row rows_index[i]: one warp per row, 16-byte vectors.
__global__ void gather_rows_kernel(const uint4* __restrict__ src, uint32_t row_vecs,
                                   const uint32_t* __restrict__ rows_index, const uint32_t* __restrict__ rows_count,
                                   uint32_t rows, uint4* __restrict__ dst) {
    const uint32_t i = blockIdx.x * (blockDim.x / 32) + warp_id();
    if (i >= min(rows, *rows_count)) return;
    const uint4* s = src + static_cast<uint64_t>(rows_index[i]) * row_vecs;
    uint4* d = dst + static_cast<uint64_t>(i) * row_vecs;
    for (uint32_t j = lane_id(); j < row_vecs; j += 32) d[j] = s[j];
}

uint32_t dh_gather_rows(const void* src, uint32_t row_bytes, const uint32_t* rows_index, const uint32_t* rows_count,
                        uint32_t rows, void* dst, void* stream) {
    if (!src || !rows_index || !rows_count || !dst) return DH_ERR_NULL_POINTER;
    if (rows == 0) return DH_OK;
    if (row_bytes == 0 || row_bytes % 16 != 0) return DH_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) return DH_ERR_ALIGNMENT;
    gather_rows_kernel<<<(rows + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(src), row_bytes / 16, rows_index, rows_count, rows, static_cast<uint4*>(dst));
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_quant_rows_bf16(const void* in, const float* smooth, const float* inv_smooth, int8_t* out, float* scale,
                            uint32_t rows, uint32_t cols, const uint32_t* run_flag, void* stream) {
    if (!in || !out || !scale) return DH_ERR_NULL_POINTER;
    if (rows == 0) return DH_OK;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out) |
         reinterpret_cast<uintptr_t>(smooth) | reinterpret_cast<uintptr_t>(inv_smooth)) & 15u)
        return DH_ERR_ALIGNMENT;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const uint32_t grid = (rows + kRowWarps - 1) / kRowWarps;
    const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(in);
    if (cols == 768 && smooth)
        quant_rows_bf16_kernel<768, true><<<grid, kRowWarps * 32, 0, st>>>(src, smooth, inv_smooth, out, scale, rows,
                                                                           run_flag);
    else if (cols == 768)
        quant_rows_bf16_kernel<768, false><<<grid, kRowWarps * 32, 0, st>>>(src, nullptr, nullptr, out, scale, rows,
                                                                            run_flag);
    else if (cols == 3072 && smooth)
        quant_rows_bf16_kernel<3072, true><<<grid, kRowWarps * 32, 0, st>>>(src, smooth, inv_smooth, out, scale, rows,
                                                                            run_flag);
    else if (cols == 3072)
        quant_rows_bf16_wide_kernel<<<(rows + kWideRowWarps - 1) / kWideRowWarps, kWideRowWarps * 32, 0, st>>>(
            src, out, scale, rows, cols, run_flag);
    else
        return DH_ERR_UNSUPPORTED_SHAPE;
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_quant_rows_bf16_amax(const void* in, uint32_t* row_amax, int8_t* out, float* scale, uint32_t rows,
                                 uint32_t cols, const uint32_t* run_flag, void* stream) {
    if (!in || !row_amax || !out || !scale) return DH_ERR_NULL_POINTER;
    if (rows == 0) return DH_OK;
    if (cols == 0 || cols % 256 != 0) return DH_ERR_UNSUPPORTED_SHAPE;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15u) return DH_ERR_ALIGNMENT;
    quant_rows_bf16_amax_kernel<<<(rows + kRowWarps - 1) / kRowWarps, kRowWarps * 32, 0,
                                  static_cast<cudaStream_t>(stream)>>>(static_cast<const __nv_bfloat16*>(in),
                                                                       row_amax, out, scale, rows, cols, run_flag);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

}  // extern "C"
