// final_layer.cu -- the prologue of the output head when the conditioning
// varies per sequence (the final layer of the DDiT, mlx_mdlm._FinalLayer,
// mlx_mdlm.py:456-498, unfolded):
//
//   dh_adaln_modulation       [shift | scale] = cond . W_ada^T + b_ada
//                             (adaLN_modulation, Linear(C -> 2 d)), per sequence;
//   dh_ln_modulate_quant_bf16 per selected row: LayerNorm (eps 1e-5, weight)
//                             of the bf16 hidden row, modulate
//                             h = n (1 + scale_b) + shift_b, then the
//                             per-token symmetric int8 of
//                             fixed_mlp._quantize_symmetric (fixed_mlp.py:11-35)
//                             -- the head's int8 input and row scale.
// One warp per row, the row in registers; HBM-bound.  Multiplications and
// additions are rounded separately, in the order the reference writes them.
#include <cuda_bf16.h>

#include "dh_common.cuh"

namespace dh {
namespace {

constexpr uint32_t kD = 768;
constexpr uint32_t kRowWarps = 2;

// out[b, n] = bias[n] + sum_c cond[b, c] W[n, c], c in order (fp32).
__global__ void __launch_bounds__(256)
adaln_kernel(const float* __restrict__ cond, const float* __restrict__ w, const float* __restrict__ bias,
             float* __restrict__ out, uint32_t C, uint32_t N) {
    extern __shared__ float cs[];
    const uint32_t b = blockIdx.y;
    for (uint32_t c = threadIdx.x; c < C; c += blockDim.x) cs[c] = cond[static_cast<uint64_t>(b) * C + c];
    __syncthreads();
    const uint32_t n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    const float* wr = w + static_cast<uint64_t>(n) * C;
    float acc = 0.f;
    for (uint32_t c = 0; c < C; ++c) acc = __fmaf_rn(cs[c], __ldg(wr + c), acc);
    out[static_cast<uint64_t>(b) * N + n] = __fadd_rn(acc, bias ? __ldg(bias + n) : 0.f);
}

// Markstein-corrected division by a row constant (see norm_quant.cu).
DH_DEVINL float div_rn(float a, float b, float r) {
    const float q0 = __fmul_rn(a, r);
    return __fmaf_rn(__fmaf_rn(-q0, b, a), r, q0);
}

DH_DEVINL uint32_t q8_bits(float a, float sc, float rsc) {
    const float q = fminf(fmaxf(div_rn(a, sc, rsc), -127.0f), 127.0f);
    return __float_as_uint(__fadd_rn(q, 12582912.0f));  // round half to even (1.5 * 2^23 shifter)
}

DH_DEVINL uint32_t pack4(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

__global__ void __launch_bounds__(kRowWarps * 32)
ln_modulate_quant_kernel(const __nv_bfloat16* __restrict__ hidden, const float* __restrict__ ln_weight,
                         const float* __restrict__ modulation, uint32_t rows_per_sequence,
                         const uint32_t* __restrict__ rows_index, const uint32_t* __restrict__ rows_count,
                         uint32_t rows, int8_t* __restrict__ out, float* __restrict__ scale) {
    const uint32_t i = blockIdx.x * kRowWarps + warp_id();
    const uint32_t n = rows_count ? min(rows, *rows_count) : rows;
    if (i >= n) return;
    const uint32_t r = rows_index ? rows_index[i] : i;
    const uint32_t b = r / rows_per_sequence;
    // lane holds columns 8 (lane + 32 j) .. +7, j < 3
    const uint4* src = reinterpret_cast<const uint4*>(hidden + static_cast<uint64_t>(r) * kD);
    float v[3][8];
    float sum = 0.f;
#pragma unroll
    for (uint32_t j = 0; j < 3; ++j) {
        const uint4 raw = src[lane_id() + 32 * j];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
        for (uint32_t e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h[e]);
            v[j][2 * e] = f.x;
            v[j][2 * e + 1] = f.y;
            sum += f.x + f.y;
        }
    }
    const float mean = warp_sum_f32(sum) * (1.0f / kD);
    float sq = 0.f;
#pragma unroll
    for (uint32_t j = 0; j < 3; ++j)
#pragma unroll
        for (uint32_t e = 0; e < 8; ++e) {
            const float d = v[j][e] - mean;
            sq += d * d;
        }
    const float rstd = rsqrtf(warp_sum_f32(sq) * (1.0f / kD) + 1e-5f);
    const float* shift = modulation + static_cast<uint64_t>(b) * 2 * kD;
    const float* scl = shift + kD;
    float amax = 0.f;
#pragma unroll
    for (uint32_t j = 0; j < 3; ++j) {
        const uint32_t c0 = 8 * (lane_id() + 32 * j);
        const float4 sh0 = __ldg(reinterpret_cast<const float4*>(shift + c0));
        const float4 sh1 = __ldg(reinterpret_cast<const float4*>(shift + c0 + 4));
        const float4 sc0 = __ldg(reinterpret_cast<const float4*>(scl + c0));
        const float4 sc1 = __ldg(reinterpret_cast<const float4*>(scl + c0 + 4));
        const float shv[8] = {sh0.x, sh0.y, sh0.z, sh0.w, sh1.x, sh1.y, sh1.z, sh1.w};
        const float scv[8] = {sc0.x, sc0.y, sc0.z, sc0.w, sc1.x, sc1.y, sc1.z, sc1.w};
        float wv[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
        if (ln_weight) {
            const float4 w0 = __ldg(reinterpret_cast<const float4*>(ln_weight + c0));
            const float4 w1 = __ldg(reinterpret_cast<const float4*>(ln_weight + c0 + 4));
            wv[0] = w0.x, wv[1] = w0.y, wv[2] = w0.z, wv[3] = w0.w;
            wv[4] = w1.x, wv[5] = w1.y, wv[6] = w1.z, wv[7] = w1.w;
        }
#pragma unroll
        for (uint32_t e = 0; e < 8; ++e) {
            const float nrm = __fmul_rn(__fmul_rn(__fsub_rn(v[j][e], mean), rstd), wv[e]);
            const float h = __fadd_rn(__fmul_rn(nrm, __fadd_rn(1.0f, scv[e])), shv[e]);
            v[j][e] = h;
            amax = fmaxf(amax, fabsf(h));
        }
    }
    amax = warp_max_f32(amax);
    const float sc = amax > 0.f ? __fdiv_rn(amax, 127.0f) : 1.0f;
    const float rsc = __frcp_rn(sc);
    uint2* dst = reinterpret_cast<uint2*>(out + static_cast<uint64_t>(i) * kD);
#pragma unroll
    for (uint32_t j = 0; j < 3; ++j)
        dst[lane_id() + 32 * j] =
            make_uint2(pack4(q8_bits(v[j][0], sc, rsc), q8_bits(v[j][1], sc, rsc), q8_bits(v[j][2], sc, rsc),
                             q8_bits(v[j][3], sc, rsc)),
                       pack4(q8_bits(v[j][4], sc, rsc), q8_bits(v[j][5], sc, rsc), q8_bits(v[j][6], sc, rsc),
                             q8_bits(v[j][7], sc, rsc)));
    if (lane_id() == 0) scale[i] = sc;
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" {

uint32_t dh_adaln_modulation(const float* cond, const float* weight, const float* bias, float* out,
                             uint32_t sequences, uint32_t condition_size, uint32_t outputs, void* stream) {
    if (!cond || !weight || !out) return DH_ERR_NULL_POINTER;
    if (sequences == 0 || condition_size == 0 || outputs == 0) return DH_ERR_INVALID_ARGUMENT;
    if (condition_size > 8192 || sequences > 65535) return DH_ERR_UNSUPPORTED_SHAPE;
    dim3 grid((outputs + 255) / 256, sequences);
    adaln_kernel<<<grid, 256, condition_size * sizeof(float), static_cast<cudaStream_t>(stream)>>>(
        cond, weight, bias, out, condition_size, outputs);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_ln_modulate_quant_bf16(const void* hidden, const float* ln_weight, const float* modulation,
                                   uint32_t rows_per_sequence, const uint32_t* rows_index,
                                   const uint32_t* rows_count, uint32_t rows, int8_t* out, float* scale,
                                   void* stream) {
    if (!hidden || !modulation || !out || !scale) return DH_ERR_NULL_POINTER;
    if (rows == 0) return DH_OK;
    if (rows_per_sequence == 0) return DH_ERR_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(hidden) | reinterpret_cast<uintptr_t>(modulation) |
         reinterpret_cast<uintptr_t>(ln_weight) | reinterpret_cast<uintptr_t>(out)) & 15u)
        return DH_ERR_ALIGNMENT;
    ln_modulate_quant_kernel<<<(rows + kRowWarps - 1) / kRowWarps, kRowWarps * 32, 0,
                               static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(hidden), ln_weight, modulation, rows_per_sequence, rows_index, rows_count,
        rows, out, scale);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

}  // extern "C"
