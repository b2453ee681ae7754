// row_quant.cuh -- the per-token int8 quantiser of the W8A8 linears and the
// warp-per-row LayerNorm + SmoothQuant + int8 of a 768-wide residual row.
//
// The quantiser divides as the reference does (fixed_mlp.py:11-35): a = x / s,
// scale = amax / 127, q = round_half_even(a / scale) clamped to +-127, every
// quotient the IEEE-rounded fp32 quotient, so the same fp32 input row gives
// the same bytes and row scale as fixed_mlp._quantize_symmetric.  Divisions by
// a value used many times (the row scale, the per-column SmoothQuant scale)
// multiply by the rounded reciprocal and correct the product once by its
// exact residual, which yields the rounded quotient at the cost of three
// FMA-pipe operations (see Divisor).
#pragma once

#include "dh_common.cuh"

namespace dh {

// Round to nearest even by the 1.5 * 2^23 shifter: for |v| <= 2^22 the low
// bits of the sum's encoding are rint(v) in two's complement, so the low byte
// is the int8 value when |v| <= 127.  One FADD instead of a float-to-integer
// conversion on the (quarter-rate) XU pipe; the result equals rintf / cvt.rni.
DH_DEVINL uint32_t rint_bits(float v) { return __float_as_uint(__fadd_rn(v, 12582912.0f)); }

// Division by b > 0 with its reciprocal r = RN(1 / b) precomputed: the
// estimate q0 = RN(a r) is within an ulp of a / b, its residual a - q0 b is
// exact in one FMA, and RN(q0 + (a - q0 b) r) is the correctly rounded
// quotient (Markstein's correction step for a correctly rounded reciprocal;
// no overflow or underflow at these magnitudes).  Checked against IEEE
// division on every quotient of the quantiser tests.
struct Divisor {
    float b, r;
};
DH_DEVINL Divisor make_divisor(float b) { return {b, __frcp_rn(b)}; }
DH_DEVINL float divide(float a, const Divisor& d) {
    const float q0 = __fmul_rn(a, d.r);
    return __fmaf_rn(__fmaf_rn(-q0, d.b, a), d.r, q0);
}

// int8 of round_half_even(a / scale) clamped to +-127
// (fixed_mlp._quantize_symmetric, fixed_mlp.py:24-35: torch.round(x /
// scale).clamp(-127, 127); clamping the quotient first gives the same byte,
// 127 being an integer).
DH_DEVINL uint32_t q8_div_bits(float a, const Divisor& scale) {
    return rint_bits(fminf(fmaxf(divide(a, scale), -127.0f), 127.0f));
}

// Row scale of the reference: amax / 127 (fp32 division), 1 for an all-zero row.
DH_DEVINL float row_scale(float amax) { return amax > 0.f ? __fdiv_rn(amax, 127.0f) : 1.0f; }

// Per-column SmoothQuant reciprocals: the caller's RN(1 / s), else computed.
DH_DEVINL float4 column_reciprocals(float4 s, const float4* inv, uint32_t i4) {
    if (inv) return __ldg(inv + i4);
    return make_float4(__frcp_rn(s.x), __frcp_rn(s.y), __frcp_rn(s.z), __frcp_rn(s.w));
}

// four int8 (low bytes of a, b, c, d) into one word, a lowest
DH_DEVINL uint32_t pack4_i8(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

constexpr uint32_t kLnCols = 768;

// One warp: LayerNorm (no affine, eps 1e-5; the adaLN affine is folded into
// the next linear, model_specialization.py:10-29) of a 768-wide fp32 row,
// divided by the SmoothQuant scale, per-token int8 into `dst_row` and the row
// scale into *scale.  The row is read once (16-byte loads) and kept in
// registers between the statistics and the quantisation.
constexpr uint32_t kLnVec = kLnCols / 128;  // float4 per lane

DH_DEVINL void ln_smooth_quant_row(const float* __restrict__ src_row, const float* __restrict__ smooth,
                                   const float* __restrict__ inv_smooth, int8_t* __restrict__ dst_row,
                                   float* __restrict__ scale, uint32_t lane) {
    const float4* src = reinterpret_cast<const float4*>(src_row);
    float4 v[kLnVec];
    float sum = 0.f;
#pragma unroll
    for (uint32_t j = 0; j < kLnVec; ++j) {
        v[j] = src[lane + 32 * j];
        sum += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    }
    const float mean = warp_sum_f32(sum) * (1.0f / kLnCols);
    float sq = 0.f;
#pragma unroll
    for (uint32_t j = 0; j < kLnVec; ++j) {
        const float a = v[j].x - mean, b = v[j].y - mean, c = v[j].z - mean, d = v[j].w - mean;
        sq += (a * a + b * b) + (c * c + d * d);
    }
    const float var = warp_sum_f32(sq) * (1.0f / kLnCols);
    const float rstd = rsqrtf(var + 1e-5f);
    const float4* sm = reinterpret_cast<const float4*>(smooth);
    float amax = 0.f;
#pragma unroll
    for (uint32_t j = 0; j < kLnVec; ++j) {
        const uint32_t i4 = lane + 32 * j;
        const float4 s = __ldg(sm + i4);
        const float4 rs = column_reciprocals(s, reinterpret_cast<const float4*>(inv_smooth), i4);
        v[j].x = divide((v[j].x - mean) * rstd, {s.x, rs.x});
        v[j].y = divide((v[j].y - mean) * rstd, {s.y, rs.y});
        v[j].z = divide((v[j].z - mean) * rstd, {s.z, rs.z});
        v[j].w = divide((v[j].w - mean) * rstd, {s.w, rs.w});
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w))));
    }
    amax = warp_max_f32(amax);
    const float sc = row_scale(amax);
    const Divisor dsc = make_divisor(sc);
    uint32_t* dst = reinterpret_cast<uint32_t*>(dst_row);
#pragma unroll
    for (uint32_t j = 0; j < kLnVec; ++j)
        dst[lane + 32 * j] = pack4_i8(q8_div_bits(v[j].x, dsc), q8_div_bits(v[j].y, dsc),
                                      q8_div_bits(v[j].z, dsc), q8_div_bits(v[j].w, dsc));
    if (lane == 0) *scale = sc;
}

}  // namespace dh
