// fixed_point.cu -- the RTL fixed-point stages of the DDiT block, bit-exact
// with the reference's integer contracts:
//
//   K11 LayerNorm      Q13.10 (24-bit) -> Q5.12 (18-bit)    fixed_norm.py:13-104
//   K12 rotary          Q5.12 x Q1.15 -> Q5.12               fixed_attention.py:24-113
//   K13 attention       Q7.10 scores, Q0.16 LUT softmax,     fixed_attention.py:174-298
//                       Q5.12 output
//   K14 wide linear     int64 accumulators of 18-bit          fixed_attention.py:301-494
//                       activations x 16-bit weights, 64-bit
//                       multiplier, symmetric rounding shift,
//                       bias, saturation
//   K15 packed int8     requantised Q / K / V and               attention_int8.py:20-315
//       attention       probabilities, Q28 score rescale
//
// All arithmetic is integer (int64 where the reference's torch int64
// tensors are), except the float -> fixed conversions, which round
// half-to-even like torch.round.  These are validation-scale stages (one
// 64-token canvas per call in the reference), so the kernels favour exact
// integer arithmetic on the CUDA cores over the tensor engine: the operand
// widths (18 x 16 bits) exceed int8.
#include "dh_common.cuh"

#include <algorithm>
#include <climits>
#include <cstdint>

namespace dh {
namespace {

DH_DEVINL long long sym_round_shift(long long v, uint32_t s) {
    const long long mag = ((v < 0 ? -v : v) + (1ll << (s - 1))) >> s;
    return v < 0 ? -mag : mag;
}

DH_DEVINL long long clampll(long long v, long long lo, long long hi) { return v < lo ? lo : (v > hi ? hi : v); }

// floor(sqrt(x)) for x < 2^62, exact: double estimate, then integer fix-up.
DH_DEVINL unsigned long long isqrt_u64(unsigned long long x) {
    unsigned long long r = static_cast<unsigned long long>(sqrt(static_cast<double>(x)));
    for (int i = 0; i < 4 && r * r > x; ++i) --r;
    for (int i = 0; i < 4 && (r + 1) * (r + 1) <= x; ++i) ++r;
    return r;
}

template <typename T>
DH_DEVINL T block_sum(T v, T* scratch) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    __syncthreads();
    if (lane_id() == 0) scratch[warp_id()] = v;
    __syncthreads();
    T t = 0;
    for (uint32_t w = 0; w < blockDim.x / 32; ++w) t += scratch[w];
    return t;
}

DH_DEVINL long long block_max_ll(long long v, long long* scratch) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    __syncthreads();
    if (lane_id() == 0) scratch[warp_id()] = v;
    __syncthreads();
    long long t = LLONG_MIN;
    for (uint32_t w = 0; w < blockDim.x / 32; ++w) t = max(t, scratch[w]);
    return t;
}

struct LnArgs {
    const float* in;
    uint32_t rows, cols;
    uint32_t in_frac, out_frac, inv_frac, sqrt_extra;
    long long eps_q;
    int32_t* out;
    long long* row_stats;  // [rows][5]: mean, variance, inverse, radicand << 2*sqrt_extra, saturated inputs
};

// One CTA per row.
__global__ void __launch_bounds__(256) fixed_layer_norm_kernel(LnArgs a) {
    __shared__ long long scratch[32];
    const uint32_t row = blockIdx.x;
    const float* x = a.in + static_cast<uint64_t>(row) * a.cols;
    const long long in_lo = -(1ll << 23), in_hi = (1ll << 23) - 1;
    long long s = 0, ss = 0, sat = 0;
    for (uint32_t c = threadIdx.x; c < a.cols; c += blockDim.x) {
        const long long u = __double2ll_rn(static_cast<double>(x[c]) * static_cast<double>(1ll << a.in_frac));
        sat += (u < in_lo || u > in_hi) ? 1 : 0;
        const long long q = clampll(u, in_lo, in_hi);
        s += q;
        ss += q * q;
    }
    s = block_sum(s, scratch);
    ss = block_sum(ss, scratch);
    sat = block_sum(sat, scratch);
    const long long C = a.cols;
    const long long mean = s < 0 ? -((-s + C / 2) / C) : (s + C / 2) / C;
    long long var = (ss + C / 2) / C - mean * mean;
    var = var < 0 ? 0 : var;
    const unsigned long long rad = static_cast<unsigned long long>(var + a.eps_q) << (2 * a.sqrt_extra);
    const long long root = static_cast<long long>(isqrt_u64(rad));
    const long long numer = 1ll << (a.inv_frac + a.in_frac + a.sqrt_extra);
    const long long inv = root > 0 ? (numer + root / 2) / root : 0;
    const uint32_t shift = a.inv_frac + a.in_frac - a.out_frac;
    for (uint32_t c = threadIdx.x; c < a.cols; c += blockDim.x) {
        const long long u = __double2ll_rn(static_cast<double>(x[c]) * static_cast<double>(1ll << a.in_frac));
        const long long q = clampll(u, in_lo, in_hi);
        const long long o = clampll(sym_round_shift((q - mean) * inv, shift), -(1ll << 17), (1ll << 17) - 1);
        a.out[static_cast<uint64_t>(row) * a.cols + c] = static_cast<int32_t>(o);
    }
    if (threadIdx.x == 0 && a.row_stats) {
        long long* st = a.row_stats + static_cast<uint64_t>(row) * 5;
        st[0] = mean;
        st[1] = var;
        st[2] = inv;
        st[3] = static_cast<long long>(rad);
        st[4] = sat;
    }
}

// qkv fp32 [T, 3, H, 64] -> qkv_q12 [T, 3, H, 64] (clamped Q5.12), rotated
// q / k Q5.12 [T, H, 64].  stats: [q/k saturated inputs, v saturated inputs,
// q min, q max, k min, k max].
__global__ void fixed_rotary_kernel(const float* __restrict__ qkv, const float* __restrict__ cosv,
                                    const float* __restrict__ sinv, uint32_t T, uint32_t H,
                                    int32_t* __restrict__ qkv_q12, int32_t* __restrict__ q_rot,
                                    int32_t* __restrict__ k_rot, long long* __restrict__ stats) {
    const long long vlo = -(1ll << 17), vhi = (1ll << 17) - 1;
    const uint64_t pairs = static_cast<uint64_t>(T) * 3 * H * 32;
    long long sat_qk = 0, sat_v = 0;
    long long qmin = LLONG_MAX, qmax = LLONG_MIN, kmin = LLONG_MAX, kmax = LLONG_MIN;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < pairs;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t j = static_cast<uint32_t>(i % 32);
        const uint64_t th = i / 32;  // (t, which, h)
        const uint32_t h = static_cast<uint32_t>(th % H);
        const uint32_t which = static_cast<uint32_t>((th / H) % 3);
        const uint32_t t = static_cast<uint32_t>(th / (3ull * H));
        const uint64_t base = ((static_cast<uint64_t>(t) * 3 + which) * H + h) * 64;
        const long long u1 = __double2ll_rn(static_cast<double>(qkv[base + j]) * 4096.0);
        const long long u2 = __double2ll_rn(static_cast<double>(qkv[base + j + 32]) * 4096.0);
        const long long nsat = (u1 < vlo || u1 > vhi ? 1 : 0) + (u2 < vlo || u2 > vhi ? 1 : 0);
        const long long f = clampll(u1, vlo, vhi), s = clampll(u2, vlo, vhi);
        qkv_q12[base + j] = static_cast<int32_t>(f);
        qkv_q12[base + j + 32] = static_cast<int32_t>(s);
        if (which == 2) {
            sat_v += nsat;
            continue;
        }
        sat_qk += nsat;
        const long long c = clampll(__double2ll_rn(static_cast<double>(cosv[t * 32 + j]) * 32768.0),
                                    -(1ll << 15), (1ll << 15) - 1);
        const long long sn = clampll(__double2ll_rn(static_cast<double>(sinv[t * 32 + j]) * 32768.0),
                                     -(1ll << 15), (1ll << 15) - 1);
        const long long o1 = clampll(sym_round_shift(f * c - s * sn, 15), vlo, vhi);
        const long long o2 = clampll(sym_round_shift(s * c + f * sn, 15), vlo, vhi);
        int32_t* dst = which == 0 ? q_rot : k_rot;
        const uint64_t ob = (static_cast<uint64_t>(t) * H + h) * 64;
        dst[ob + j] = static_cast<int32_t>(o1);
        dst[ob + j + 32] = static_cast<int32_t>(o2);
        const long long lo = min(o1, o2), hi = max(o1, o2);
        if (which == 0) {
            qmin = min(qmin, lo);
            qmax = max(qmax, hi);
        } else {
            kmin = min(kmin, lo);
            kmax = max(kmax, hi);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        sat_qk += __shfl_xor_sync(0xFFFFFFFFu, sat_qk, o);
        sat_v += __shfl_xor_sync(0xFFFFFFFFu, sat_v, o);
        qmin = min(qmin, __shfl_xor_sync(0xFFFFFFFFu, qmin, o));
        qmax = max(qmax, __shfl_xor_sync(0xFFFFFFFFu, qmax, o));
        kmin = min(kmin, __shfl_xor_sync(0xFFFFFFFFu, kmin, o));
        kmax = max(kmax, __shfl_xor_sync(0xFFFFFFFFu, kmax, o));
    }
    if (lane_id() == 0 && stats) {
        atomicAdd(reinterpret_cast<unsigned long long*>(stats), static_cast<unsigned long long>(sat_qk));
        atomicAdd(reinterpret_cast<unsigned long long*>(stats + 1), static_cast<unsigned long long>(sat_v));
        atomicMin(stats + 2, qmin);
        atomicMax(stats + 3, qmax);
        atomicMin(stats + 4, kmin);
        atomicMax(stats + 5, kmax);
    }
}

constexpr uint32_t kAttnThreads = 128;
constexpr uint32_t kMaxTokens = 2048;

struct FixedAttnArgs {
    const int32_t* q;  // [T, H, 64] Q5.12 (rotated)
    const int32_t* k;  // [T, H, 64]
    const int32_t* v;  // qkv_q12 [T, 3, H, 64]; value at which = 2
    uint32_t T, H;
    uint32_t address_shift, lut_entries;
    long long cutoff;
    const int32_t* lut;  // Q0.16 exponentials
    int32_t* out;        // [T, H * 64] Q5.12
    int32_t* scores;     // optional [H, T, T] Q7.10
    int32_t* probs;      // optional [H, T, T] Q0.16
    long long* stats;    // [score sat, score min, score max, min delta, max |row sum - 65536|]
};

// One CTA per (head, query row).
__global__ void __launch_bounds__(kAttnThreads) fixed_attention_kernel(FixedAttnArgs a) {
    __shared__ int32_t sc[kMaxTokens];
    __shared__ int32_t qrow[64];
    __shared__ long long scratch[32];
    __shared__ long long part[kAttnThreads];
    const uint32_t h = blockIdx.x % a.H, t = blockIdx.x / a.H;
    const uint32_t T = a.T;
    const long long lo = -(1ll << 17), hi = (1ll << 17) - 1;
    if (threadIdx.x < 64) qrow[threadIdx.x] = a.q[(static_cast<uint64_t>(t) * a.H + h) * 64 + threadIdx.x];
    __syncthreads();
    long long sat = 0, smin = LLONG_MAX, smax = LLONG_MIN, rmax = LLONG_MIN;
    for (uint32_t s = threadIdx.x; s < T; s += blockDim.x) {
        const int32_t* kr = a.k + (static_cast<uint64_t>(s) * a.H + h) * 64;
        long long dot = 0;
#pragma unroll 8
        for (uint32_t d = 0; d < 64; ++d) dot += static_cast<long long>(qrow[d]) * kr[d];
        const long long u = sym_round_shift(dot, 17);
        sat += (u < lo || u > hi) ? 1 : 0;
        const long long sv = clampll(u, lo, hi);
        sc[s] = static_cast<int32_t>(sv);
        smin = min(smin, sv);
        smax = max(smax, sv);
        rmax = max(rmax, sv);
    }
    rmax = block_max_ll(rmax, scratch);
    const long long row_min = -block_max_ll(smin == LLONG_MAX ? LLONG_MIN : -smin, scratch);
    long long esum = 0;
    long long min_delta = 0;
    for (uint32_t s = threadIdx.x; s < T; s += blockDim.x) {
        long long dl = sc[s] - rmax;
        dl = dl < -a.cutoff ? -a.cutoff : dl;
        min_delta = min(min_delta, dl);
        long long addr = (-dl + (1ll << (a.address_shift - 1))) >> a.address_shift;
        addr = addr > a.lut_entries - 1 ? a.lut_entries - 1 : addr;
        const int32_t e = a.lut[addr];
        if (a.scores) a.scores[(static_cast<uint64_t>(h) * T + t) * T + s] = sc[s];
        sc[s] = e;
        esum += e;
    }
    esum = block_sum(esum, scratch);
    const long long recip = ((1ll << 30) + esum / 2) / esum;
    long long psum = 0;
    for (uint32_t s = threadIdx.x; s < T; s += blockDim.x) {
        long long p = (static_cast<long long>(sc[s]) * recip + (1ll << 13)) >> 14;
        p = p > 65535 ? 65535 : p;
        sc[s] = static_cast<int32_t>(p);
        psum += p;
        if (a.probs) a.probs[(static_cast<uint64_t>(h) * T + t) * T + s] = static_cast<int32_t>(p);
    }
    psum = block_sum(psum, scratch);  // ends with a barrier: sc holds the probabilities
    // P . V: thread (d, half) sums keys s = half, half + 2, ...
    const uint32_t d = threadIdx.x & 63u, half = threadIdx.x >> 6;
    long long acc = 0;
    for (uint32_t s = half; s < T; s += 2)
        acc += static_cast<long long>(sc[s]) * a.v[((static_cast<uint64_t>(s) * 3 + 2) * a.H + h) * 64 + d];
    part[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x < 64) {
        const long long tot = part[threadIdx.x] + part[threadIdx.x + 64];
        a.out[static_cast<uint64_t>(t) * a.H * 64 + h * 64 + d] =
            static_cast<int32_t>(clampll(sym_round_shift(tot, 16), lo, hi));
    }
    sat = block_sum(sat, scratch);
    min_delta = -block_max_ll(-min_delta, scratch);
    if (threadIdx.x == 0 && a.stats) {
        atomicAdd(reinterpret_cast<unsigned long long*>(a.stats), static_cast<unsigned long long>(sat));
        atomicMin(a.stats + 1, row_min);
        atomicMax(a.stats + 2, rmax);
        atomicMin(a.stats + 3, min_delta);
        const long long err = psum - 65536;
        atomicMax(a.stats + 4, err < 0 ? -err : err);
    }
}

// ------------------------------------------- K15 packed int8 attention
// The paired-token INT8 attention candidates of attention_int8.py: Q / K
// (rotated Q5.12) and V (Q5.12) requantised to signed integers of
// `levels` magnitude, scores rescaled to Q7.10 by a Q28 multiplier, the K13
// LUT softmax, and probabilities optionally requantised to `p_levels`
// unsigned levels for an integer P . V.
//   qk_mode 0  Q / K not requantised
//           1  calibrated-head: one multiplier per head from a calibration
//              maximum (attention_int8.py:178-190, 212-240)
//           2  dynamic-vector: one maximum per token vector
//              (attention_int8.py:61-90, 191-210)
//   quant_scores  scores from the requantised vectors; else the fixed18
//              scores of K13 (the vectors are still requantised, for the
//              saturation counts the reference reports either way)
// V is requantised when v_levels != 0, and P . V runs on the requantised
// probabilities and values when p_levels != 0 (which needs v_levels).
// Per-head parameters, int64 [H][8]: query / key / value multipliers
// round(levels * 2^frac / maximum), the calibrated score multiplier, the
// output multiplier round(v_max * 2^24 / (v_levels * p_levels)), and the
// query / key / value calibration maxima (saturation counts only).
enum : uint32_t { kPkQMult, kPkKMult, kPkVMult, kPkScoreMult, kPkOutMult, kPkQMax, kPkKMax, kPkVMax, kPkParams };

struct PackedQuantArgs {
    const int32_t* q12;    // [T, H, 64] rotated query, Q5.12
    const int32_t* k12;    // [T, H, 64] rotated key
    const int32_t* qkv12;  // [T, 3, H, 64]; value at which = 2
    uint32_t T, H, qk_mode, qk_levels, qk_frac, v_levels;
    const long long* params;  // [H][kPkParams]
    int32_t* q8;  // [T, H, 64] requantised query (qk_mode != 0)
    int32_t* k8;
    int32_t* v8;  // [T, H, 64] requantised value (v_levels != 0)
    int32_t* q_max;  // [T, H] dynamic vector maxima (qk_mode 2)
    int32_t* k_max;
    long long* head_stats;  // [H][4]: saturated query / key / value inputs, zero probabilities
};

// One warp per (token, head, q | k | v) vector of 64; lane holds elements
// lane and lane + 32.  q = clamp(sym_round_shift(x * multiplier, frac),
// -levels, levels) (attention_int8.py:20-25, 181-190).
__global__ void __launch_bounds__(256) packed_quant_kernel(PackedQuantArgs a) {
    const uint32_t wg = blockIdx.x * (blockDim.x / 32) + warp_id();
    if (wg >= a.T * a.H * 3) return;
    const uint32_t which = wg % 3, row = wg / 3;  // row = t * H + h
    const uint32_t h = row % a.H, t = row / a.H;
    if (which < 2 && a.qk_mode == 0) return;
    if (which == 2 && a.v_levels == 0) return;
    const uint32_t lane = lane_id();
    const int32_t* src = which == 0   ? a.q12 + static_cast<uint64_t>(row) * 64
                         : which == 1 ? a.k12 + static_cast<uint64_t>(row) * 64
                                      : a.qkv12 + ((static_cast<uint64_t>(t) * 3 + 2) * a.H + h) * 64;
    const long long x0 = src[lane], x1 = src[lane + 32];
    const long long* prm = a.params + static_cast<uint64_t>(h) * kPkParams;
    long long mult, levels, sat = 0;
    uint32_t frac;
    if (which == 2 || a.qk_mode == 1) {
        mult = prm[which == 0 ? kPkQMult : which == 1 ? kPkKMult : kPkVMult];
        const long long cal = prm[which == 0 ? kPkQMax : which == 1 ? kPkKMax : kPkVMax];
        frac = which == 2 ? 24u : a.qk_frac;
        levels = which == 2 ? a.v_levels : a.qk_levels;
        sat = ((x0 < 0 ? -x0 : x0) > cal ? 1 : 0) + ((x1 < 0 ? -x1 : x1) > cal ? 1 : 0);
    } else {
        // dynamic: this vector's own maximum (at least 1); the multiplier
        // rounds the correctly rounded double quotient half-to-even like
        // torch.round
        long long m = max(x0 < 0 ? -x0 : x0, x1 < 0 ? -x1 : x1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
        m = m < 1 ? 1 : m;
        frac = a.qk_frac;
        levels = a.qk_levels;
        mult = static_cast<long long>(rint(static_cast<double>(levels << frac) / static_cast<double>(m)));
        if (lane == 0) (which == 0 ? a.q_max : a.k_max)[row] = static_cast<int32_t>(m);
    }
    int32_t* dst = (which == 0 ? a.q8 : which == 1 ? a.k8 : a.v8) + static_cast<uint64_t>(row) * 64;
    dst[lane] = static_cast<int32_t>(clampll(sym_round_shift(x0 * mult, frac), -levels, levels));
    dst[lane + 32] = static_cast<int32_t>(clampll(sym_round_shift(x1 * mult, frac), -levels, levels));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sat += __shfl_xor_sync(0xFFFFFFFFu, sat, o);
    if (lane == 0 && sat && a.head_stats)
        atomicAdd(reinterpret_cast<unsigned long long*>(a.head_stats + h * 4 + which),
                  static_cast<unsigned long long>(sat));
}

struct PackedAttnArgs {
    const int32_t* q;      // [T, H, 64]: requantised (quant_scores) or rotated Q5.12
    const int32_t* k;
    const int32_t* v8;     // [T, H, 64] requantised value (p_levels != 0)
    const int32_t* qkv12;  // [T, 3, H, 64] (p_levels == 0)
    const int32_t* q_max;  // [T, H] (qk_mode 2)
    const int32_t* k_max;
    const long long* params;
    uint32_t T, H, qk_mode, quant_scores, qk_levels, p_levels, sum_correction;
    uint32_t address_shift, lut_entries;
    long long cutoff;
    const int32_t* lut;
    int32_t* out;       // [T, H * 64] Q5.12
    int32_t* scores;    // optional [H, T, T] Q7.10
    int32_t* probs;     // optional [H, T, T] Q0.16
    int32_t* probs_q;   // optional [H, T, T] requantised probabilities (after the sum correction)
    long long* head_stats;
};

// One CTA per (head, query row), like K13.
__global__ void __launch_bounds__(kAttnThreads) packed_attention_kernel(PackedAttnArgs a) {
    __shared__ int32_t sc[kMaxTokens];
    __shared__ int32_t qrow[64];
    __shared__ long long scratch[32];
    __shared__ long long part[kAttnThreads];
    const uint32_t h = blockIdx.x % a.H, t = blockIdx.x / a.H;
    const uint32_t T = a.T;
    const long long lo = -(1ll << 17), hi = (1ll << 17) - 1;
    const long long* prm = a.params + static_cast<uint64_t>(h) * kPkParams;
    if (threadIdx.x < 64) qrow[threadIdx.x] = a.q[(static_cast<uint64_t>(t) * a.H + h) * 64 + threadIdx.x];
    __syncthreads();
    // Q28 score multiplier: per head (calibrated) or per (query, key) pair
    // from the two vector maxima (dynamic; attention_int8.py:81-86, 215-228)
    const double qm =
        a.quant_scores && a.qk_mode == 2 ? static_cast<double>(a.q_max[static_cast<uint64_t>(t) * a.H + h]) : 0.0;
    const double denom = static_cast<double>(static_cast<long long>(a.qk_levels) * a.qk_levels * (1ll << 17));
    long long rmax = LLONG_MIN;
    for (uint32_t s = threadIdx.x; s < T; s += blockDim.x) {
        const int32_t* kr = a.k + (static_cast<uint64_t>(s) * a.H + h) * 64;
        long long dot = 0;
#pragma unroll 8
        for (uint32_t d = 0; d < 64; ++d) dot += static_cast<long long>(qrow[d]) * kr[d];
        long long u;
        if (!a.quant_scores) {
            u = sym_round_shift(dot, 17);
        } else {
            long long m = prm[kPkScoreMult];
            if (a.qk_mode == 2)
                m = static_cast<long long>(
                    rint(qm * static_cast<double>(a.k_max[static_cast<uint64_t>(s) * a.H + h]) * 268435456.0 / denom));
            u = sym_round_shift(dot * m, 28);
        }
        const long long sv = clampll(u, lo, hi);
        sc[s] = static_cast<int32_t>(sv);
        rmax = max(rmax, sv);
    }
    rmax = block_max_ll(rmax, scratch);
    long long esum = 0;
    for (uint32_t s = threadIdx.x; s < T; s += blockDim.x) {
        long long dl = sc[s] - rmax;
        dl = dl < -a.cutoff ? -a.cutoff : dl;
        long long addr = (-dl + (1ll << (a.address_shift - 1))) >> a.address_shift;
        addr = addr > a.lut_entries - 1 ? a.lut_entries - 1 : addr;
        if (a.scores) a.scores[(static_cast<uint64_t>(h) * T + t) * T + s] = sc[s];
        sc[s] = a.lut[addr];
        esum += sc[s];
    }
    esum = block_sum(esum, scratch);
    const long long recip = ((1ll << 30) + esum / 2) / esum;
    // Q0.16 probabilities; with p_levels, requantised to
    // clamp((p * levels + 2^15) >> 16, 0, levels), counting zeros, and the
    // (first) largest Q0.16 probability tracked for the sum correction
    long long qsum = 0, zeros = 0, best = -1;
    for (uint32_t s = threadIdx.x; s < T; s += blockDim.x) {
        long long p = (static_cast<long long>(sc[s]) * recip + (1ll << 13)) >> 14;
        p = p > 65535 ? 65535 : p;
        if (a.probs) a.probs[(static_cast<uint64_t>(h) * T + t) * T + s] = static_cast<int32_t>(p);
        if (a.p_levels) {
            const long long key = (p << 12) | (4095 - s);  // larger p, then lower index
            best = max(best, key);
            long long pq = (p * a.p_levels + (1ll << 15)) >> 16;
            pq = clampll(pq, 0, a.p_levels);
            zeros += pq == 0 ? 1 : 0;
            qsum += pq;
            p = pq;
        }
        sc[s] = static_cast<int32_t>(p);
    }
    if (a.p_levels) {
        qsum = block_sum(qsum, scratch);
        zeros = block_sum(zeros, scratch);
        best = block_max_ll(best, scratch);  // its barrier orders every sc write above
        if (a.sum_correction && threadIdx.x == 0) sc[4095 - (best & 4095)] += static_cast<int32_t>(a.p_levels - qsum);
        __syncthreads();
        if (a.probs_q)
            for (uint32_t s = threadIdx.x; s < T; s += blockDim.x)
                a.probs_q[(static_cast<uint64_t>(h) * T + t) * T + s] = sc[s];
    } else {
        __syncthreads();
    }
    // P . V: thread (d, half) sums keys s = half, half + 2, ...
    const uint32_t d = threadIdx.x & 63u, half = threadIdx.x >> 6;
    long long acc = 0;
    if (a.p_levels) {
        for (uint32_t s = half; s < T; s += 2)
            acc += static_cast<long long>(sc[s]) * a.v8[(static_cast<uint64_t>(s) * a.H + h) * 64 + d];
    } else {
        for (uint32_t s = half; s < T; s += 2)
            acc += static_cast<long long>(sc[s]) * a.qkv12[((static_cast<uint64_t>(s) * 3 + 2) * a.H + h) * 64 + d];
    }
    part[threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.x < 64) {
        const long long tot = part[threadIdx.x] + part[threadIdx.x + 64];
        const long long y = a.p_levels ? sym_round_shift(tot * prm[kPkOutMult], 24) : sym_round_shift(tot, 16);
        a.out[static_cast<uint64_t>(t) * a.H * 64 + h * 64 + d] = static_cast<int32_t>(clampll(y, lo, hi));
    }
    if (threadIdx.x == 0 && a.p_levels && zeros && a.head_stats)
        atomicAdd(reinterpret_cast<unsigned long long*>(a.head_stats + h * 4 + 3),
                  static_cast<unsigned long long>(zeros));
}

constexpr uint32_t kLinTile = 64, kLinK = 32;

struct WideLinearArgs {
    const int32_t* act;  // [rows, K]
    const int16_t* w;    // [N, K]
    const long long* mult;
    const int32_t* bias;  // [N] or null
    uint32_t rows, n, k, shift;
    long long lo, hi;
    int32_t* out;       // [rows, N]
    long long* acc;     // optional [rows, N]
    long long* stats;   // [acc min, acc max, saturated, max |acc|]
};

// 64 x 64 output tile per CTA of 256 threads, 4 x 4 int64 accumulators per
// thread (32 x 32 -> 64-bit multiply-adds).
__global__ void __launch_bounds__(256) fixed_wide_linear_kernel(WideLinearArgs a) {
    __shared__ int32_t As[kLinK][kLinTile + 1];
    __shared__ int32_t Ws[kLinK][kLinTile + 1];
    const uint32_t r0 = blockIdx.y * kLinTile, c0 = blockIdx.x * kLinTile;
    const uint32_t tr = threadIdx.x / 16, tc = threadIdx.x % 16;
    long long acc[4][4] = {};
    for (uint32_t k0 = 0; k0 < a.k; k0 += kLinK) {
        for (uint32_t i = threadIdx.x; i < kLinK * kLinTile; i += blockDim.x) {
            const uint32_t kk = i % kLinK, rr = i / kLinK;
            const uint32_t gk = k0 + kk;
            As[kk][rr] = (r0 + rr < a.rows && gk < a.k) ? a.act[static_cast<uint64_t>(r0 + rr) * a.k + gk] : 0;
            Ws[kk][rr] = (c0 + rr < a.n && gk < a.k) ? a.w[static_cast<uint64_t>(c0 + rr) * a.k + gk] : 0;
        }
        __syncthreads();
#pragma unroll 4
        for (uint32_t kk = 0; kk < kLinK; ++kk) {
            int32_t av[4], wv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                av[i] = As[kk][tr + 16 * i];
                wv[i] = Ws[kk][tc + 16 * i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += static_cast<long long>(av[i]) * wv[j];
        }
        __syncthreads();
    }
    long long amin = LLONG_MAX, amax = LLONG_MIN, aabs = 0, sat = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t r = r0 + tr + 16 * i;
        if (r >= a.rows) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t c = c0 + tc + 16 * j;
            if (c >= a.n) continue;
            const long long v = acc[i][j];
            amin = min(amin, v);
            amax = max(amax, v);
            aabs = max(aabs, v < 0 ? -v : v);
            // int64 product with two's-complement wrap, as torch int64 tensors
            const long long prod = static_cast<long long>(static_cast<unsigned long long>(v) *
                                                          static_cast<unsigned long long>(a.mult[c]));
            long long o = sym_round_shift(prod, a.shift) + (a.bias ? a.bias[c] : 0);
            if (o < a.lo || o > a.hi) {
                ++sat;
                o = o < a.lo ? a.lo : a.hi;
            }
            a.out[static_cast<uint64_t>(r) * a.n + c] = static_cast<int32_t>(o);
            if (a.acc) a.acc[static_cast<uint64_t>(r) * a.n + c] = v;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        amin = min(amin, __shfl_xor_sync(0xFFFFFFFFu, amin, o));
        amax = max(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
        aabs = max(aabs, __shfl_xor_sync(0xFFFFFFFFu, aabs, o));
        sat += __shfl_xor_sync(0xFFFFFFFFu, sat, o);
    }
    if (lane_id() == 0 && a.stats && amin <= amax) {
        atomicMin(a.stats, amin);
        atomicMax(a.stats + 1, amax);
        atomicAdd(reinterpret_cast<unsigned long long*>(a.stats + 2), static_cast<unsigned long long>(sat));
        atomicMax(a.stats + 3, aabs);
    }
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" {

uint32_t dh_fixed_layer_norm_q12(const float* in, uint32_t rows, uint32_t cols, uint32_t input_fraction_bits,
                                 uint32_t output_fraction_bits, uint32_t inverse_fraction_bits,
                                 uint32_t sqrt_extra_fraction_bits, int64_t epsilon_q, int32_t* out,
                                 int64_t* row_stats, void* stream) {
    if (!in || !out) return DH_ERR_NULL_POINTER;
    if (rows == 0 || cols == 0) return DH_OK;
    if (input_fraction_bits > 20 || sqrt_extra_fraction_bits > 8 || epsilon_q < 0 ||
        inverse_fraction_bits + input_fraction_bits + sqrt_extra_fraction_bits > 60 ||
        inverse_fraction_bits + input_fraction_bits <= output_fraction_bits)
        return DH_ERR_INVALID_ARGUMENT;
    LnArgs a{in, rows, cols, input_fraction_bits, output_fraction_bits, inverse_fraction_bits,
             sqrt_extra_fraction_bits, static_cast<long long>(epsilon_q), out,
             reinterpret_cast<long long*>(row_stats)};
    fixed_layer_norm_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_fixed_rotary_q12(const float* qkv, const float* cosine, const float* sine, uint32_t tokens,
                             uint32_t heads, int32_t* qkv_q12, int32_t* query_q12, int32_t* key_q12,
                             int64_t* stats, void* stream) {
    if (!qkv || !cosine || !sine || !qkv_q12 || !query_q12 || !key_q12) return DH_ERR_NULL_POINTER;
    if (tokens == 0 || heads == 0) return DH_OK;
    const uint64_t pairs = static_cast<uint64_t>(tokens) * 3 * heads * 32;
    const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((pairs + 255) / 256, 4096));
    fixed_rotary_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        qkv, cosine, sine, tokens, heads, qkv_q12, query_q12, key_q12, reinterpret_cast<long long*>(stats));
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_fixed_attention_q12(const int32_t* query_q12, const int32_t* key_q12, const int32_t* qkv_q12,
                                uint32_t tokens, uint32_t heads, uint32_t exponential_step_bits,
                                int64_t cutoff_q10, const int32_t* exponential_lut_q16, uint32_t lut_entries,
                                int32_t* out_q12, int32_t* scores_q10, int32_t* probabilities_q16,
                                int64_t* stats, void* stream) {
    if (!query_q12 || !key_q12 || !qkv_q12 || !exponential_lut_q16 || !out_q12) return DH_ERR_NULL_POINTER;
    if (tokens == 0 || heads == 0) return DH_OK;
    if (tokens > kMaxTokens) return DH_ERR_UNSUPPORTED_SHAPE;
    if (exponential_step_bits < 1 || exponential_step_bits > 9 || cutoff_q10 <= 0 || lut_entries == 0)
        return DH_ERR_INVALID_ARGUMENT;
    FixedAttnArgs a{query_q12, key_q12, qkv_q12, tokens, heads, 10u - exponential_step_bits, lut_entries,
                    static_cast<long long>(cutoff_q10), exponential_lut_q16, out_q12, scores_q10,
                    probabilities_q16, reinterpret_cast<long long*>(stats)};
    fixed_attention_kernel<<<tokens * heads, kAttnThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_fixed_wide_linear(const int32_t* activation, const int16_t* weight, const int64_t* multiplier,
                              const int32_t* bias_q, uint32_t rows, uint32_t n, uint32_t k, uint32_t shift,
                              int64_t output_min, int64_t output_max, int32_t* out, int64_t* accumulators,
                              int64_t* stats, void* stream) {
    if (!activation || !weight || !multiplier || !out) return DH_ERR_NULL_POINTER;
    if (rows == 0 || n == 0) return DH_OK;
    if (k == 0 || shift == 0 || shift > 62 || output_min > output_max || output_min < INT32_MIN ||
        output_max > INT32_MAX)
        return DH_ERR_INVALID_ARGUMENT;
    WideLinearArgs a{activation, weight, reinterpret_cast<const long long*>(multiplier), bias_q, rows, n, k, shift,
                     static_cast<long long>(output_min), static_cast<long long>(output_max), out,
                     reinterpret_cast<long long*>(accumulators), reinterpret_cast<long long*>(stats)};
    dim3 grid((n + kLinTile - 1) / kLinTile, (rows + kLinTile - 1) / kLinTile);
    fixed_wide_linear_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_packed_int8_attention_q12(const int32_t* query_q12, const int32_t* key_q12, const int32_t* qkv_q12,
                                      uint32_t tokens, uint32_t heads, uint32_t qk_mode, uint32_t qk_scores,
                                      uint32_t qk_levels, uint32_t qk_fraction_bits, uint32_t pv_probability_levels,
                                      uint32_t pv_sum_correction, uint32_t pv_value_levels,
                                      const int64_t* head_params, uint32_t exponential_step_bits, int64_t cutoff_q10,
                                      const int32_t* exponential_lut_q16, uint32_t lut_entries, int32_t* workspace,
                                      int32_t* out_q12, int32_t* scores_q10, int32_t* probabilities_q16,
                                      int32_t* probabilities_quantized, int32_t* query_maxima,
                                      int32_t* key_maxima, int64_t* head_stats, void* stream) {
    if (!query_q12 || !key_q12 || !qkv_q12 || !head_params || !exponential_lut_q16 || !out_q12)
        return DH_ERR_NULL_POINTER;
    if (qk_mode > 2 || exponential_step_bits < 1 || exponential_step_bits > 9 || cutoff_q10 <= 0 ||
        lut_entries == 0 || pv_probability_levels > 65535 || pv_value_levels > 32767)
        return DH_ERR_INVALID_ARGUMENT;
    if (qk_mode != 0 && (qk_levels < 1 || qk_levels > 32767 || qk_fraction_bits < 1 || qk_fraction_bits > 30))
        return DH_ERR_INVALID_ARGUMENT;
    if ((pv_probability_levels != 0 && pv_value_levels == 0) || (qk_scores && qk_mode == 0))
        return DH_ERR_INVALID_ARGUMENT;
    if ((qk_mode != 0 || pv_value_levels != 0) && !workspace) return DH_ERR_NULL_POINTER;
    if (qk_mode == 2 && (!query_maxima || !key_maxima)) return DH_ERR_NULL_POINTER;
    if (tokens == 0 || heads == 0) return DH_OK;
    if (tokens > kMaxTokens) return DH_ERR_UNSUPPORTED_SHAPE;
    const uint64_t vec = static_cast<uint64_t>(tokens) * heads * 64;
    int32_t* q8 = workspace;
    int32_t* k8 = workspace ? workspace + vec : nullptr;
    int32_t* v8 = workspace ? workspace + 2 * vec : nullptr;
    const long long* prm = reinterpret_cast<const long long*>(head_params);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (qk_mode != 0 || pv_value_levels != 0) {
        PackedQuantArgs qa{query_q12, key_q12, qkv_q12, tokens, heads, qk_mode, qk_levels, qk_fraction_bits,
                           pv_value_levels, prm, q8, k8, v8, query_maxima, key_maxima,
                           reinterpret_cast<long long*>(head_stats)};
        const uint32_t warps = tokens * heads * 3;
        packed_quant_kernel<<<(warps + 7) / 8, 256, 0, st>>>(qa);
        DH_LAUNCH_CHECK();
    }
    PackedAttnArgs aa{qk_scores ? q8 : query_q12, qk_scores ? k8 : key_q12, v8, qkv_q12, query_maxima, key_maxima,
                      prm, tokens, heads, qk_mode, qk_scores ? 1u : 0u, qk_levels, pv_probability_levels,
                      pv_sum_correction ? 1u : 0u, 10u - exponential_step_bits, lut_entries,
                      static_cast<long long>(cutoff_q10), exponential_lut_q16, out_q12, scores_q10,
                      probabilities_q16, probabilities_quantized, reinterpret_cast<long long*>(head_stats)};
    packed_attention_kernel<<<tokens * heads, kAttnThreads, 0, st>>>(aa);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

}  // extern "C"
