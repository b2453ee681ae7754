// head.cu -- K9: the 768 x 50258 int8 output head fused with Philox-Gumbel
// noisy argmax; logits never reach HBM.
//
// The int8 GEMM runs on tcgen05 (gemm_tc.cuh); the epilogue turns each
// accumulator into a score and keeps, per row, the running (max score, lowest
// token id) in registers, merged across tiles with one 64-bit atomicMax per
// row and tile (score in the high word with the sign bit flipped, ~id in the
// low word -- the tie rule of output_head.cpp:147-151 and
// ordered_noisy_argmax_reducer.sv:106-133).
//
// Score modes:
//   kRequantQ20    the HLS contract (output_head.cpp:126-146): round-half-away
//                  (acc * mult_q20[v]) >> 20, + bias_q10[v] + noise
//   kDequantNoisy  the model path: logit = float(double(acc) *
//                  double(a_scale[r] * w_scale[v]) + double(bias[v])) -- exactly
//                  the reference W8A8 output (fixed_mlp.py:98-106) -- then
//                  round_half_even(logit * 1024) + Gumbel_Q10 (rng.py:262)
//   kDequantGreedy argmax of the same fp32 logit (final greedy pass)
// noise = factorized Gumbel of philox((v/4, pos[r], eval[r], stream),
// (key_lo, key_hi[r]))[v%4], or an explicit [rows, vocab] int32 array.
// Integer scores saturate at +-2^31-1 (the reference keeps int64); the two
// agree whenever |score| < 2^31, i.e. |logit| < 2^21 in Q10 units.
#include <cuda_bf16.h>

#include "dh_philox.cuh"
#include "gemm_tc.cuh"
#include "tmap.h"

namespace dh {

uint32_t make_i8_operand_maps(CUtensorMap* ta, CUtensorMap* tb, const int8_t* a, uint64_t lda,
                              const int8_t* w, uint64_t ldw, uint32_t m, uint32_t n, uint32_t k,
                              uint32_t bn);

namespace {

enum HeadMode : uint32_t { kRequantQ20 = 0, kDequantNoisy = 1, kDequantGreedy = 2 };

struct HeadParams {
    uint32_t mode;
    uint32_t vocab, mask_id;   // vocab: columns of this weight slice; mask_id: global token id
    uint32_t vocab_offset;     // global id of column 0 (vocab-sharded head), multiple of 4
    const float* a_scale;      // [rows]          (dequant modes)
    const float* w_scale;      // [vocab]
    const float* bias;         // [vocab] fp32
    const int32_t* mult_q20;   // [vocab]         (requant mode)
    const int32_t* bias_q10;   // [vocab]
    const int32_t* noise;      // [rows, vocab] or null -> Philox
    const uint32_t* row_position;  // null -> row index
    const uint32_t* row_key_hi;    // null -> const_key_hi
    const uint32_t* row_eval;      // null -> const_eval
    uint32_t const_eval, const_key_hi, key_lo, stream_id;
    unsigned long long* packed;    // [rows] running (score, ~id), zero-initialised
};

DH_DEVINL int32_t sat_i32(int64_t v) {
    return v > 2147483647LL ? 2147483647 : (v < -2147483647LL ? -2147483647 : static_cast<int32_t>(v));
}

DH_DEVINL int32_t requant_q20(int32_t acc, int32_t mult) {
    const int64_t prod = static_cast<int64_t>(acc) * mult;
    const int64_t half = 1LL << 19;
    return prod >= 0 ? static_cast<int32_t>((prod + half) >> 20)
                     : -static_cast<int32_t>((-prod + half) >> 20);
}

DH_DEVINL float ref_logit(int32_t acc, float a_scale, float w_scale, float bias) {
    const float combined = __fmul_rn(a_scale, w_scale);
    // double(acc) * double(combined) is exact (24 x 24 bits), so one DFMA equals
    // the reference's separate multiply and add in float64.
    const double v = __fma_rn(static_cast<double>(acc), static_cast<double>(combined),
                              static_cast<double>(bias));
    return __double2float_rn(v);
}

// The same logit with the int and float to double conversions done on the
// integer and FP64 pipes instead of the conversion unit:
//   double(acc): the double 2^52 + 2^31 + acc assembled from bits, minus
//   2^52 + 2^31 (exact for any int32);
//   double(combined): for a positive normal float the double's bits are the
//   float's re-biased (exact); other values take the converting path.
DH_DEVINL float ref_logit_bits(int32_t acc, float a_scale, float w_scale, double bias) {
    const float combined = __fmul_rn(a_scale, w_scale);
    const double acc_d = __hiloint2double(0x43300000, static_cast<int32_t>(static_cast<uint32_t>(acc) ^ 0x80000000u)) -
                         4503601774854144.0;  // 2^52 + 2^31
    const uint32_t cb = __float_as_uint(combined);
    double comb_d;
    if (cb - 0x00800000u < 0x7F000000u)  // positive, normal, finite
        comb_d = __hiloint2double(static_cast<int32_t>((cb >> 3) + 0x38000000u), static_cast<int32_t>(cb << 29));
    else
        comb_d = static_cast<double>(combined);
    return __double2float_rn(__fma_rn(acc_d, comb_d, bias));
}

DH_DEVINL int32_t q10(float logit);

// q10 with round-half-even through the 1.5 * 2^23 shifter when |x| < 2^22
// (the common case), else the converting path.
DH_DEVINL int32_t q10_shift(float logit) {
    const float scaled = __fmul_rn(logit, 1024.0f);
    if (fabsf(scaled) < 4194304.0f) return __float_as_int(__fadd_rn(scaled, 12582912.0f)) - 0x4B400000;
    return q10(logit);
}

DH_DEVINL int32_t q10(float logit) {
    const float scaled = __fmul_rn(logit, 1024.0f);
    if (!(scaled == scaled)) return -(1 << 30);
    if (scaled > 1073741824.0f) return 1 << 30;
    if (scaled < -1073741824.0f) return -(1 << 30);
    return __float2int_rn(scaled);
}

// Philox4x32-10 of counter (c0, pos, ev, stream) under key (key_lo, key_hi)
// when only c0 changes between calls: the first round's product of the
// third counter word, and the words it mixes with, are fixed per row and
// come in precomputed (r0 = hi(M1 * ev) ^ pos ^ key_lo, r1 = lo(M1 * ev),
// r2 = stream ^ key_hi).  The rounds are those of dh_philox.cuh.
struct PhiloxRow {
    uint32_t r0, r1, r2;
};

DH_DEVINL PhiloxRow philox_row(uint32_t pos, uint32_t ev, uint32_t stream, uint32_t key_lo, uint32_t key_hi) {
    const uint64_t p1 = static_cast<uint64_t>(0xCD9E8D57u) * ev;
    return PhiloxRow{static_cast<uint32_t>(p1 >> 32) ^ pos ^ key_lo, static_cast<uint32_t>(p1), stream ^ key_hi};
}

DH_DEVINL Philox4 philox_row_block(uint32_t c0, const PhiloxRow& pr, uint32_t key_lo, uint32_t key_hi) {
    const uint64_t p0 = static_cast<uint64_t>(0xD2511F53u) * c0;
    uint32_t x0 = pr.r0, x1 = pr.r1;
    uint32_t x2 = static_cast<uint32_t>(p0 >> 32) ^ pr.r2, x3 = static_cast<uint32_t>(p0);
#pragma unroll
    for (int r = 1; r < 10; ++r) {
        key_lo += 0x9E3779B9u;
        key_hi += 0xBB67AE85u;
        const uint64_t q0 = static_cast<uint64_t>(0xD2511F53u) * x0;
        const uint64_t q1 = static_cast<uint64_t>(0xCD9E8D57u) * x2;
        const uint32_t n0 = static_cast<uint32_t>(q1 >> 32) ^ x1 ^ key_lo;
        const uint32_t n2 = static_cast<uint32_t>(q0 >> 32) ^ x3 ^ key_hi;
        x1 = static_cast<uint32_t>(q1);
        x3 = static_cast<uint32_t>(q0);
        x0 = n0;
        x2 = n2;
    }
    return Philox4{x0, x1, x2, x3};
}

// gumbel_q10 with the mantissa taken from d normalised to bit 31 (one
// variable shift instead of two shift directions): same table index.  The
// lookup happens before the d == 0 select, so e is kept to 0..31 (clz of 0
// is 32, whose row lies past the 32 x 256 table).
DH_DEVINL int32_t gumbel_q10_norm(uint32_t word, const int16_t* smem_table) {
    const uint32_t d = ~word;
    const uint32_t e = __clz(d) & 31u;
    const uint32_t m = ((d << e) >> 23) & 0xFFu;
    const int32_t v = smem_table[(e << 8) | m];
    return d == 0u ? DH_GUMBEL_TOP_Q10 : v;
}

struct EpiHead : EpiBase {
    static constexpr uint32_t kChunk = 32;
    // two groups of 8 epilogue warps: the per-logit work (Philox, Gumbel,
    // dequant, race) is a chain of dependent integer / FP64 operations that
    // 2 warps per scheduler cannot keep the pipes busy with
    static constexpr uint32_t kGroups = 2;
    static constexpr uint32_t kStages = 3;
    // per warp: its 128 columns' bias as double (1 KB) and w_scale (512 B),
    // converted once per tile instead of once per logit
    static constexpr uint32_t kStagingPerWarp = 1536;
    static constexpr uint32_t kExtraSmem = 32 * 256 * 2;  // merged Gumbel table
    // few rows (the revealed rows of one sequence): all four lane quadrants
    // race a quarter of the columns each
    static constexpr bool kReplicateRows = true;
    using Params = HeadParams;
    struct TileState {
        unsigned long long best;
        float a_scale;
        uint32_t pos, key_hi, ev;
        PhiloxRow pr;
        const int16_t* table;
        const uint8_t* stage;
    };
    static DH_DEVINL void init_smem(const Params&, uint8_t* extra, uint32_t tid, uint32_t count) {
        load_gumbel_table(reinterpret_cast<int16_t*>(extra), tid, count);
    }
    static DH_DEVINL bool tile_begin(const Params& p, TileState& st, const EpiCtx& ctx, uint32_t col_start) {
        const uint32_t row = ctx.row;
        if (p.mode == kDequantNoisy) {
            double* bd = reinterpret_cast<double*>(ctx.stage);
            float* wsd = reinterpret_cast<float*>(ctx.stage + 1024);
#pragma unroll
            for (uint32_t i = 0; i < 4; ++i) {
                const uint32_t c = col_start + ctx.lane + 32 * i;
                bd[ctx.lane + 32 * i] = c < p.vocab ? static_cast<double>(__ldg(p.bias + c)) : 0.0;
                wsd[ctx.lane + 32 * i] = c < p.vocab ? __ldg(p.w_scale + c) : 0.f;
            }
            __syncwarp();
        }
        st.stage = ctx.stage;
        st.best = 0ull;
        st.table = reinterpret_cast<const int16_t*>(ctx.extra);
        if (!ctx.row_ok) return true;
        st.a_scale = p.a_scale ? p.a_scale[row] : 0.f;
        st.pos = p.row_position ? p.row_position[row] : row;
        st.key_hi = p.row_key_hi ? p.row_key_hi[row] : p.const_key_hi;
        st.ev = p.row_eval ? p.row_eval[row] : p.const_eval;
        st.pr = philox_row(st.pos, st.ev, p.stream_id, p.key_lo, st.key_hi);
        return true;
    }
    // The common chunk: Philox noise, dequant scores, all 32 columns inside
    // the vocabulary and none of them the mask token.  Written for
    // instruction-level parallelism (the chunk is otherwise one long
    // dependent chain per warp): the 8 Philox blocks and the 32 scores are
    // independent, and the running maximum is a tree over (score, column)
    // pairs in which the left (lower-id) side wins ties, so the result equals
    // the sequential strict-greater scan.
    static DH_DEVINL void noisy_chunk(const Params& p, TileState& st, uint32_t col0, const uint32_t* v) {
        const uint32_t gid0 = col0 + p.vocab_offset;
        int32_t best_s = INT32_MIN;
        uint32_t best_j = 0;
#pragma unroll
        for (uint32_t qq = 0; qq < 4; ++qq) {  // 8 columns: two Philox blocks
            uint32_t wd[8];
#pragma unroll
            for (uint32_t g = 0; g < 2; ++g) {
                const Philox4 r = philox_row_block((gid0 >> 2) + 2 * qq + g, st.pr, p.key_lo, st.key_hi);
                wd[4 * g] = r.x;
                wd[4 * g + 1] = r.y;
                wd[4 * g + 2] = r.z;
                wd[4 * g + 3] = r.w;
            }
            int32_t sc[8];
            // this warp's staged column parameters (the chunk lies in its half tile)
            const uint32_t cl = (col0 % 128u) + 8 * qq;
            const float4* w4p = reinterpret_cast<const float4*>(st.stage + 1024 + cl * 4);
            const double2* b2p = reinterpret_cast<const double2*>(st.stage + cl * 8);
#pragma unroll
            for (uint32_t q = 0; q < 2; ++q) {
                const float4 w4 = w4p[q];
                const double2 b01 = b2p[2 * q], b23 = b2p[2 * q + 1];
                const float ws[4] = {w4.x, w4.y, w4.z, w4.w};
                const double bs[4] = {b01.x, b01.y, b23.x, b23.y};
#pragma unroll
                for (uint32_t e = 0; e < 4; ++e) {
                    const uint32_t j = 4 * q + e;
                    // |q10| <= 2^30 and |noise| < 2^15: the sum fits in int32
                    sc[j] = q10_shift(ref_logit_bits(static_cast<int32_t>(v[8 * qq + j]), st.a_scale, ws[e], bs[e])) +
                            gumbel_q10_norm(wd[j], st.table);
                }
            }
            uint32_t ix[8];
#pragma unroll
            for (uint32_t j = 0; j < 8; ++j) ix[j] = 8 * qq + j;
#pragma unroll
            for (uint32_t stride = 1; stride < 8; stride <<= 1) {
#pragma unroll
                for (uint32_t j = 0; j < 8; j += 2 * stride) {
                    const bool right = sc[j + stride] > sc[j];
                    sc[j] = right ? sc[j + stride] : sc[j];
                    ix[j] = right ? ix[j + stride] : ix[j];
                }
            }
            if (sc[0] > best_s) {
                best_s = sc[0];
                best_j = ix[0];
            }
        }
        const unsigned long long pk = pack_score_id(best_s, gid0 + best_j);
        st.best = pk > st.best ? pk : st.best;
    }
    static DH_DEVINL void chunk(const Params& p, TileState& st, const EpiCtx& ctx, uint32_t col0,
                                const uint32_t* v) {
        const uint32_t row = ctx.row;
        if (!ctx.row_ok || col0 >= p.vocab) return;
        if (p.mode == kDequantNoisy && !p.noise && col0 + 32 <= p.vocab &&
            p.mask_id - (col0 + p.vocab_offset) >= 32u) {
            noisy_chunk(p, st, col0, v);
            return;
        }
        unsigned long long best = st.best;
        if (p.mode == kDequantGreedy) {
#pragma unroll
            for (uint32_t j = 0; j < 32; ++j) {
                const uint32_t t = col0 + j;
                if (t >= p.vocab || t + p.vocab_offset == p.mask_id) continue;
                const float l = ref_logit(static_cast<int32_t>(v[j]), st.a_scale,
                                          __ldg(p.w_scale + t), __ldg(p.bias + t));
                const unsigned long long pk = pack_float_id(l, t + p.vocab_offset);
                best = pk > best ? pk : best;
            }
            st.best = best;
            return;
        }
        const bool full_chunk = col0 + 32 <= p.vocab && (p.vocab & 3u) == 0;
#pragma unroll
        for (uint32_t g = 0; g < 32; g += 4) {
            const uint32_t t0 = col0 + g;
            if (t0 >= p.vocab) break;
            Philox4 w{0, 0, 0, 0};
            if (!p.noise)
                w = philox4x32_10((t0 + p.vocab_offset) >> 2, st.pos, st.ev, p.stream_id, p.key_lo, st.key_hi);
            float ws[4] = {0.f, 0.f, 0.f, 0.f}, bs[4] = {0.f, 0.f, 0.f, 0.f};
            int32_t ms[4] = {0, 0, 0, 0}, bq[4] = {0, 0, 0, 0};
            if (p.mode == kRequantQ20) {
#pragma unroll
                for (uint32_t i = 0; i < 4; ++i)
                    if (t0 + i < p.vocab) {
                        ms[i] = __ldg(p.mult_q20 + t0 + i);
                        bq[i] = __ldg(p.bias_q10 + t0 + i);
                    }
            } else if (full_chunk) {
                const float4 w4 = __ldg(reinterpret_cast<const float4*>(p.w_scale + t0));
                const float4 b4 = __ldg(reinterpret_cast<const float4*>(p.bias + t0));
                ws[0] = w4.x; ws[1] = w4.y; ws[2] = w4.z; ws[3] = w4.w;
                bs[0] = b4.x; bs[1] = b4.y; bs[2] = b4.z; bs[3] = b4.w;
            } else {
#pragma unroll
                for (uint32_t i = 0; i < 4; ++i)
                    if (t0 + i < p.vocab) {
                        ws[i] = __ldg(p.w_scale + t0 + i);
                        bs[i] = __ldg(p.bias + t0 + i);
                    }
            }
#pragma unroll
            for (uint32_t i = 0; i < 4; ++i) {
                const uint32_t t = t0 + i;
                if (t >= p.vocab || t + p.vocab_offset == p.mask_id) continue;
                const int32_t acc = static_cast<int32_t>(v[g + i]);
                const int32_t noise = p.noise ? p.noise[static_cast<uint64_t>(row) * p.vocab + t]
                                              : gumbel_q10(philox_lane(w, i), st.table);
                int64_t s;
                if (p.mode == kRequantQ20)
                    s = static_cast<int64_t>(requant_q20(acc, ms[i])) + bq[i] + noise;
                else
                    s = static_cast<int64_t>(q10(ref_logit(acc, st.a_scale, ws[i], bs[i]))) + noise;
                const unsigned long long pk = pack_score_id(sat_i32(s), t + p.vocab_offset);
                best = pk > best ? pk : best;
            }
        }
        st.best = best;
    }
    static DH_DEVINL void tile_end(const Params& p, TileState& st, const EpiCtx& ctx) {
        if (ctx.row_ok && st.best) atomicMax(p.packed + ctx.row, st.best);
    }
};

__global__ void zero_u64_kernel(unsigned long long* p, uint32_t n, const uint32_t* count) {
    const uint32_t m = count ? min(n, *count) : n;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < m; i += gridDim.x * blockDim.x)
        p[i] = 0ull;
}

__global__ void head_finalize_kernel(const unsigned long long* packed, uint32_t rows,
                                     const uint32_t* count, uint32_t greedy, int32_t* ids,
                                     int32_t* scores, uint16_t* ids16) {
    const uint32_t m = count ? min(rows, *count) : rows;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < m; i += gridDim.x * blockDim.x) {
        const unsigned long long b = packed[i];
        const uint32_t id = b == 0ull ? 0u : packed_id(b);
        if (ids) ids[i] = static_cast<int32_t>(id);
        if (ids16) ids16[i] = static_cast<uint16_t>(id);
        if (scores) {
            if (!greedy) {
                scores[i] = packed_score(b);
            } else {
                const uint32_t k = static_cast<uint32_t>(b >> 32);
                scores[i] = static_cast<int32_t>((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
            }
        }
    }
}

uint32_t launch_head(const int8_t* hidden, uint64_t ld_hidden, const int8_t* weights,
                     uint64_t ld_weights, uint32_t rows, const uint32_t* rows_count,
                     uint32_t hidden_size, const HeadParams& hp, cudaStream_t st) {
    CUtensorMap ta, tb;
    uint32_t s = make_i8_operand_maps(&ta, &tb, hidden, ld_hidden, weights, ld_weights, rows,
                                      hp.vocab, hidden_size, 256);
    if (s != DH_OK) return s;
    // the same rows with a 32-row box, for launches with at most 32 valid rows
    CUtensorMap ta32;
    if (!make_tmap_2d(&ta32, hidden, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rows, hidden_size, ld_hidden, 32, 128))
        return DH_ERR_CUDA;
    const uint32_t zb = std::min<uint32_t>((rows + 255) / 256, 1024u);
    zero_u64_kernel<<<zb, 256, 0, st>>>(hp.packed, rows, rows_count);
    DH_LAUNCH_CHECK();
    GemmShape shape{rows, hp.vocab, hidden_size, rows_count};
    const uint32_t tiles = ((rows + 127) / 128) * ((hp.vocab + 255) / 256);
    if (launch_gemm_i8<256, EpiHead>(ta, tb, shape, hp, tiles, st, &ta32) != cudaSuccess) return DH_ERR_CUDA;
    return DH_OK;
}

// The head's noise path alone: the (score, lowest id) race of the Philox /
// Gumbel Q10 noise over rows x vocab with every logit zero -- the same
// counters, key, words, table lookup and tie rule as the fused head, and no
// GEMM, dequantisation or logit.  One thread per (row, segment of
// kNoiseSeg tokens), all SMs full; per-segment winners merge with one
// 64-bit atomicMax per thread into `packed` (zero-initialised).  Its time
// over the head's rows and vocabulary is what generating the noise costs
// with nothing else competing for the integer pipes.
constexpr uint32_t kNoiseSeg = 512;

__global__ void __launch_bounds__(256)
noise_argmax_kernel(uint32_t rows, uint32_t vocab, uint32_t mask_id, const uint32_t* __restrict__ row_position,
                    const uint32_t* __restrict__ row_key_hi, const uint32_t* __restrict__ row_eval,
                    uint32_t const_eval, uint32_t const_key_hi, uint32_t key_lo, uint32_t stream_id,
                    unsigned long long* __restrict__ packed) {
    __shared__ int16_t table[32 * 256];
    load_gumbel_table(table);
    __syncthreads();
    const uint32_t segs = (vocab + kNoiseSeg - 1) / kNoiseSeg;
    const uint64_t work = static_cast<uint64_t>(rows) * segs;
    for (uint64_t t = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; t < work;
         t += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t row = static_cast<uint32_t>(t / segs);
        const uint32_t s0 = static_cast<uint32_t>(t % segs) * kNoiseSeg;
        const uint32_t end = min(vocab, s0 + kNoiseSeg);
        const uint32_t key_hi = row_key_hi ? row_key_hi[row] : const_key_hi;
        const PhiloxRow pr = philox_row(row_position ? row_position[row] : row, row_eval ? row_eval[row] : const_eval,
                                        stream_id, key_lo, key_hi);
        int32_t best_s = INT32_MIN;
        uint32_t best_id = 0;
#pragma unroll 1
        for (uint32_t v0 = s0; v0 < end; v0 += 8) {
            uint32_t wd[8];
#pragma unroll
            for (uint32_t g = 0; g < 2; ++g) {
                const Philox4 r = philox_row_block((v0 >> 2) + g, pr, key_lo, key_hi);
                wd[4 * g] = r.x;
                wd[4 * g + 1] = r.y;
                wd[4 * g + 2] = r.z;
                wd[4 * g + 3] = r.w;
            }
            int32_t sc[8];
            uint32_t ix[8];
#pragma unroll
            for (uint32_t j = 0; j < 8; ++j) {
                const uint32_t id = v0 + j;
                sc[j] = (id < end && id != mask_id) ? gumbel_q10_norm(wd[j], table) : INT32_MIN;
                ix[j] = id;
            }
            // tree over the 8 columns, the lower id winning ties
#pragma unroll
            for (uint32_t stride = 1; stride < 8; stride <<= 1) {
#pragma unroll
                for (uint32_t j = 0; j < 8; j += 2 * stride) {
                    const bool right = sc[j + stride] > sc[j];
                    sc[j] = right ? sc[j + stride] : sc[j];
                    ix[j] = right ? ix[j + stride] : ix[j];
                }
            }
            if (sc[0] > best_s) {
                best_s = sc[0];
                best_id = ix[0];
            }
        }
        if (best_s != INT32_MIN) atomicMax(packed + row, pack_score_id(best_s, best_id));
    }
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" {

uint32_t dh_noise_argmax(uint32_t rows, uint32_t vocabulary_size, uint32_t mask_token_id,
                         const uint32_t* row_position, const uint32_t* row_key_hi, const uint32_t* row_eval,
                         uint32_t const_eval, uint32_t const_key_hi, uint32_t key_lo, uint32_t stream_id,
                         uint64_t* packed, int32_t* out_ids, void* stream) {
    if (rows == 0) return DH_RNG_INVALID_POSITION_COUNT;
    if (vocabulary_size == 0 || vocabulary_size > 65535 || mask_token_id >= vocabulary_size)
        return DH_RNG_INVALID_VOCABULARY_SIZE;
    if (!packed) return DH_ERR_NULL_POINTER;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int sms = kNumSMs, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) sms = v;
    }
    const uint64_t work = static_cast<uint64_t>(rows) * ((vocabulary_size + kNoiseSeg - 1) / kNoiseSeg);
    const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((work + 255) / 256, 8ull * sms));
    noise_argmax_kernel<<<blocks, 256, 0, st>>>(rows, vocabulary_size, mask_token_id, row_position, row_key_hi,
                                               row_eval, const_eval, const_key_hi, key_lo, stream_id,
                                               reinterpret_cast<unsigned long long*>(packed));
    DH_LAUNCH_CHECK();
    if (out_ids) {
        head_finalize_kernel<<<std::min<uint32_t>((rows + 255) / 256, 1024u), 256, 0, st>>>(
            reinterpret_cast<unsigned long long*>(packed), rows, nullptr, 0u, out_ids, nullptr, nullptr);
        DH_LAUNCH_CHECK();
    }
    return DH_OK;
}

uint32_t dh_head_argmax_i8(const int8_t* hidden, uint64_t ld_hidden, const int8_t* weights,
                           uint64_t ld_weights, uint32_t rows, const uint32_t* rows_count,
                           uint32_t hidden_size, uint32_t vocabulary_size, uint32_t vocab_offset,
                           uint32_t mask_token_id, uint32_t mode, const float* a_scale, const float* w_scale,
                           const float* bias, const int32_t* mult_q20, const int32_t* bias_q10,
                           const int32_t* noise, const uint32_t* row_position,
                           const uint32_t* row_key_hi, const uint32_t* row_eval,
                           uint32_t const_eval, uint32_t key_lo, uint32_t stream_id,
                           uint64_t* packed, int32_t* out_ids, int32_t* out_scores, void* stream) {
    if (rows == 0) return DH_HEAD_INVALID_POSITION_COUNT;
    if (hidden_size == 0) return DH_HEAD_INVALID_HIDDEN_SIZE;
    if (vocabulary_size == 0 || vocab_offset + static_cast<uint64_t>(vocabulary_size) > 65535)
        return DH_HEAD_INVALID_VOCABULARY_SIZE;
    // the mask id is global and may lie outside this (shard's) row range
    if (mask_token_id > 65535) return DH_HEAD_INVALID_MASK_TOKEN;
    if (mode > kDequantGreedy || (vocab_offset & 3u)) return DH_ERR_INVALID_ARGUMENT;
    if (!packed) return DH_ERR_NULL_POINTER;
    if (mode == kRequantQ20 && (!mult_q20 || !bias_q10)) return DH_ERR_NULL_POINTER;
    if (mode != kRequantQ20 && (!a_scale || !w_scale || !bias)) return DH_ERR_NULL_POINTER;
    if ((reinterpret_cast<uintptr_t>(w_scale) | reinterpret_cast<uintptr_t>(bias)) & 15u)
        return DH_ERR_ALIGNMENT;
    HeadParams hp{mode, vocabulary_size, mask_token_id, vocab_offset, a_scale, w_scale, bias, mult_q20,
                  bias_q10, noise, row_position, row_key_hi, row_eval, const_eval, 0u, key_lo, stream_id,
                  reinterpret_cast<unsigned long long*>(packed)};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint32_t s = launch_head(hidden, ld_hidden, weights, ld_weights, rows, rows_count, hidden_size,
                             hp, st);
    if (s != DH_OK) return s;
    if (out_ids || out_scores) {
        head_finalize_kernel<<<std::min<uint32_t>((rows + 255) / 256, 1024u), 256, 0, st>>>(
            hp.packed, rows, rows_count, mode == kDequantGreedy, out_ids, out_scores, nullptr);
        DH_LAUNCH_CHECK();
    }
    return DH_OK;
}

// Mirror of output_head_int8_kernel (output_head.cpp:23-157): same arguments
// and status codes; the noise stream is either given as a [positions, vocab]
// array or generated in place as philox_gumbel_stream_kernel would
// (counter (v/4, position, evaluation_id, stream_id), key (seed_low, seed_high)).
// hidden / weights rows are `hidden_size` bytes and must be 16-byte aligned
// (hidden_size a multiple of 16: pad with zeros otherwise).  `workspace`
// holds position_count uint64 words.
uint32_t dh_output_head_int8(const int8_t* hidden, const int8_t* weights,
                             const int32_t* requant_multiplier_q20, const int32_t* bias,
                             const int32_t* noise, uint16_t* candidate_ids,
                             uint32_t position_count, uint32_t hidden_size,
                             uint32_t vocabulary_size, uint32_t mask_token_id,
                             uint32_t evaluation_id, uint32_t stream_id, uint32_t seed_low,
                             uint32_t seed_high, uint64_t* workspace, void* stream) {
    if (position_count == 0 || position_count > 64) return DH_HEAD_INVALID_POSITION_COUNT;
    if (hidden_size == 0 || hidden_size > 768) return DH_HEAD_INVALID_HIDDEN_SIZE;
    if (vocabulary_size == 0 || vocabulary_size > 65535) return DH_HEAD_INVALID_VOCABULARY_SIZE;
    if (mask_token_id >= vocabulary_size) return DH_HEAD_INVALID_MASK_TOKEN;
    if (!requant_multiplier_q20 || !bias || !candidate_ids || !workspace) return DH_ERR_NULL_POINTER;
    if (hidden_size % 16 != 0) return DH_ERR_ALIGNMENT;
    HeadParams hp{kRequantQ20, vocabulary_size, mask_token_id, 0u, nullptr, nullptr, nullptr,
                  requant_multiplier_q20, bias, noise, nullptr, nullptr, nullptr, evaluation_id,
                  seed_high, seed_low, stream_id, reinterpret_cast<unsigned long long*>(workspace)};
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint32_t s = launch_head(hidden, hidden_size, weights, hidden_size, position_count, nullptr,
                             hidden_size, hp, st);
    if (s != DH_OK) return s;
    head_finalize_kernel<<<1, 64, 0, st>>>(hp.packed, position_count, nullptr, 0u, nullptr,
                                           nullptr, candidate_ids);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

}  // extern "C"
