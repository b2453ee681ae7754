// dh_philox.cuh -- counter-based Philox4x32-10 and the factorized Q5.10 Gumbel
// score, as device functions.
//
// Philox4x32-10 follows Random123 (multipliers 0xD2511F53 / 0xCD9E8D57, Weyl
// key increments 0x9E3779B9 / 0xBB67AE85; reference hls/rng/philox_rng.cpp:33-54,
// src/diffusion_accel/rng.py:36-61).  The Gumbel score follows
// hls/rng/philox_rng.cpp:74-93: d = ~w, e = clz(d), 8-bit mantissa after the
// leading one, exact tables for e < 3, (e+1)*ln2 + base[m] above, d == 0 -> top.
// Here the two table families are merged into one 32x256 int16 table that the
// kernels keep in shared memory (one LDS per score).
#pragma once

#include "dh_common.cuh"
#include "gumbel_lut.h"

namespace dh {

struct Philox4 {
    uint32_t x, y, z, w;
};

// Round keys for one (key_lo, key_hi) pair are the same for every counter, so
// kernels that draw many words under one key precompute them.
struct PhiloxKeySchedule {
    uint32_t k0[10], k1[10];
};

DH_DEVINL PhiloxKeySchedule philox_schedule(uint32_t key_lo, uint32_t key_hi) {
    PhiloxKeySchedule s;
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        s.k0[r] = key_lo + static_cast<uint32_t>(r) * 0x9E3779B9u;
        s.k1[r] = key_hi + static_cast<uint32_t>(r) * 0xBB67AE85u;
    }
    return s;
}

DH_DEVINL Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                uint32_t key_lo, uint32_t key_hi) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = static_cast<uint64_t>(0xD2511F53u) * c0;
        const uint64_t p1 = static_cast<uint64_t>(0xCD9E8D57u) * c2;
        const uint32_t n0 = static_cast<uint32_t>(p1 >> 32) ^ c1 ^ key_lo;
        const uint32_t n2 = static_cast<uint32_t>(p0 >> 32) ^ c3 ^ key_hi;
        c1 = static_cast<uint32_t>(p1);
        c3 = static_cast<uint32_t>(p0);
        c0 = n0;
        c2 = n2;
        key_lo += 0x9E3779B9u;
        key_hi += 0xBB67AE85u;
    }
    return Philox4{c0, c1, c2, c3};
}

DH_DEVINL Philox4 philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3,
                                const PhiloxKeySchedule& ks) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = static_cast<uint64_t>(0xD2511F53u) * c0;
        const uint64_t p1 = static_cast<uint64_t>(0xCD9E8D57u) * c2;
        const uint32_t n0 = static_cast<uint32_t>(p1 >> 32) ^ c1 ^ ks.k0[r];
        const uint32_t n2 = static_cast<uint32_t>(p0 >> 32) ^ c3 ^ ks.k1[r];
        c1 = static_cast<uint32_t>(p1);
        c3 = static_cast<uint32_t>(p0);
        c0 = n0;
        c2 = n2;
    }
    return Philox4{c0, c1, c2, c3};
}

DH_DEVINL uint32_t philox_lane(const Philox4& r, uint32_t i) {
    return i == 0 ? r.x : i == 1 ? r.y : i == 2 ? r.z : r.w;
}

// Copies the merged Gumbel table into shared memory, word i by thread
// i % count of the `count` threads that call it (the one-argument form: all
// threads of the block); those threads synchronise before reading it.
DH_DEVINL void load_gumbel_table(int16_t* smem_table, uint32_t tid, uint32_t count) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(DH_GUMBEL_MERGED_Q10_DEV);
    uint32_t* dst = reinterpret_cast<uint32_t*>(smem_table);
    for (uint32_t i = tid; i < 32u * 256u / 2u; i += count) dst[i] = src[i];
}
DH_DEVINL void load_gumbel_table(int16_t* smem_table) { load_gumbel_table(smem_table, threadIdx.x, blockDim.x); }

// Score of one word using the shared-memory merged table.
DH_DEVINL int32_t gumbel_q10(uint32_t word, const int16_t* smem_table) {
    const uint32_t d = ~word;
    if (d == 0u) return DH_GUMBEL_TOP_Q10;
    const uint32_t e = __clz(d);                 // 0..31
    const uint32_t top_bit_shift = 31u - e;      // floor(log2 d)
    // 9-bit normalised value 1mmmmmmmm: shift right when the leading one is
    // at bit 8 or above, left otherwise.
    const uint32_t norm = top_bit_shift >= 8u ? (d >> (top_bit_shift - 8u))
                                              : (d << (8u - top_bit_shift));
    const uint32_t m = norm & 0xFFu;
    return smem_table[(e << 8) | m];
}

}  // namespace dh
