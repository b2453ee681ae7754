// attention.cu -- K5: bidirectional attention softmax(Q K^T / 8) V for the
// DDiT blocks (mlx_mdlm.py:431-436, hardware_package.py:239-245), with the
// prefix-cached form where K / V = [cached prefix ; active rows]
// (prefix_drift.py:213-223).
//
// Layouts (written by the QKV epilogue): Q [B, H, q_len, 64] and K [B, H, kv_len, 64]
// bf16, V transposed [B, H, 64, kv_len] f16.  Output O [B * q_len, H * 64] bf16
// (token-major, heads concatenated, the input of the attention-out linear).
//
// Persistent kernel, two CTAs per SM, 6 warps each.  A work item is
// (128-query tile, head, sequence); keys are processed in tiles of 64:
//   warp 0   TMA: Q once per item (staged in shared memory, copied into
//            TMEM by the softmax warps), then K_j (4-deep ring) and V_j (3-deep)
//   warp 1   tcgen05 MMA (kind::f16 -> fp32 in TMEM):
//            S_j = Q K_j^T (bf16, 128 x 64 x 64, Q from TMEM, K from shared
//            memory) into one of two TMEM S/P buffers, then
//            [O | l] += P_j [V_j | 1] (f16, 128 x 80 x 64) with P_j read from
//            TMEM; a ones row under each V tile makes the tensor core also
//            sum P into column 64.
//   warps 2-5 softmax: one thread per query row reads its 64 scores from
//            TMEM, keeps the running max in a register (base-2 domain), and
//            writes P_j = 2^(s*c - m) as packed f16 back over S_j in TMEM.
//            O accumulates in TMEM across key tiles and is rescaled in place
//            only when the row max grows by more than 2^8.
// Keeping Q and P in TMEM takes their reads (and P's write) off shared
// memory, whose bandwidth (128 B/clk) the MMA operand reads otherwise
// saturate at these shapes: per 64-key tile only K, V and their TMA writes
// touch it.  Two S/P buffers let the softmax of tile j+1 run while PV_j
// executes.  ~78 KB shared memory and 256 TMEM columns per CTA.  All waits
// are bounded, and a waiting thread sleeps on its mbarrier instead of
// polling: the TMA and MMA warps share schedulers with softmax warps, whose
// issue slots the polls took (147 -> 144.5 us at 32 x 1024).
#include <cuda.h>
#include <cuda_bf16.h>

#include "tc_ptx.cuh"
#include "tmap.h"

#include <algorithm>

namespace dh {
namespace {

constexpr uint32_t kHeads = 12;
constexpr uint32_t kDh = 64;
constexpr uint32_t kQTile = 128;                      // queries per work item
constexpr uint32_t kKT = 64;                          // keys per tile
constexpr uint32_t kThreads = 192;
constexpr uint32_t kQBytes = kQTile * kDh * 2;        // 16 KB
constexpr uint32_t kKBytes = kKT * kDh * 2;           // 8 KB (64 keys x 128 B)
// V tile: [64 value rows ; 16 constant rows] x 64 keys, f16, SW128 K-major.
// The constant rows are one row of ones and 15 of zeros, so the PV MMA
// (N = 80) also produces l = sum_j P_j in O column 64, accumulated in fp32
// from exactly the P values that weight V.
constexpr uint32_t kVRows = kDh + 16;
constexpr uint32_t kVBytes = kVRows * 128;            // 10 KB per stage
constexpr uint32_t kVLoadBytes = kDh * kKT * 2;       // 8 KB brought by TMA per tile
constexpr uint32_t kKStages = 4;
constexpr uint32_t kVStages = 3;
constexpr uint32_t kSmemBytes = 1024 + kQBytes + kKStages * kKBytes + kVStages * kVBytes + 256;
// TMEM: two S/P buffers of 64 columns (S_j fp32, then P_j f16 packed into
// the first 32 columns of the same buffer), O [128,192), l at 192, and Q
// (bf16 packed, 32 columns) at [224,256).
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kOCol = 128;
constexpr uint32_t kQCol = 224;
constexpr uint32_t kIdescS = tc::idesc_bf16_f32<128, kKT>();     // Q, K bf16
constexpr uint32_t kIdescO = tc::idesc_f16_f32<128, kVRows>();   // P, V f16

struct AttnArgs {
    uint32_t sequences, q_len, kv_len, kv_stride;
    __nv_bfloat16* out;
    const uint32_t* run_flag;
};

// Ring barriers come in one copy per stage / buffer: kKFull + stage, etc.
// kSPFree + b: PV of the tile held in S/P buffer b finished (the buffer may
// take the next S; O holds that tile's contribution).
enum Bar : uint32_t {
    kQFull = 0, kQEmpty, kKFull, kKEmpty = kKFull + kKStages, kVFull = kKEmpty + kKStages,
    kVEmpty = kVFull + kVStages, kSFull = kVEmpty + kVStages, kPFull = kSFull + 2, kSPFree = kPFull + 2,
    kOFull = kSPFree + 2, kOFree, kQReady, kDrain, kNumBars
};

DH_DEVINL void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Hardware base-2 exponential (MUFU), flush-to-zero.
DH_DEVINL float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

DH_DEVINL uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// (lo, hi) fp32 -> f16x2, round to nearest even.
DH_DEVINL uint32_t pack_f16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// 2^x of two fp32 values on the FMA pipe, for x <= 8: Cody-Waite split
// x = n + f with n = rint(x) taken by the 1.5 * 2^23 shifter and f in
// [-0.5, 0.5]; 2^f by a degree-3 polynomial whose coefficients were fitted
// for this kernel (least squares on Chebyshev nodes, reweighted toward
// minimax: max relative error 7.8e-5, below the f16 half-ulp of P); 2^n is
// added into the exponent field.  x is clamped at -120 (2^-120 is 0 in f16).
constexpr float kExp2C0 = 0.99992895f, kExp2C1 = 0.69327623f, kExp2C2 = 0.24260406f,
                kExp2C3 = 0.05508874f;
DH_DEVINL float2 exp2_poly2(float2 x) {
    x = make_float2(fmaxf(x.x, -120.f), fmaxf(x.y, -120.f));
    const float2 t = __fadd2_rn(x, make_float2(12582912.f, 12582912.f));
    const float2 n = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
    const float2 f = __ffma2_rn(n, make_float2(-1.f, -1.f), x);
    float2 p = __ffma2_rn(make_float2(kExp2C3, kExp2C3), f, make_float2(kExp2C2, kExp2C2));
    p = __ffma2_rn(p, f, make_float2(kExp2C1, kExp2C1));
    p = __ffma2_rn(p, f, make_float2(kExp2C0, kExp2C0));
    return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                       __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

// Pairs of P computed on the FMA pipe instead of the MUFU: pair e of a row
// uses the polynomial when bit (e % 8) of this mask is set (a quarter of
// them: the MUFU stays the busier unit, the FMA pipe takes the rest).
constexpr uint32_t kPolyPairMask = 0x11u;

// Hardware base-2 exponential of two f16 values at once (MUFU).
DH_DEVINL uint32_t ex2_f16x2(uint32_t x) {
    uint32_t y;
    asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

struct Item {
    uint32_t seq, head, q_tile, bh;
};

DH_DEVINL Item item_of(uint32_t w, uint32_t n_qt) {
    Item it;
    it.q_tile = w % n_qt;
    it.bh = w / n_qt;
    it.head = it.bh % kHeads;
    it.seq = it.bh / kHeads;
    return it;
}

// Every role walks the same (item, key tile) sequence; a global key-tile
// counter g drives the ring / buffer / phase bookkeeping, so the next item's
// Q and K loads overlap the current item's last tiles.
__global__ void __launch_bounds__(kThreads, 2)
attention_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                 const __grid_constant__ CUtensorMap tv, const AttnArgs args) {
    // sequences processed: all, or those of the first *run_flag query rows
    const uint32_t live_seqs =
        args.run_flag ? min(args.sequences, *args.run_flag / args.q_len) : args.sequences;
    if (live_seqs == 0) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* q_s = smem;
    uint8_t* k_ring = q_s + kQBytes;                    // kKStages x 8 KB
    uint8_t* v_ring = k_ring + kKStages * kKBytes;      // kVStages x 10 KB
    uint64_t* bars = reinterpret_cast<uint64_t*>(v_ring + kVStages * kVBytes);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);

    const uint32_t warp = warp_id(), lane = lane_id();
    const uint32_t n_kv = (args.kv_len + kKT - 1) / kKT;
    const uint32_t n_qt = (args.q_len + kQTile - 1) / kQTile;
    // keys of the last tile that exist (kKT when kv_len is a multiple of it)
    const uint32_t kv_rem = args.kv_len - (n_kv - 1) * kKT;
    const uint32_t total = live_seqs * kHeads * n_qt;

    if (warp == 0 && lane == 0) {
        for (uint32_t i = 0; i < kNumBars; ++i) {
            const bool softmax_side =
                (i >= kPFull && i < kPFull + 2) || i == kOFree || i == kQEmpty || i == kQReady;
            tc::mbar_init(&bars[i], softmax_side ? 128u : 1u);
        }
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tq);
        tc::prefetch_tmap(&tk);
        tc::prefetch_tmap(&tv);
    }
    // constant rows of every V stage: row 64 = f16 ones, rows 65-79 = 0
    // (a constant row reads the same under the 128-byte swizzle)
    for (uint32_t i = threadIdx.x; i < kVStages * 512; i += blockDim.x) {
        const uint32_t st = i / 512, w = i % 512;  // 512 words = 2 KB per stage
        reinterpret_cast<uint32_t*>(v_ring + st * kVBytes + kDh * 128)[w] = w < 32 ? 0x3C003C00u : 0u;
    }
    fence_proxy_async_smem();
    if (warp == 1) tc::tmem_alloc(tmem_holder, kTmemCols);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA
        if (tc::elect_one()) {
            uint32_t g = 0, it = 0;
            bool ok = true;
            for (uint32_t w = blockIdx.x; w < total && ok; w += gridDim.x, ++it) {
                const Item item = item_of(w, n_qt);
                if (!tc::mbar_wait_suspend(&bars[kQEmpty], (it & 1u) ^ 1u, tc::kErrTimeoutEmpty)) break;
                tc::mbar_arrive_expect_tx(&bars[kQFull], kQBytes);
                tc::tma_load_2d(q_s, &tq, &bars[kQFull], 0,
                                static_cast<int32_t>(item.bh * args.q_len + item.q_tile * kQTile));
                for (uint32_t j = 0; j < n_kv; ++j, ++g) {
                    const uint32_t ks = g % kKStages, vs_i = g % kVStages;
                    if (!tc::mbar_wait_suspend(&bars[kKEmpty + ks], ((g / kKStages) & 1u) ^ 1u, tc::kErrTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_arrive_expect_tx(&bars[kKFull + ks], kKBytes);
                    tc::tma_load_2d(k_ring + ks * kKBytes, &tk, &bars[kKFull + ks], 0,
                                    static_cast<int32_t>(item.bh * args.kv_stride + j * kKT));
                    if (!tc::mbar_wait_suspend(&bars[kVEmpty + vs_i], ((g / kVStages) & 1u) ^ 1u, tc::kErrTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_arrive_expect_tx(&bars[kVFull + vs_i], kVLoadBytes);
                    tc::tma_load_2d(v_ring + vs_i * kVBytes, &tv, &bars[kVFull + vs_i],
                                    static_cast<int32_t>(j * kKT), static_cast<int32_t>(item.bh * kDh));
                }
            }
            // Drain: every copy this CTA issued has landed before it may exit.
            if (it > 0) tc::mbar_wait_suspend(&bars[kQFull], (it - 1) & 1u, tc::kErrTimeoutFull);
            for (uint32_t x = g > kKStages ? g - kKStages : 0; x < g; ++x)
                tc::mbar_wait_suspend(&bars[kKFull + x % kKStages], (x / kKStages) & 1u, tc::kErrTimeoutFull);
            for (uint32_t x = g > kVStages ? g - kVStages : 0; x < g; ++x)
                tc::mbar_wait_suspend(&bars[kVFull + x % kVStages], (x / kVStages) & 1u, tc::kErrTimeoutFull);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA
        if (tc::elect_one()) {
            const uint32_t o_tmem = tmem + kOCol;
            // S_g into TMEM buffer g % 2 once PV_{g-2} has consumed P_{g-2} there.
            auto issue_s = [&](uint32_t g) -> bool {
                const uint32_t ks = g % kKStages, sb = g & 1u;
                if (!tc::mbar_wait_suspend(&bars[kKFull + ks], (g / kKStages) & 1u, tc::kErrTimeoutFull) ||
                    !tc::mbar_wait_suspend(&bars[kSPFree + sb], ((g >> 1) & 1u) ^ 1u, tc::kErrTimeoutAccEmpty))
                    return false;
                tc::tc_fence_after();
                const uint64_t k_desc = tc::smem_desc_sw128(k_ring + ks * kKBytes);
#pragma unroll
                for (uint32_t kk = 0; kk < kDh / 16; ++kk)  // A = Q from TMEM, 8 columns per 16 dims
                    tc::mma_f16_ts(tmem + sb * kKT, tmem + kQCol + kk * 8, tc::desc_advance(k_desc, kk * 32),
                                   kIdescS, kk != 0);
                tc::mma_commit(&bars[kSFull + sb]);
                tc::mma_commit(&bars[kKEmpty + ks]);
                return true;
            };
            uint32_t g = 0, it = 0;
            bool ok = true;
            for (uint32_t w = blockIdx.x; w < total && ok; w += gridDim.x, ++it) {
                if (!tc::mbar_wait_suspend(&bars[kQReady], it & 1u, tc::kErrTimeoutFull)) break;
                tc::tc_fence_after();
                if (!issue_s(g)) break;
                for (uint32_t j = 0; j < n_kv; ++j, ++g) {
                    if (j + 1 < n_kv && !issue_s(g + 1)) {
                        ok = false;
                        break;
                    }
                    const uint32_t vs_i = g % kVStages, sb = g & 1u;
                    ok = tc::mbar_wait_suspend(&bars[kPFull + sb], (g >> 1) & 1u, tc::kErrTimeoutFull) &&
                         tc::mbar_wait_suspend(&bars[kVFull + vs_i], (g / kVStages) & 1u, tc::kErrTimeoutFull) &&
                         (j != 0 || tc::mbar_wait_suspend(&bars[kOFree], (it & 1u) ^ 1u, tc::kErrTimeoutAccEmpty));
                    if (!ok) break;
                    tc::tc_fence_after();
                    const uint64_t v_desc = tc::smem_desc_sw128(v_ring + vs_i * kVBytes);
#pragma unroll
                    for (uint32_t kk = 0; kk < kKT / 16; ++kk)  // A = P_j from TMEM, 8 columns per 16 keys
                        tc::mma_f16_ts(o_tmem, tmem + sb * kKT + kk * 8, tc::desc_advance(v_desc, kk * 32),
                                       kIdescO, (kk | j) != 0);
                    tc::mma_commit(&bars[kVEmpty + vs_i]);
                    tc::mma_commit(&bars[kSPFree + sb]);
                    if (j + 1 == n_kv) tc::mma_commit(&bars[kOFull]);
                }
            }
            tc::mma_commit(&bars[kDrain]);
            tc::mbar_wait_suspend(&bars[kDrain], 0, tc::kErrTimeoutAccFull);
        }
    } else {
        // ----------------------------------------------------------- softmax
        // One thread per query row.  p = 2^(s*c - m) with the running max m
        // kept stale until a tile's max exceeds it by more than 8 (p <= 2^8
        // meanwhile); only then are O and l (accumulated in TMEM across
        // tiles) rescaled -- a warp-uniform, rare path.
        const uint32_t quad = warp & 3u;
        const uint32_t r = quad * 32 + lane;  // query row within the tile
        const uint32_t lane_base = (quad * 32u) << 16;
        const float c = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
        // Q row r of item `qi` from the TMA-staged (128-byte swizzled) tile into
        // TMEM lane r, then release the staging buffer and signal the MMA warp.
        // Called before the item's first S and only after every S of the
        // previous item completed (this thread saw their kSFull).
        auto copy_q = [&](uint32_t qi) -> bool {
            if (!tc::mbar_wait_suspend(&bars[kQFull], qi & 1u, tc::kErrTimeoutFull)) return false;
            const uint8_t* rowq = q_s + (r >> 3) * 1024 + (r & 7u) * 128;
            uint32_t qv[32];
#pragma unroll
            for (uint32_t cc = 0; cc < 8; ++cc) {
                const uint4 v = *reinterpret_cast<const uint4*>(rowq + ((cc ^ (r & 7u)) * 16));
                qv[4 * cc] = v.x;
                qv[4 * cc + 1] = v.y;
                qv[4 * cc + 2] = v.z;
                qv[4 * cc + 3] = v.w;
            }
            tc::tmem_st_32x32b_x32(tmem + lane_base + kQCol, qv);
            tc::tmem_st_wait();
            tc::tc_fence_before();
            tc::mbar_arrive(&bars[kQEmpty]);
            tc::mbar_arrive(&bars[kQReady]);
            return true;
        };
        uint32_t g = 0, it = 0;
        bool ok = blockIdx.x >= total || copy_q(0);
        for (uint32_t w = blockIdx.x; w < total && ok; w += gridDim.x, ++it) {
            const Item item = item_of(w, n_qt);
            float m = 0.f;
            for (uint32_t j = 0; j < n_kv; ++j, ++g) {
                const uint32_t sb = g & 1u;
                if (!tc::mbar_wait_suspend(&bars[kSFull + sb], (g >> 1) & 1u, tc::kErrTimeoutAccFull)) { ok = false; break; }
                tc::tc_fence_after();
                uint32_t sv[64];
                tc::tmem_ld_32x32b_x32(tmem + lane_base + sb * kKT, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
                tc::tmem_ld_32x32b_x32(tmem + lane_base + sb * kKT + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
                tc::tmem_ld_wait();
                // ragged key tail: keys past kv_len score -inf (p = 0); their
                // K rows are whatever the tile read, V rows are finite (zero
                // padding or other rows), so 0 * V adds nothing.
                if (j + 1 == n_kv && kv_rem != kKT) {
#pragma unroll
                    for (uint32_t e = 0; e < 64; ++e)
                        if (e >= kv_rem) sv[e] = 0xFF800000u;
                }
                // row max with 8 independent partial maxima (short dependency chains)
                float pm[8];
#pragma unroll
                for (uint32_t q = 0; q < 8; ++q) pm[q] = __uint_as_float(sv[q]);
#pragma unroll
                for (uint32_t e = 8; e < 64; e += 16) {
#pragma unroll
                    for (uint32_t q = 0; q < 8; ++q) {
                        const uint32_t i0 = e + q, i1 = e + 8 + q;
                        if (i1 < 64) {
                            float t3;
                            asm("max.f32 %0, %1, %2, %3;" : "=f"(t3) : "f"(pm[q]), "f"(__uint_as_float(sv[i0])),
                                "f"(__uint_as_float(sv[i1])));
                            pm[q] = t3;
                        } else {
                            pm[q] = fmaxf(pm[q], __uint_as_float(sv[i0]));
                        }
                    }
                }
                const float tmax = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                                         fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
                const float mt = tmax * c;
                float alpha = 1.f;
                bool need = false;
                if (j == 0) {
                    m = mt;
                } else if (mt > m + 8.0f) {
                    need = true;
                    alpha = ex2_approx(m - mt);
                    m = mt;
                }
                // p = 2^(s*c - m) <= 2^8 as packed f16, stored over S_j in
                // TMEM: the A operand of PV_j.
                const float2 c2 = make_float2(c, c);
                const float2 nm2 = make_float2(-m, -m);
                uint32_t pk[32];
#pragma unroll
                for (uint32_t e = 0; e < 32; ++e) {
                    const float2 sv2 = make_float2(__uint_as_float(sv[2 * e]), __uint_as_float(sv[2 * e + 1]));
                    const float2 a = __ffma2_rn(sv2, c2, nm2);
                    if ((kPolyPairMask >> (e & 7u)) & 1u) {
                        const float2 y = exp2_poly2(a);
                        pk[e] = pack_f16x2(y.x, y.y);
                    } else {
                        pk[e] = ex2_f16x2(pack_f16x2(a.x, a.y));
                    }
                }
                tc::tmem_st_32x32b_x32(tmem + lane_base + sb * kKT, pk);
                if (__any_sync(0xFFFFFFFFu, need)) {
                    // O and l must be stable: PV_{g-1} (the only one that may
                    // still run; PV_g waits for this tile's kPFull) finished.
                    if (!tc::mbar_wait_suspend(&bars[kSPFree + (sb ^ 1u)], ((g - 1) >> 1) & 1u, tc::kErrTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
#pragma unroll
                    for (uint32_t h2 = 0; h2 < 3; ++h2) {  // columns 128..223 (208.. unused)
                        uint32_t ov[32];
                        tc::tmem_ld_32x32b_x32(tmem + lane_base + kOCol + 32 * h2, ov);
                        tc::tmem_ld_wait();
#pragma unroll
                        for (uint32_t d = 0; d < 32; ++d) ov[d] = __float_as_uint(__uint_as_float(ov[d]) * alpha);
                        tc::tmem_st_32x32b_x32(tmem + lane_base + kOCol + 32 * h2, ov);
                    }
                    tc::tmem_st_wait();
                }
                tc::tmem_st_wait();
                tc::tc_fence_before();
                tc::mbar_arrive(&bars[kPFull + sb]);
            }
            if (!ok) break;
            // next item's Q into TMEM before this item's epilogue, so its S can start
            if (w + gridDim.x < total && !copy_q(it + 1)) break;
            // item done: O = accumulated P V, l in column 64; normalise and store
            if (!tc::mbar_wait_suspend(&bars[kOFull], it & 1u, tc::kErrTimeoutAccFull)) break;
            tc::tc_fence_after();
            uint32_t v0[32], v1[32];
            tc::tmem_ld_32x32b_x32(tmem + lane_base + kOCol, v0);
            tc::tmem_ld_32x32b_x32(tmem + lane_base + kOCol + 32, v1);
            const uint32_t l_bits = tc::tmem_ld_32x32b_x1(tmem + lane_base + kOCol + kDh);
            tc::tmem_ld_wait();
            tc::tc_fence_before();
            tc::mbar_arrive(&bars[kOFree]);
            const float inv_l = 1.0f / __uint_as_float(l_bits);
            if (item.q_tile * kQTile + r >= args.q_len) continue;  // ragged query tail
            const uint64_t tok = static_cast<uint64_t>(item.seq) * args.q_len + item.q_tile * kQTile + r;
            __nv_bfloat16* dst = args.out + tok * (kHeads * kDh) + item.head * kDh;
#pragma unroll
            for (uint32_t d = 0; d < 32; d += 8) {
                uint4 a, b;
                a.x = pack_bf16(__uint_as_float(v0[d]) * inv_l, __uint_as_float(v0[d + 1]) * inv_l);
                a.y = pack_bf16(__uint_as_float(v0[d + 2]) * inv_l, __uint_as_float(v0[d + 3]) * inv_l);
                a.z = pack_bf16(__uint_as_float(v0[d + 4]) * inv_l, __uint_as_float(v0[d + 5]) * inv_l);
                a.w = pack_bf16(__uint_as_float(v0[d + 6]) * inv_l, __uint_as_float(v0[d + 7]) * inv_l);
                b.x = pack_bf16(__uint_as_float(v1[d]) * inv_l, __uint_as_float(v1[d + 1]) * inv_l);
                b.y = pack_bf16(__uint_as_float(v1[d + 2]) * inv_l, __uint_as_float(v1[d + 3]) * inv_l);
                b.z = pack_bf16(__uint_as_float(v1[d + 4]) * inv_l, __uint_as_float(v1[d + 5]) * inv_l);
                b.w = pack_bf16(__uint_as_float(v1[d + 6]) * inv_l, __uint_as_float(v1[d + 7]) * inv_l);
                *reinterpret_cast<uint4*>(dst + d) = a;
                *reinterpret_cast<uint4*>(dst + 32 + d) = b;
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" uint32_t dh_attention(const void* q, const void* k, const void* vt, void* out,
                                 uint32_t sequences, uint32_t q_len, uint32_t kv_len,
                                 uint32_t kv_stride, const uint32_t* run_flag, void* stream) {
    if (!q || !k || !vt || !out) return DH_ERR_NULL_POINTER;
    if (sequences == 0 || q_len == 0 || kv_len == 0 || kv_stride < kv_len)
        return DH_ERR_INVALID_ARGUMENT;
    if (q_len % 32 != 0 || kv_len % 32 != 0 || kv_stride % 8 != 0)
        return DH_ERR_UNSUPPORTED_SHAPE;
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
         reinterpret_cast<uintptr_t>(vt) | reinterpret_cast<uintptr_t>(out)) & 15u)
        return DH_ERR_ALIGNMENT;
    CUtensorMap tq, tk, tv;
    const uint64_t bh = static_cast<uint64_t>(sequences) * kHeads;
    if (!make_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, bh * q_len, kDh, kDh * 2, kQTile, 64) ||
        !make_tmap_2d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, bh * kv_stride, kDh, kDh * 2, kKT, 64) ||
        !make_tmap_2d(&tv, vt, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, bh * kDh, kv_stride,
                      static_cast<uint64_t>(kv_stride) * 2, 64, 64))
        return DH_ERR_CUDA;
    static std::atomic<uint64_t> configured{0};
    if (smem_optin_once(attention_kernel, kSmemBytes, configured) != cudaSuccess) return DH_ERR_CUDA;
    AttnArgs a{sequences, q_len, kv_len, kv_stride, static_cast<__nv_bfloat16*>(out), run_flag};
    int sms = kNumSMs, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) sms = v;
    }
    const uint64_t items = static_cast<uint64_t>(sequences) * kHeads * ((q_len + kQTile - 1) / kQTile);
    const uint32_t grid = static_cast<uint32_t>(std::min<uint64_t>(items, 2ull * sms));
    attention_kernel<<<grid, kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, a);
    DH_LAUNCH_CHECK();
    return DH_OK;
}
