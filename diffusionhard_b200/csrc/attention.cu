// attention.cu -- K5: bidirectional attention softmax(Q K^T / 8) V for the
// DDiT blocks (mlx_mdlm.py:431-436, hardware_package.py:239-245), with the
// prefix-cached form where K / V = [cached prefix ; active rows]
// (prefix_drift.py:213-223).
//
// Layouts (written by the QKV epilogue): Q [B, H, q_len, 64], K [B, H, kv_len, 64]
// and V transposed [B, H, 64, kv_len], bf16.  Output O [B * q_len, H * 64] bf16
// (token-major, heads concatenated, the input of the attention-out linear).
//
// One CTA per (128-query tile, head, sequence), 6 warps:
//   warp 0   TMA: Q once, then K_j and V_j tiles of 128 keys
//   warp 1   tcgen05 MMA (kind::f16, bf16 x bf16 -> fp32 in TMEM):
//            S_j = Q K_j^T (128 x 128 x 64), O_j = P_j V_j (128 x 64 x 128)
//   warps 2-5 softmax: one thread per query row reads its S row from TMEM
//            once, keeps the running max / sum in registers (base-2 domain),
//            writes P_j (bf16) to 128-byte-swizzled shared memory as the A
//            operand of the PV MMA; O accumulates in TMEM across key tiles and
//            is rescaled in place only when the row max grows by > 2^8.
// K tiles are double-buffered so S_{j+1} can start while tile j's softmax runs
// (V_{j+1} has that whole softmax to arrive).  96 KB shared memory and 256
// TMEM columns per CTA: two CTAs share an SM and one CTA's softmax overlaps the
// other's MMAs.  All waits are bounded.
#include <cuda.h>
#include <cuda_bf16.h>

#include "tc_ptx.cuh"
#include "tmap.h"

#include <algorithm>

namespace dh {
namespace {

constexpr uint32_t kHeads = 12;
constexpr uint32_t kDh = 64;
constexpr uint32_t kTile = 128;
constexpr uint32_t kThreads = 192;
constexpr uint32_t kQBytes = kTile * kDh * 2;        // 16 KB
constexpr uint32_t kKBytes = kTile * kDh * 2;        // 16 KB
constexpr uint32_t kVBytes = kDh * kTile * 2;        // 16 KB (2 sub-tiles of 64 keys)
constexpr uint32_t kPBytes = kTile * kTile * 2;      // 32 KB (2 sub-tiles of 64 keys)
constexpr uint32_t kKStages = 2;                      // K ring depth (S_{j+1} needs K_{j+1} early)
constexpr uint32_t kVStages = 1;                      // V_{j+1} has a whole softmax to arrive
constexpr uint32_t kSmemBytes = 1024 + kQBytes + kKStages * kKBytes + kVStages * kVBytes + kPBytes + 256;
constexpr uint32_t kTmemCols = 256;                   // S: [0,128), O: [128,192)
constexpr uint32_t kIdescS = tc::idesc_bf16_f32<128, 128>();
constexpr uint32_t kIdescO = tc::idesc_bf16_f32<128, 64>();

struct AttnArgs {
    uint32_t sequences, q_len, kv_len, kv_stride;
    __nv_bfloat16* out;
    const uint32_t* run_flag;
};

// K / V barriers come in one copy per ring stage: kKFull + stage, etc.
enum Bar : uint32_t {
    kQFull = 0, kQEmpty, kKFull, kKEmpty = kKFull + kKStages, kVFull = kKEmpty + kKStages,
    kVEmpty = kVFull + kVStages, kSFull = kVEmpty + kVStages, kSFree, kPFull, kPEmpty, kOFull,
    kOFree, kDrain, kNumBars
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

// Persistent kernel: each CTA loops over work items w = (sequence, head,
// 128-query tile), items of one head adjacent so concurrently running CTAs
// share K / V in L2.  Every role walks the same (item, key tile) sequence; a
// global key-tile counter g drives the ring / phase bookkeeping, so the next
// item's Q and K loads overlap the current item's last tiles.
__global__ void __launch_bounds__(kThreads, 2)
attention_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                 const __grid_constant__ CUtensorMap tv, const AttnArgs args) {
    if (args.run_flag && *args.run_flag == 0u) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* q_s = smem;
    uint8_t* k_ring = q_s + kQBytes;                    // kKStages x 16 KB
    uint8_t* v_ring = k_ring + kKStages * kKBytes;      // kVStages x 16 KB
    uint8_t* p_s = v_ring + kVStages * kVBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + kPBytes);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);

    const uint32_t warp = warp_id(), lane = lane_id();
    const uint32_t n_kv = (args.kv_len + kTile - 1) / kTile;
    const uint32_t n_qt = (args.q_len + kTile - 1) / kTile;
    // keys of the last tile that exist (kTile when kv_len is a multiple of it)
    const uint32_t kv_rem = args.kv_len - (n_kv - 1) * kTile;
    const uint32_t total = args.sequences * kHeads * n_qt;

    if (warp == 0 && lane == 0) {
        for (uint32_t i = 0; i < kNumBars; ++i) {
            const bool softmax_side = i == kSFree || i == kPFull || i == kOFree;
            tc::mbar_init(&bars[i], softmax_side ? 128u : 1u);
        }
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tq);
        tc::prefetch_tmap(&tk);
        tc::prefetch_tmap(&tv);
    }
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
                if (!tc::mbar_wait(&bars[kQEmpty], (it & 1u) ^ 1u, tc::kErrTimeoutEmpty)) break;
                tc::mbar_arrive_expect_tx(&bars[kQFull], kQBytes);
                tc::tma_load_2d(q_s, &tq, &bars[kQFull], 0,
                                static_cast<int32_t>(item.bh * args.q_len + item.q_tile * kTile));
                for (uint32_t j = 0; j < n_kv; ++j, ++g) {
                    const uint32_t ks = g % kKStages, vs_i = g % kVStages;
                    if (!tc::mbar_wait(&bars[kKEmpty + ks], ((g / kKStages) & 1u) ^ 1u, tc::kErrTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_arrive_expect_tx(&bars[kKFull + ks], kKBytes);
                    tc::tma_load_2d(k_ring + ks * kKBytes, &tk, &bars[kKFull + ks], 0,
                                    static_cast<int32_t>(item.bh * args.kv_stride + j * kTile));
                    if (!tc::mbar_wait(&bars[kVEmpty + vs_i], ((g / kVStages) & 1u) ^ 1u, tc::kErrTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_arrive_expect_tx(&bars[kVFull + vs_i], kVBytes);
                    uint8_t* vs = v_ring + vs_i * kVBytes;
                    tc::tma_load_2d(vs, &tv, &bars[kVFull + vs_i], static_cast<int32_t>(j * kTile),
                                    static_cast<int32_t>(item.bh * kDh));
                    tc::tma_load_2d(vs + kVBytes / 2, &tv, &bars[kVFull + vs_i],
                                    static_cast<int32_t>(j * kTile + 64), static_cast<int32_t>(item.bh * kDh));
                }
            }
            // Drain: every copy this CTA issued has landed before it may exit.
            if (it > 0) tc::mbar_wait(&bars[kQFull], (it - 1) & 1u, tc::kErrTimeoutFull);
            for (uint32_t x = g > kKStages ? g - kKStages : 0; x < g; ++x)
                tc::mbar_wait(&bars[kKFull + x % kKStages], (x / kKStages) & 1u, tc::kErrTimeoutFull);
            for (uint32_t x = g > kVStages ? g - kVStages : 0; x < g; ++x)
                tc::mbar_wait(&bars[kVFull + x % kVStages], (x / kVStages) & 1u, tc::kErrTimeoutFull);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA
        if (tc::elect_one()) {
            const uint32_t s_tmem = tmem, o_tmem = tmem + 128;
            const uint64_t q_desc = tc::smem_desc_sw128(q_s);
            // S_{g+1} is issued as soon as the softmax has read S_g, before
            // PV_g, so the next tile's scores are ready when the softmax needs
            // them (within an item; Q is single-buffered across items).
            auto issue_s = [&](uint32_t g, bool last_of_item) -> bool {
                const uint32_t ks = g % kKStages;
                if (!tc::mbar_wait(&bars[kKFull + ks], (g / kKStages) & 1u, tc::kErrTimeoutFull) ||
                    !tc::mbar_wait(&bars[kSFree], (g & 1u) ^ 1u, tc::kErrTimeoutAccEmpty))
                    return false;
                tc::tc_fence_after();
                const uint64_t k_desc = tc::smem_desc_sw128(k_ring + ks * kKBytes);
#pragma unroll
                for (uint32_t kk = 0; kk < kDh / 16; ++kk)
                    tc::mma_bf16(s_tmem, tc::desc_advance(q_desc, kk * 32), tc::desc_advance(k_desc, kk * 32),
                                 kIdescS, kk != 0);
                tc::mma_commit(&bars[kSFull]);
                tc::mma_commit(&bars[kKEmpty + ks]);
                if (last_of_item) tc::mma_commit(&bars[kQEmpty]);
                return true;
            };
            uint32_t g = 0, it = 0;
            bool ok = true;
            for (uint32_t w = blockIdx.x; w < total && ok; w += gridDim.x, ++it) {
                if (!tc::mbar_wait(&bars[kQFull], it & 1u, tc::kErrTimeoutFull)) break;
                if (!issue_s(g, n_kv == 1)) break;
                for (uint32_t j = 0; j < n_kv; ++j, ++g) {
                    if (j + 1 < n_kv && !issue_s(g + 1, j + 2 == n_kv)) {
                        ok = false;
                        break;
                    }
                    const uint32_t vs_i = g % kVStages;
                    ok = tc::mbar_wait(&bars[kPFull], g & 1u, tc::kErrTimeoutFull) &&
                         tc::mbar_wait(&bars[kVFull + vs_i], (g / kVStages) & 1u, tc::kErrTimeoutFull) &&
                         (j != 0 || tc::mbar_wait(&bars[kOFree], (it & 1u) ^ 1u, tc::kErrTimeoutAccEmpty));
                    if (!ok) break;
                    tc::tc_fence_after();
                    uint8_t* vs = v_ring + vs_i * kVBytes;
#pragma unroll
                    for (uint32_t kk = 0; kk < kTile / 16; ++kk) {
                        const uint32_t sub = kk >> 2, off = (kk & 3u) * 32;
                        tc::mma_bf16(o_tmem,
                                     tc::desc_advance(tc::smem_desc_sw128(p_s + sub * (kPBytes / 2)), off),
                                     tc::desc_advance(tc::smem_desc_sw128(vs + sub * (kVBytes / 2)), off),
                                     kIdescO, (kk | j) != 0);
                    }
                    tc::mma_commit(&bars[kVEmpty + vs_i]);
                    tc::mma_commit(&bars[kPEmpty]);
                    if (j + 1 == n_kv) tc::mma_commit(&bars[kOFull]);
                }
            }
            tc::mma_commit(&bars[kDrain]);
            tc::mbar_wait(&bars[kDrain], 0, tc::kErrTimeoutAccFull);
        }
    } else {
        // ----------------------------------------------------------- softmax
        // One thread per query row.  S_j is read from TMEM once into
        // registers; p = exp2(s*c - m) with the running max m kept stale
        // until the tile max exceeds it by more than 8 (p <= 2^8 meanwhile),
        // and only then O (accumulated in TMEM across tiles) and l are
        // rescaled -- a warp-uniform, rare path.
        const uint32_t quad = warp & 3u;
        const uint32_t r = quad * 32 + lane;  // query row within the tile
        const uint32_t lane_base = (quad * 32u) << 16;
        const float c = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
        uint32_t g = 0, it = 0;
        bool ok = true;
        for (uint32_t w = blockIdx.x; w < total && ok; w += gridDim.x, ++it) {
            const Item item = item_of(w, n_qt);
            float m = 0.f, l = 0.f;
            for (uint32_t j = 0; j < n_kv; ++j, ++g) {
                if (!tc::mbar_wait(&bars[kSFull], g & 1u, tc::kErrTimeoutAccFull)) { ok = false; break; }
                tc::tc_fence_after();
                uint32_t sv[128];
#pragma unroll
                for (uint32_t cc = 0; cc < 4; ++cc)
                    tc::tmem_ld_32x32b_x32(tmem + lane_base + cc * 32,
                                           *reinterpret_cast<uint32_t(*)[32]>(&sv[cc * 32]));
                tc::tmem_ld_wait();
                tc::tc_fence_before();
                tc::mbar_arrive(&bars[kSFree]);
                // ragged key tail: keys past kv_len score -inf (p = 0); their
                // K rows are whatever the tile read, V rows are finite (zero
                // padding or other rows), so 0 * V adds nothing.
                if (j + 1 == n_kv && kv_rem != kTile) {
#pragma unroll
                    for (uint32_t e = 0; e < 128; ++e)
                        if (e >= kv_rem) sv[e] = 0xFF800000u;
                }
                // row max with 8 independent partial maxima (short dependency chains)
                float pm[8];
#pragma unroll
                for (uint32_t q = 0; q < 8; ++q) pm[q] = __uint_as_float(sv[q]);
#pragma unroll
                for (uint32_t e = 8; e < 128; e += 16) {
#pragma unroll
                    for (uint32_t q = 0; q < 8; ++q) {
                        const uint32_t i0 = e + q, i1 = e + 8 + q;
                        if (i1 < 128) {
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
                    l *= alpha;
                }
                const float2 c2 = make_float2(c, c);
                const float2 nm2 = make_float2(-m, -m);
                float2 ps[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                                make_float2(0.f, 0.f)};
                uint32_t pk[64];
#pragma unroll
                for (uint32_t e = 0; e < 64; ++e) {
                    const float2 sv2 = make_float2(__uint_as_float(sv[2 * e]), __uint_as_float(sv[2 * e + 1]));
                    const float2 a = __ffma2_rn(sv2, c2, nm2);
                    const float2 pe = make_float2(ex2_approx(a.x), ex2_approx(a.y));
                    ps[e & 3u] = __fadd2_rn(ps[e & 3u], pe);
                    pk[e] = pack_bf16(pe.x, pe.y);
                }
                const float2 sum2 = __fadd2_rn(__fadd2_rn(ps[0], ps[1]), __fadd2_rn(ps[2], ps[3]));
                // P buffer free and O stable: the previous PV finished.
                if (!tc::mbar_wait(&bars[kPEmpty], (g & 1u) ^ 1u, tc::kErrTimeoutEmpty)) { ok = false; break; }
                if (__any_sync(0xFFFFFFFFu, need)) {
                    tc::tc_fence_after();
#pragma unroll
                    for (uint32_t h2 = 0; h2 < 2; ++h2) {
                        uint32_t ov[32];
                        tc::tmem_ld_32x32b_x32(tmem + lane_base + 128 + 32 * h2, ov);
                        tc::tmem_ld_wait();
#pragma unroll
                        for (uint32_t d = 0; d < 32; ++d) ov[d] = __float_as_uint(__uint_as_float(ov[d]) * alpha);
                        tc::tmem_st_32x32b_x32(tmem + lane_base + 128 + 32 * h2, ov);
                    }
                    tc::tmem_st_wait();
                }
                uint8_t* rowp = p_s + (r >> 3) * 1024 + (r & 7u) * 128;
#pragma unroll
                for (uint32_t gg = 0; gg < 16; ++gg) {  // 16 chunks of 8 keys
                    const uint32_t sub = gg >> 3;
                    const uint32_t chunk = (gg & 7u) ^ (r & 7u);
                    *reinterpret_cast<uint4*>(rowp + sub * (kPBytes / 2) + chunk * 16) =
                        make_uint4(pk[4 * gg], pk[4 * gg + 1], pk[4 * gg + 2], pk[4 * gg + 3]);
                }
                l += sum2.x + sum2.y;
                fence_proxy_async_smem();
                tc::tc_fence_before();
                tc::mbar_arrive(&bars[kPFull]);
            }
            if (!ok) break;
            // item done: O = accumulated P V; normalise and store
            if (!tc::mbar_wait(&bars[kOFull], it & 1u, tc::kErrTimeoutAccFull)) break;
            tc::tc_fence_after();
            uint32_t v0[32], v1[32];
            tc::tmem_ld_32x32b_x32(tmem + lane_base + 128, v0);
            tc::tmem_ld_32x32b_x32(tmem + lane_base + 160, v1);
            tc::tmem_ld_wait();
            tc::tc_fence_before();
            tc::mbar_arrive(&bars[kOFree]);
            const float inv_l = 1.0f / l;
            if (item.q_tile * kTile + r >= args.q_len) continue;  // ragged query tail
            const uint64_t tok = static_cast<uint64_t>(item.seq) * args.q_len + item.q_tile * kTile + r;
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
    if (!make_tmap_2d(&tq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, bh * q_len, kDh, kDh * 2, kTile, 64) ||
        !make_tmap_2d(&tk, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, bh * kv_stride, kDh, kDh * 2, kTile, 64) ||
        !make_tmap_2d(&tv, vt, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, bh * kDh, kv_stride,
                      static_cast<uint64_t>(kv_stride) * 2, 64, 64))
        return DH_ERR_CUDA;
    static bool configured = false;
    if (!configured) {
        if (cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kSmemBytes) != cudaSuccess)
            return DH_ERR_CUDA;
        configured = true;
    }
    AttnArgs a{sequences, q_len, kv_len, kv_stride, static_cast<__nv_bfloat16*>(out), run_flag};
    int sms = kNumSMs, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) sms = v;
    }
    const uint64_t items = static_cast<uint64_t>(sequences) * kHeads * ((q_len + kTile - 1) / kTile);
    const uint32_t grid = static_cast<uint32_t>(std::min<uint64_t>(items, 2ull * sms));
    attention_kernel<<<grid, kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, a);
    DH_LAUNCH_CHECK();
    return DH_OK;
}
