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
//   warps 2-5 softmax: one thread per query row reads its S row from TMEM,
//            keeps the running max / sum in registers (base-2 domain), writes
//            P_j (bf16) to 128-byte-swizzled shared memory as the A operand of
//            the PV MMA, and folds O_j into a register accumulator.
// 80 KB shared memory and 256 TMEM columns per CTA, so two CTAs share an SM
// and one CTA's softmax overlaps the other's MMAs.  All waits are bounded.
#include <cuda.h>
#include <cuda_bf16.h>

#include "tc_ptx.cuh"
#include "tmap.h"

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
constexpr uint32_t kSmemBytes = 1024 + kQBytes + kKBytes + kVBytes + kPBytes + 256;
constexpr uint32_t kTmemCols = 256;                   // S: [0,128), O: [128,192)
constexpr uint32_t kIdescS = tc::idesc_bf16_f32<128, 128>();
constexpr uint32_t kIdescO = tc::idesc_bf16_f32<128, 64>();

struct AttnArgs {
    uint32_t q_len, kv_len, kv_stride;
    __nv_bfloat16* out;
    const uint32_t* run_flag;
};

enum Bar : uint32_t {
    kQFull = 0, kKFull, kKEmpty, kVFull, kVEmpty, kSFull, kSFree, kPFull, kPEmpty, kOFull, kOFree,
    kDrain, kNumBars
};

DH_DEVINL void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__global__ void __launch_bounds__(kThreads, 2)
attention_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                 const __grid_constant__ CUtensorMap tv, const AttnArgs args) {
    if (args.run_flag && *args.run_flag == 0u) return;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* q_s = smem;
    uint8_t* k_s = q_s + kQBytes;
    uint8_t* v_s = k_s + kKBytes;
    uint8_t* p_s = v_s + kVBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + kPBytes);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + kNumBars);

    const uint32_t warp = warp_id(), lane = lane_id();
    const uint32_t q_tile = blockIdx.x, head = blockIdx.y, seq = blockIdx.z;
    const uint32_t bh = seq * kHeads + head;
    const uint32_t n_kv = args.kv_len / kTile;

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
        if (tc::elect_one()) {
            tc::mbar_arrive_expect_tx(&bars[kQFull], kQBytes);
            tc::tma_load_2d(q_s, &tq, &bars[kQFull], 0,
                            static_cast<int32_t>(bh * args.q_len + q_tile * kTile));
            for (uint32_t j = 0; j < n_kv; ++j) {
                const uint32_t par = (j & 1u) ^ 1u;
                if (!tc::mbar_wait(&bars[kKEmpty], par, tc::kErrTimeoutEmpty)) break;
                tc::mbar_arrive_expect_tx(&bars[kKFull], kKBytes);
                tc::tma_load_2d(k_s, &tk, &bars[kKFull], 0,
                                static_cast<int32_t>(bh * args.kv_stride + j * kTile));
                if (!tc::mbar_wait(&bars[kVEmpty], par, tc::kErrTimeoutEmpty)) break;
                tc::mbar_arrive_expect_tx(&bars[kVFull], kVBytes);
                tc::tma_load_2d(v_s, &tv, &bars[kVFull], static_cast<int32_t>(j * kTile),
                                static_cast<int32_t>(bh * kDh));
                tc::tma_load_2d(v_s + kVBytes / 2, &tv, &bars[kVFull],
                                static_cast<int32_t>(j * kTile + 64), static_cast<int32_t>(bh * kDh));
            }
            // Drain the last K / V copies before exit.
            if (n_kv > 0) {
                tc::mbar_wait(&bars[kKFull], (n_kv - 1) & 1u, tc::kErrTimeoutFull);
                tc::mbar_wait(&bars[kVFull], (n_kv - 1) & 1u, tc::kErrTimeoutFull);
            }
        }
    } else if (warp == 1) {
        if (tc::elect_one()) {
            const uint32_t s_tmem = tmem, o_tmem = tmem + 128;
            bool ok = tc::mbar_wait(&bars[kQFull], 0, tc::kErrTimeoutFull);
            const uint64_t q_desc = tc::smem_desc_sw128(q_s);
            const uint64_t k_desc = tc::smem_desc_sw128(k_s);
            for (uint32_t j = 0; j < n_kv && ok; ++j) {
                const uint32_t full = j & 1u, empty = full ^ 1u;
                ok = tc::mbar_wait(&bars[kKFull], full, tc::kErrTimeoutFull) &&
                     tc::mbar_wait(&bars[kSFree], empty, tc::kErrTimeoutAccEmpty);
                if (!ok) break;
                tc::tc_fence_after();
#pragma unroll
                for (uint32_t kk = 0; kk < kDh / 16; ++kk)
                    tc::mma_bf16(s_tmem, tc::desc_advance(q_desc, kk * 32),
                                 tc::desc_advance(k_desc, kk * 32), kIdescS, kk != 0);
                tc::mma_commit(&bars[kSFull]);
                tc::mma_commit(&bars[kKEmpty]);
                ok = tc::mbar_wait(&bars[kPFull], full, tc::kErrTimeoutFull) &&
                     tc::mbar_wait(&bars[kVFull], full, tc::kErrTimeoutFull) &&
                     tc::mbar_wait(&bars[kOFree], empty, tc::kErrTimeoutAccEmpty);
                if (!ok) break;
                tc::tc_fence_after();
#pragma unroll
                for (uint32_t kk = 0; kk < kTile / 16; ++kk) {
                    const uint32_t sub = kk >> 2, off = (kk & 3u) * 32;
                    tc::mma_bf16(o_tmem,
                                 tc::desc_advance(tc::smem_desc_sw128(p_s + sub * (kPBytes / 2)), off),
                                 tc::desc_advance(tc::smem_desc_sw128(v_s + sub * (kVBytes / 2)), off),
                                 kIdescO, kk != 0);
                }
                tc::mma_commit(&bars[kOFull]);
                tc::mma_commit(&bars[kVEmpty]);
                tc::mma_commit(&bars[kPEmpty]);
            }
            tc::mma_commit(&bars[kDrain]);
            tc::mbar_wait(&bars[kDrain], 0, tc::kErrTimeoutAccFull);
        }
    } else {
        // ----------------------------------------------------------- softmax
        const uint32_t quad = warp & 3u;
        const uint32_t r = quad * 32 + lane;  // query row within the tile
        const uint32_t lane_base = (quad * 32u) << 16;
        const float c = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
        float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
        float o[kDh];
#pragma unroll
        for (uint32_t d = 0; d < kDh; ++d) o[d] = 0.f;
        bool ok = true;
        for (uint32_t j = 0; j < n_kv && ok; ++j) {
            const uint32_t full = j & 1u, empty = full ^ 1u;
            if (!tc::mbar_wait(&bars[kSFull], full, tc::kErrTimeoutAccFull)) { ok = false; break; }
            tc::tc_fence_after();
            // pass 1: row max of this tile
            float tmax = -INFINITY;
#pragma unroll 1
            for (uint32_t cc = 0; cc < 4; ++cc) {
                uint32_t v[32];
                tc::tmem_ld_32x32b_x32(tmem + lane_base + cc * 32, v);
                tc::tmem_ld_wait();
#pragma unroll
                for (uint32_t e = 0; e < 32; ++e) tmax = fmaxf(tmax, __uint_as_float(v[e]));
            }
            const float m_new = fmaxf(m, tmax * c);
            const float alpha = exp2f(m - m_new);
            m = m_new;
            // P buffer free (previous PV finished reading it)
            if (!tc::mbar_wait(&bars[kPEmpty], empty, tc::kErrTimeoutEmpty)) { ok = false; break; }
            // pass 2: p = exp2(s*c - m), bf16 into swizzled smem
            float sum = 0.f;
#pragma unroll 1
            for (uint32_t cc = 0; cc < 4; ++cc) {
                uint32_t v[32];
                tc::tmem_ld_32x32b_x32(tmem + lane_base + cc * 32, v);
                tc::tmem_ld_wait();
                uint8_t* sub = p_s + (cc >> 1) * (kPBytes / 2) + (r >> 3) * 1024 + (r & 7u) * 128;
#pragma unroll
                for (uint32_t g = 0; g < 4; ++g) {  // 4 chunks of 8 keys
                    uint4 pk;
                    __nv_bfloat162* hp = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                    for (uint32_t e = 0; e < 4; ++e) {
                        const float p0 = exp2f(__uint_as_float(v[8 * g + 2 * e]) * c - m_new);
                        const float p1 = exp2f(__uint_as_float(v[8 * g + 2 * e + 1]) * c - m_new);
                        const __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
                        // the sum uses the rounded values the MMA will see
                        const float2 f2 = __bfloat1622float2(b2);
                        sum += f2.x + f2.y;
                        hp[e] = b2;
                    }
                    const uint32_t chunk = ((cc & 1u) * 4 + g) ^ (r & 7u);
                    *reinterpret_cast<uint4*>(sub + chunk * 16) = pk;
                }
            }
            l = l * alpha + sum;
            tc::tc_fence_before();
            tc::mbar_arrive(&bars[kSFree]);
            fence_proxy_async_smem();
            tc::mbar_arrive(&bars[kPFull]);
            // fold the previous tile's O (lagged by one tile)
            if (j > 0) {
                if (!tc::mbar_wait(&bars[kOFull], empty, tc::kErrTimeoutAccFull)) { ok = false; break; }
                tc::tc_fence_after();
                uint32_t v0[32], v1[32];
                tc::tmem_ld_32x32b_x32(tmem + lane_base + 128, v0);
                tc::tmem_ld_32x32b_x32(tmem + lane_base + 160, v1);
                tc::tmem_ld_wait();
                tc::tc_fence_before();
                tc::mbar_arrive(&bars[kOFree]);
#pragma unroll
                for (uint32_t d = 0; d < 32; ++d) {
                    o[d] = o[d] * alpha_prev + __uint_as_float(v0[d]);
                    o[d + 32] = o[d + 32] * alpha_prev + __uint_as_float(v1[d]);
                }
            }
            alpha_prev = alpha;
        }
        if (ok && n_kv > 0) {
            if (tc::mbar_wait(&bars[kOFull], (n_kv - 1) & 1u, tc::kErrTimeoutAccFull)) {
                tc::tc_fence_after();
                uint32_t v0[32], v1[32];
                tc::tmem_ld_32x32b_x32(tmem + lane_base + 128, v0);
                tc::tmem_ld_32x32b_x32(tmem + lane_base + 160, v1);
                tc::tmem_ld_wait();
#pragma unroll
                for (uint32_t d = 0; d < 32; ++d) {
                    o[d] = o[d] * alpha_prev + __uint_as_float(v0[d]);
                    o[d + 32] = o[d + 32] * alpha_prev + __uint_as_float(v1[d]);
                }
                const float inv_l = 1.0f / l;
                const uint64_t tok = static_cast<uint64_t>(seq) * args.q_len + q_tile * kTile + r;
                __nv_bfloat16* dst = args.out + tok * (kHeads * kDh) + head * kDh;
#pragma unroll
                for (uint32_t d = 0; d < kDh; d += 8) {
                    uint4 pk;
                    __nv_bfloat162* hp = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
                    for (uint32_t e = 0; e < 4; ++e)
                        hp[e] = __floats2bfloat162_rn(o[d + 2 * e] * inv_l, o[d + 2 * e + 1] * inv_l);
                    *reinterpret_cast<uint4*>(dst + d) = pk;
                }
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
    if (q_len % kTile != 0 || kv_len % kTile != 0 || kv_stride % 8 != 0)
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
    AttnArgs a{q_len, kv_len, kv_stride, static_cast<__nv_bfloat16*>(out), run_flag};
    dim3 grid(q_len / kTile, kHeads, sequences);
    attention_kernel<<<grid, kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(tq, tk, tv, a);
    DH_LAUNCH_CHECK();
    return DH_OK;
}
