// gemm.cu -- W8A8 GEMM entry points on the tcgen05 kernel (gemm_tc.cuh).
//
// dh_gemm_i8_s32 exposes the raw int32 accumulators: the tensor-engine
// contract of the reference (torch._int_mm in fixed_mlp._integer_matmul,
// src/diffusion_accel/fixed_mlp.py:55-62; the 4x8x32 HLS MAC tile,
// hls/tensor_engine/int8_mac_tile.cpp:7-41) -- bit-exact by construction.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "gemm_tc.cuh"

#include <algorithm>
#include <climits>
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
    static DH_DEVINL bool tile_begin(const Params&, TileState&, const EpiCtx&, uint32_t) { return true; }
    static DH_DEVINL void chunk(const Params& p, TileState&, const EpiCtx& ctx, uint32_t col0,
                                const uint32_t* v) {
        if (!ctx.row_ok) return;
        int32_t* dst = p.c + static_cast<uint64_t>(ctx.row) * p.ldc + col0;
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
    static DH_DEVINL void tile_end(const Params&, TileState&, const EpiCtx&) {}
};

// 16-byte global -> shared copy that bypasses the registers (cp.async).
DH_DEVINL void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
                 "l"(gmem)
                 : "memory");
}
DH_DEVINL void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// `count` (<= 128, a multiple of 4) consecutive floats from each of up to
// three per-column vectors (the warp's columns; a null source leaves its
// 512-byte slot unset) into dst.  Issued when a tile starts, so the chunks
// read them from shared memory instead of each issuing broadcast global loads.
DH_DEVINL void stage_columns(uint8_t* dst, uint32_t lane, const float* a, const float* b, const float* c,
                             uint32_t count = 128) {
    __syncwarp();  // the previous tile's chunks finished reading the slots
    if (lane * 4 < count) {
        if (a) cp_async16(dst + lane * 16, a + lane * 4);
        if (b) cp_async16(dst + 512 + lane * 16, b + lane * 4);
        if (c) cp_async16(dst + 1024 + lane * 16, c + lane * 4);
    }
    cp_async_wait_all();
    __syncwarp();
}

DH_DEVINL void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// y = acc * (a_scale[row] * w_scale[col]) + bias[col]   (fp32)
DH_DEVINL float dequant(uint32_t acc, float ab, float w, float b) {
    return __fmaf_rn(static_cast<float>(static_cast<int32_t>(acc)), ab * w, b);
}

// Staging layouts (per epilogue warp, 32 rows): a row of 128 B is 8 chunks of
// 16 B stored at chunk c ^ (row & 7); a row of 64 B is 4 chunks stored at
// c ^ ((row >> 1) & 3).  Row-owner writes and row-major reads by 8 (resp. 4)
// consecutive lanes are both bank-conflict free.
DH_DEVINL uint32_t swz128(uint32_t row, uint32_t chunk) { return row * 128 + ((chunk ^ (row & 7u)) << 4); }
DH_DEVINL uint32_t swz64(uint32_t row, uint32_t chunk) { return row * 64 + ((chunk ^ ((row >> 1) & 3u)) << 4); }

DH_DEVINL uint32_t pack_bf16x2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// QKV projection (N = 3 * 768): dequant + rotary on q and k (rotate-half,
// mlx_mdlm.py:316-329 / mdlm.py:399-410), then scatter to the attention
// layouts: Q [B, H, len, 64], K [B, H, kv_stride, 64] and V transposed
// [B, H, 64, kv_stride], all bf16.  A chunk is 64 columns = one head of one of
// q / k / v.  A warp's 32 rows are 32 consecutive tokens of one sequence, so
// its Q / K block is 4 KB contiguous and its V^T block is 64 runs of 64 bytes:
// both are written through the warp's staging buffer with full-line stores.
struct QKVParams {
    CUtensorMap q_map;   // Q as [B * 12 * seq_len, 64] bf16, box 32 x 64, 128-byte swizzle
    CUtensorMap k_map;   // K as [B * 12 * kv_stride, 64] bf16, same box
    const float* a_scale;
    const float* w_scale;
    const float* bias;
    const float* rope_cos;  // [max_pos, 32]
    const float* rope_sin;
    const float* v_scale;   // [768] per-channel factor on V (SmoothQuant 1/s of attn-out), or null
    uint32_t seq_len;       // rows per sequence in this forward
    uint32_t pos_offset;    // rotary position of the first row of a sequence
    uint32_t kv_stride;     // rows per (sequence, head) in the K / V buffers
    uint32_t kv_offset;     // where this forward's rows go in K / V
    __nv_bfloat16* q;
    __nv_bfloat16* k;
    __half* vt;  // V^T, f16
};

// kHalf: columns per epilogue warp, half the tile (128 for 128 x 256 tiles;
// 64 for the 128 x 128 tiles of a forward of one sequence).
template <uint32_t kHalf_>
struct EpiQKVT : EpiBase {
    static constexpr uint32_t kHalf = kHalf_;
    static_assert(kHalf == 64 || kHalf == 128, "a tile half is one or two heads");
    // four stages fit beside the staging buffers with 128 x 128 tiles
    static constexpr uint32_t kStages = kHalf == 64 ? 4 : 3;
    static constexpr uint32_t kChunk = 64;
    // per warp: the 4 KB source of its q / k TMA stores, then its 128
    // columns' w_scale, bias and v_scale (512 B each); 1 KB multiples keep
    // every source 1024-byte aligned for the 128-byte swizzle
    static constexpr uint32_t kStagingPerWarp = 6144;
    // Rotary rows of each lane quadrant's 32 positions, shared by the two
    // warps that cover that quadrant's rows: [quadrant][cos 4 KB | sin 4 KB],
    // row r's 16-byte piece c at swz128(r, c).
    static constexpr uint32_t kExtraSmem = 4 * 8192;
    using Params = QKVParams;
    struct TileState {
        float ab;  // a_scale of this thread's row
    };
    // Row scale; for q / k tiles, the quadrant's 32 rotary rows (positions
    // t0 .. t0+31, contiguous in the tables) are copied into shared memory
    // with coalesced asynchronous copies -- one warp of the pair copies the
    // cos rows, the other the sin rows -- instead of per-lane row loads in
    // every chunk.  Both halves of a 256-column tile are q, k or v alike, so
    // the pair agrees on the branch and on the named barriers.
    static DH_DEVINL bool tile_begin(const Params& p, TileState& st, const EpiCtx& ctx, uint32_t col_start) {
        st.ab = ctx.row_ok ? p.a_scale[ctx.row] : 0.f;
        // the warp's 128 columns of w_scale / bias (/ v_scale, indexed from 0 at the v block)
        stage_columns(ctx.stage + 4096, ctx.lane, p.w_scale + col_start, p.bias + col_start,
                      col_start >= 1536u && p.v_scale ? p.v_scale + (col_start - 1536u) : nullptr, kHalf);
        if (col_start >= 1536u) return true;
        const uint32_t quad = (ctx.row0 / 32u) & 3u;
        const uint32_t half = static_cast<uint32_t>(ctx.stage - ctx.extra - kExtraSmem) / kStagingPerWarp / 4u;
        uint8_t* buf = ctx.extra + quad * 8192u + half * 4096u;
        // the pair finished reading the previous tile's rows
        if (!tc::mbar_arrive_wait(ctx.pair_bar, tc::kErrTimeoutPair)) return false;
        if (ctx.row0 < ctx.m_eff) {
            const float* table = (half == 0 ? p.rope_cos : p.rope_sin) +
                                 static_cast<uint64_t>(ctx.row0 % p.seq_len + p.pos_offset) * 32;
#pragma unroll
            for (uint32_t i = 0; i < 8; ++i) {  // 256 pieces of 16 B, 32 per instruction
                const uint32_t piece = i * 32 + ctx.lane;
                cp_async16(buf + swz128(piece >> 3, piece & 7u), table + piece * 4);
            }
        }
        cp_async_wait_all();
        return tc::mbar_arrive_wait(ctx.pair_bar, tc::kErrTimeoutPair);  // both tables landed
    }
    static DH_DEVINL void chunk(const Params& p, TileState& st, const EpiCtx& ctx, uint32_t col0,
                                const uint32_t* v) {
        constexpr uint32_t heads = 12;
        const float ab = st.ab;
        const uint32_t which = col0 / 768u;
        const uint32_t h = (col0 % 768u) / 64u;
        float y[64];
        const uint32_t cw = (col0 % kHalf) * 4u;  // byte offset of this chunk in the warp's parameters
        const float4* w4 = reinterpret_cast<const float4*>(ctx.stage + 4096 + cw);
        const float4* b4 = reinterpret_cast<const float4*>(ctx.stage + 4096 + 512 + cw);
#pragma unroll
        for (uint32_t j = 0; j < 16; ++j) {
            const float4 w = w4[j], bb = b4[j];
            y[4 * j] = dequant(v[4 * j], ab, w.x, bb.x);
            y[4 * j + 1] = dequant(v[4 * j + 1], ab, w.y, bb.y);
            y[4 * j + 2] = dequant(v[4 * j + 2], ab, w.z, bb.z);
            y[4 * j + 3] = dequant(v[4 * j + 3], ab, w.w, bb.w);
        }
        const uint32_t b = ctx.row0 / p.seq_len;
        const uint32_t t0 = ctx.row0 % p.seq_len;
        const uint32_t lane = ctx.lane;
        // The warp's 32 rows lie in one sequence and are all valid or all
        // past m_eff (both multiples of 32).
        const bool live = ctx.row0 < ctx.m_eff;
        if (which < 2) {
            // q / k chunk: staged in shared memory (128-byte swizzle), then one
            // TMA store, once the previous chunk's store has read the buffer
            uint8_t* src = ctx.stage;
            if (lane == 0) tc::tma_store_wait_read<0>();
            __syncwarp();
            const uint8_t* rope = ctx.extra + ((ctx.row0 / 32u) & 3u) * 8192u;
#pragma unroll
            for (uint32_t i4 = 0; i4 < 8; ++i4) {
                const float4 c4 = *reinterpret_cast<const float4*>(rope + swz128(lane, i4));
                const float4 s4 = *reinterpret_cast<const float4*>(rope + 4096 + swz128(lane, i4));
                const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
                const float ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                for (uint32_t e = 0; e < 4; ++e) {
                    const uint32_t i = 4 * i4 + e;
                    const float x1 = y[i], x2 = y[i + 32];
                    y[i] = x1 * cc[e] - x2 * ss[e];
                    y[i + 32] = x2 * cc[e] + x1 * ss[e];
                }
            }
#pragma unroll
            for (uint32_t w = 0; w < 32; w += 4)
                *reinterpret_cast<uint4*>(src + swz128(lane, w / 4)) =
                    make_uint4(pack_bf16x2(y[2 * w], y[2 * w + 1]), pack_bf16x2(y[2 * w + 2], y[2 * w + 3]),
                               pack_bf16x2(y[2 * w + 4], y[2 * w + 5]), pack_bf16x2(y[2 * w + 6], y[2 * w + 7]));
            if (live) {
                // rows of (b, h) at position pos0.. in Q [.., seq_len, 64] or K [.., kv_stride, 64]
                const uint32_t len = which == 0 ? p.seq_len : p.kv_stride;
                const uint32_t pos0 = which == 0 ? t0 : t0 + p.kv_offset;
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tc::tma_store_2d(which == 0 ? &p.q_map : &p.k_map, src, 0,
                                     static_cast<int32_t>((b * heads + h) * len + pos0));
                    tc::tma_store_commit();
                }
            }
            __syncwarp();
        } else {
            if (p.v_scale) {
                const float4* vs4 = reinterpret_cast<const float4*>(ctx.stage + 4096 + 1024 + cw);
#pragma unroll
                for (uint32_t j = 0; j < 16; ++j) {
                    const float4 f = vs4[j];
                    y[4 * j] *= f.x;
                    y[4 * j + 1] *= f.y;
                    y[4 * j + 2] *= f.z;
                    y[4 * j + 3] *= f.w;
                }
            }
            // V^T: for each channel d the warp's 32 consecutive tokens form
            // one 64-byte run, so lane = token stores are already coalesced
            // (measured faster than staging the transpose through shared
            // memory, which the tensor core's operand reads also use).
            if (live) {
                __half* dst = p.vt + (static_cast<uint64_t>(b) * heads + h) * 64 * p.kv_stride + t0 + lane +
                              p.kv_offset;
#pragma unroll
                for (uint32_t d = 0; d < 64; ++d)
                    dst[static_cast<uint64_t>(d) * p.kv_stride] = __float2half_rn(y[d]);
            }
        }
    }
    static DH_DEVINL void tile_end(const Params&, TileState&, const EpiCtx&) {}
    static DH_DEVINL void finish(uint32_t lane) {
        if (lane == 0) tc::tma_store_wait_all();
    }
};
using EpiQKV = EpiQKVT<128>;
using EpiQKVNarrow = EpiQKVT<64>;

// x[row, col] += acc * (a_scale * w_scale) + bias  (attention out, MLP down).
// The residual read-modify-write goes through the staging buffer with one
// 128-byte row segment per warp instruction.
template <uint32_t kStages_, uint32_t kHalfCols_, bool kPrefetchNext_ = false, uint32_t kAhead_ = 1>
struct EpiResidualT : EpiBase {
    static constexpr uint32_t kStages = kStages_;
    static constexpr uint32_t kHalfCols = kHalfCols_;  // columns per epilogue warp (half the tile)
    static constexpr bool kPrefetchNext = kPrefetchNext_;
    // x chunks in flight ahead of the one being summed (1 or 2)
    static constexpr uint32_t kAhead = kAhead_;
    static_assert(kAhead == 1 || kAhead == 2, "one or two chunks ahead");
    static constexpr uint32_t kChunk = 32;
    // per warp: dequant staging (4 KB), then its 128 columns' w_scale and bias
    static constexpr uint32_t kStagingPerWarp = 32 * 128 + 2 * 512;
    struct Params {
        const float* a_scale;
        const float* w_scale;
        const float* bias;  // may be null
        float* x;
        uint32_t n;
    };
    // x is loaded kAhead chunks ahead (the first kAhead chunks before the
    // accumulator is ready), chunk k into slot k % kAhead: lane -> (row
    // i*4 + lane/8, 4 columns).
    struct TileState {
        float4 xv[kAhead][8];
        uint32_t col_end;
        float ab;
    };
    static DH_DEVINL void load_into(const Params& p, float4 (&dst)[8], const EpiCtx& ctx, uint32_t col0) {
        const uint32_t cq = (ctx.lane & 7u) * 4;
#pragma unroll
        for (uint32_t i = 0; i < 8; ++i) {
            const uint32_t rr = i * 4 + (ctx.lane >> 3);
            if (ctx.row0 + rr < ctx.m_eff)
                dst[i] = *reinterpret_cast<const float4*>(p.x + static_cast<uint64_t>(ctx.row0 + rr) * p.n + col0 + cq);
        }
    }
    static DH_DEVINL void load_x(const Params& p, TileState& st, const EpiCtx& ctx, uint32_t col0, uint32_t slot) {
        if (kAhead == 2 && slot)
            load_into(p, st.xv[kAhead - 1], ctx, col0);
        else
            load_into(p, st.xv[0], ctx, col0);
    }
    static DH_DEVINL bool tile_begin(const Params& p, TileState& st, const EpiCtx& ctx, uint32_t col_start) {
        st.col_end = col_start + kHalfCols;
        st.ab = ctx.row_ok ? p.a_scale[ctx.row] : 0.f;
        load_x(p, st, ctx, col_start, 0);
        if (kAhead == 2 && kHalfCols > 32) load_x(p, st, ctx, col_start + 32, 1);
        stage_columns(ctx.stage + 4096, ctx.lane, p.w_scale + col_start, p.bias ? p.bias + col_start : nullptr,
                      nullptr, kHalfCols);
        // The residual rows of this warp's next tile start towards L2 now,
        // a whole tile ahead of their loads.  For K = 768 the epilogue, not
        // the tensor core, sets the pace, so DRAM latency would be exposed;
        // at K = 3072 the tile is long enough that this only adds traffic.
        if (kPrefetchNext && ctx.has_next && ctx.next_row0 + ctx.lane < ctx.m_eff) {
            const char* r = reinterpret_cast<const char*>(p.x + static_cast<uint64_t>(ctx.next_row0 + ctx.lane) * p.n +
                                                          ctx.next_col);
#pragma unroll
            for (uint32_t b = 0; b < kHalfCols * 4; b += 128)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(r + b));
        }
        return true;
    }
    static DH_DEVINL void chunk(const Params& p, TileState& st, const EpiCtx& ctx, uint32_t col0,
                                const uint32_t* v) {
        const float ab = st.ab;
        const uint32_t lane = ctx.lane;
        const uint8_t* prm = ctx.stage + 4096 + (col0 % kHalfCols) * 4u;
#pragma unroll
        for (uint32_t j = 0; j < 32; j += 4) {
            const float4 w = *reinterpret_cast<const float4*>(prm + j * 4);
            float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
            if (p.bias) bb = *reinterpret_cast<const float4*>(prm + 512 + j * 4);
            *reinterpret_cast<float4*>(ctx.stage + swz128(lane, j / 4)) =
                make_float4(dequant(v[j], ab, w.x, bb.x), dequant(v[j + 1], ab, w.y, bb.y),
                            dequant(v[j + 2], ab, w.z, bb.z), dequant(v[j + 3], ab, w.w, bb.w));
        }
        __syncwarp();
        const uint32_t cq = (lane & 7u) * 4;
        const uint32_t slot = kAhead == 2 ? ((col0 % kHalfCols) / 32u) & 1u : 0u;
        float4 out[8];
#pragma unroll
        for (uint32_t i = 0; i < 8; ++i) {
            const uint32_t rr = i * 4 + (lane >> 3);
            const float4 y = *reinterpret_cast<const float4*>(ctx.stage + swz128(rr, lane & 7u));
            const float4 xv = slot ? st.xv[kAhead - 1][i] : st.xv[0][i];
            out[i] = make_float4(xv.x + y.x, xv.y + y.y, xv.z + y.z, xv.w + y.w);
        }
        __syncwarp();
        // the chunk kAhead ahead, in flight during the stores
        if (col0 + 32 * kAhead < st.col_end) load_x(p, st, ctx, col0 + 32 * kAhead, slot);
#pragma unroll
        for (uint32_t i = 0; i < 8; ++i) {
            const uint32_t rr = i * 4 + (lane >> 3);
            if (ctx.row0 + rr < ctx.m_eff)
                *reinterpret_cast<float4*>(p.x + static_cast<uint64_t>(ctx.row0 + rr) * p.n + col0 + cq) = out[i];
        }
    }
    static DH_DEVINL void tile_end(const Params&, TileState&, const EpiCtx&) {}
};
// N = 768 runs as 4 column tiles of 192: 1,024 tiles fill 6.9 waves of 148 SMs
// (128 x 256 tiles would leave the 6th wave 19% full).
// K = 768: x two chunks ahead (53.4 -> 49.5 us at 32,768 rows); at K = 3072
// the mainloop is long enough that one chunk ahead is as fast.
using EpiResidual = EpiResidualT<3, 96, true, 2>;  // K = 768
using EpiResidualDeep = EpiResidualT<4, 96>;  // K = 3072: deeper TMA pipeline
using EpiResidual256 = EpiResidualT<3, 128>;  // other N, multiples of 256
// 128 x 64 tiles for a forward of few rows, where 128 x 192 tiles would
// leave most SMs idle (1,024 rows: 32 tiles; 128 x 64: 96)
// The 128 x 64 tiles run where each CTA holds about one tile, so the first
// tile's loads are all the pipeline sees: it keeps 6 (K = 768: the whole of
// K) or 7 stages of 24 KB in flight.
using EpiResidualNarrow = EpiResidualT<6, 32, true, 1>;  // K = 768
using EpiResidualNarrowDeep = EpiResidualT<7, 32>;       // K = 3072

DH_DEVINL float gelu_tanh(float x) {
    // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))   (nn.GELU(approx="tanh"))
    const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
    float t;
    asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
    return 0.5f * x * (1.0f + t);
}

// out[row, col] = bf16(gelu_tanh(acc * (a_scale * w_scale) + bias) * out_scale)
// (MLP up).  Each 32 x 32 chunk is written into a 64-byte-swizzled shared
// buffer and stored by the TMA unit; reading the buffer back through the
// registers would double the epilogue's shared-memory traffic, which competes
// with the tensor core's operand reads.  Two epilogue warp groups.
struct EpiGelu : EpiBase {
    static constexpr uint32_t kStages = 3;
    static constexpr uint32_t kGroups = 2;
    static constexpr uint32_t kChunk = 32;
    static constexpr uint32_t kMaxCols = 3584;
    // CTA-wide: w_scale, bias and out_scale of every column, copied in once
    // when the CTA starts (no per-tile staging wait), then one slot of 32
    // row scales per epilogue warp that carries the next tile's a_scale
    static constexpr uint32_t kTableBytes = 3 * kMaxCols * 4;
    static constexpr uint32_t kExtraSmem = kTableBytes + 16 * 128;
    // per warp: the 2 KB source of its TMA stores (1 KB multiples keep it
    // aligned for the swizzle)
    static constexpr uint32_t kStagingPerWarp = 2048;
    struct Params {
        CUtensorMap out_map;  // out as [m, n] bf16, box 32 x 32, 64-byte swizzle
        const float* a_scale;
        const float* w_scale;
        const float* bias;
        const float* out_scale;  // per-column factor (SmoothQuant 1/s of the next linear) or null
        __nv_bfloat16* out;
        uint32_t n;
        // or null: per output row, the bits of max |out| over the row (as
        // stored, bf16) are merged in with atomicMax -- the row amax the
        // per-token quantiser of the next linear needs, so that it reads the
        // row once; the buffer must hold 0 (the quantiser clears it again)
        uint32_t* row_amax;
    };
    struct TileState {
        float ab;
        __nv_bfloat162 amax2;  // running max |out| of this thread's row over the tile's chunks
    };
    static DH_DEVINL void init_smem(const Params& p, uint8_t* extra, uint32_t tid, uint32_t count) {
        const uint32_t pieces = p.n / 4;  // 16-byte pieces per vector
        for (uint32_t i = tid; i < 3 * pieces; i += count) {
            const uint32_t v = i / pieces, j = i % pieces;
            const float* src = v == 0 ? p.w_scale : (v == 1 ? p.bias : p.out_scale);
            if (src) cp_async16(extra + v * (kMaxCols * 4) + j * 16, src + j * 4);
        }
        cp_async_wait_all();
    }
    static DH_DEVINL float* carry_slot(const EpiCtx& ctx) {
        const uint32_t ew = static_cast<uint32_t>(ctx.stage - (ctx.extra + kExtraSmem)) / kStagingPerWarp;
        return reinterpret_cast<float*>(ctx.extra + kTableBytes + ew * 128);
    }
    // Row scale of this tile (carried from the previous tile's prefetch), and
    // an asynchronous copy of the next tile's row scales into the carry slot.
    static DH_DEVINL bool tile_begin(const Params& p, TileState& st, const EpiCtx& ctx, uint32_t) {
        st.amax2 = __float2bfloat162_rn(0.f);
        float* carry = carry_slot(ctx);
        if (ctx.first_tile) {
            st.ab = ctx.row_ok ? p.a_scale[ctx.row] : 0.f;
        } else {
            cp_async_wait_all();
            __syncwarp();
            st.ab = carry[ctx.lane];
        }
        __syncwarp();
        if (ctx.has_next && ctx.next_row0 + ctx.lane < ctx.m_eff)
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                             static_cast<uint32_t>(__cvta_generic_to_shared(carry + ctx.lane))),
                         "l"(p.a_scale + ctx.next_row0 + ctx.lane)
                         : "memory");
        return true;
    }
    static DH_DEVINL void chunk(const Params& p, TileState& st, const EpiCtx& ctx, uint32_t col0,
                                const uint32_t* v) {
        const float ab = st.ab;
        const uint32_t lane = ctx.lane;
        uint32_t pk[16];
        const float4* w4 = reinterpret_cast<const float4*>(ctx.extra + col0 * 4u);
        const float4* b4 = reinterpret_cast<const float4*>(ctx.extra + kMaxCols * 4 + col0 * 4u);
        const float4* o4 = reinterpret_cast<const float4*>(ctx.extra + 2 * kMaxCols * 4 + col0 * 4u);
        // two columns per packed fp32x2 instruction:
        //   x = acc * (a_scale * w_scale) + bias
        //   u = k c x^3 + k x                (k = sqrt(2/pi), c = 0.044715)
        //   g = h tanh(u) + h,  h = x * (out_scale / 2)
        const float2 ab2 = make_float2(ab, ab);
        const float2 kc2 = make_float2(0.7978845608028654f * 0.044715f, 0.7978845608028654f * 0.044715f);
        const float2 k2 = make_float2(0.7978845608028654f, 0.7978845608028654f);
        const float2 half2 = make_float2(0.5f, 0.5f);
#pragma unroll
        for (uint32_t q = 0; q < 8; ++q) {
            const float4 w = w4[q], bb = b4[q];
            const float4 os = p.out_scale ? o4[q] : make_float4(1.f, 1.f, 1.f, 1.f);
#pragma unroll
            for (uint32_t hh = 0; hh < 2; ++hh) {
                const float2 wv = hh ? make_float2(w.z, w.w) : make_float2(w.x, w.y);
                const float2 bv = hh ? make_float2(bb.z, bb.w) : make_float2(bb.x, bb.y);
                const float2 ov = hh ? make_float2(os.z, os.w) : make_float2(os.x, os.y);
                const float2 acc = make_float2(static_cast<float>(static_cast<int32_t>(v[4 * q + 2 * hh])),
                                               static_cast<float>(static_cast<int32_t>(v[4 * q + 2 * hh + 1])));
                const float2 x = __ffma2_rn(acc, __fmul2_rn(ab2, wv), bv);
                const float2 t1 = __fmul2_rn(__fmul2_rn(x, x), kc2);
                const float2 u = __ffma2_rn(t1, x, __fmul2_rn(x, k2));
                float2 t;
                asm("tanh.approx.f32 %0, %1;" : "=f"(t.x) : "f"(u.x));
                asm("tanh.approx.f32 %0, %1;" : "=f"(t.y) : "f"(u.y));
                const float2 h = __fmul2_rn(x, __fmul2_rn(ov, half2));
                const float2 g = __ffma2_rn(h, t, h);
                pk[2 * q + hh] = pack_bf16x2(g.x, g.y);
            }
        }
        if (p.row_amax) {
#pragma unroll
            for (uint32_t w = 0; w < 16; ++w)
                st.amax2 = __hmax2(st.amax2, __habs2(*reinterpret_cast<const __nv_bfloat162*>(&pk[w])));
        }
        uint8_t* src = ctx.stage;
        if (lane == 0) tc::tma_store_wait_read<0>();  // the previous chunk's store has read `src`
        __syncwarp();
#pragma unroll
        for (uint32_t w = 0; w < 16; w += 4)
            *reinterpret_cast<uint4*>(src + swz64(lane, w / 4)) = make_uint4(pk[w], pk[w + 1], pk[w + 2], pk[w + 3]);
        if (ctx.row0 + 32 <= ctx.m_eff) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                tc::tma_store_2d(&p.out_map, src, static_cast<int32_t>(col0), static_cast<int32_t>(ctx.row0));
                tc::tma_store_commit();
            }
        } else {
            // ragged last rows: store only the valid ones through the registers
            __syncwarp();
#pragma unroll
            for (uint32_t i = 0; i < 4; ++i) {
                const uint32_t rr = i * 8 + (lane >> 2);
                const uint32_t r = ctx.row0 + rr;
                if (r < ctx.m_eff)
                    *reinterpret_cast<uint4*>(p.out + static_cast<uint64_t>(r) * p.n + col0 + (lane & 3u) * 8) =
                        *reinterpret_cast<const uint4*>(src + swz64(rr, lane & 3u));
            }
            __syncwarp();
        }
    }
    static DH_DEVINL void tile_end(const Params& p, TileState& st, const EpiCtx& ctx) {
        // non-negative floats order like their bit patterns
        if (p.row_amax && ctx.row_ok)
            atomicMax(p.row_amax + ctx.row,
                      __float_as_uint(fmaxf(__low2float(st.amax2), __high2float(st.amax2))));
    }
    static DH_DEVINL void finish(uint32_t lane) {
        if (lane == 0) tc::tma_store_wait_all();
    }
};

// 128 x 128 MLP-up tiles (one per epilogue group and CTA): a fourth stage fits.
struct EpiGeluNarrow : EpiGelu {
    static constexpr uint32_t kStages = 4;
};

// Integer requantisation of the int32 accumulators, the RTL form of
// fixed_mlp.hardware_requantized_linear (fixed_mlp.py:139-224):
//   mult = rint(double(fp32(a_scale[r] * w_scale[c])) * 2^(shift + frac))   (mode 0)
//   mult = (token_factor[r] * output_factor[c] + 2^(fs-1)) >> fs              (mode 1,
//          the factorised multipliers of fixed_mlp.factorize_up_requant_scales, :327-392)
//   p = acc * mult (int64);  q = sign(p) * ((|p| + 2^(shift-1)) >> shift)
//   out = clamp(q + bias_q[c], lo, hi)   (int32)
// Statistics (accumulator range, saturated outputs, largest multiplier) are
// merged into stats[4] with one atomic per warp and chunk.
struct EpiRequantQ : EpiBase {
    static constexpr uint32_t kChunk = 32;
    struct Params {
        uint32_t mode;
        const float* a_scale;
        uint32_t a_scale_stride;  // 1: per row, 0: one tensor scale
        const float* w_scale;
        const int32_t* token_factor;
        const int32_t* output_factor;
        uint32_t factor_shift;
        const int32_t* bias_q;
        double mult_scale;  // 2^(shift + frac)
        uint32_t shift;
        long long lo, hi;
        int32_t* out;
        uint32_t n;
        long long* stats;  // [min acc, max acc, saturated count, max multiplier]
    };
    struct TileState {};
    static DH_DEVINL bool tile_begin(const Params&, TileState&, const EpiCtx&, uint32_t) { return true; }
    static DH_DEVINL void chunk(const Params& p, TileState&, const EpiCtx& ctx, uint32_t col0,
                                const uint32_t* v) {
        long long acc_min = LLONG_MAX, acc_max = LLONG_MIN, sat = 0, mult_max = 0;
        if (ctx.row_ok) {
            const float as = p.a_scale ? p.a_scale[p.a_scale_stride ? ctx.row : 0u] : 0.f;
            const long long tf = p.token_factor ? p.token_factor[ctx.row] : 0;
            int32_t* dst = p.out + static_cast<uint64_t>(ctx.row) * p.n;
            const long long half = 1ll << (p.shift - 1);
            for (uint32_t j = 0; j < 32; ++j) {
                const uint32_t c = col0 + j;
                if (c >= p.n) break;
                long long mult;
                if (p.mode == 0) {
                    const float prod = __fmul_rn(as, p.w_scale[c]);
                    mult = __double2ll_rn(static_cast<double>(prod) * p.mult_scale);
                } else {
                    mult = (tf * static_cast<long long>(p.output_factor[c]) + (1ll << (p.factor_shift - 1))) >>
                           p.factor_shift;
                }
                const long long acc = static_cast<int32_t>(v[j]);
                const long long prd = acc * mult;
                const long long mag = ((prd < 0 ? -prd : prd) + half) >> p.shift;
                long long o = (prd < 0 ? -mag : mag) + p.bias_q[c];
                if (o < p.lo || o > p.hi) {
                    ++sat;
                    o = o < p.lo ? p.lo : p.hi;
                }
                dst[c] = static_cast<int32_t>(o);
                acc_min = acc < acc_min ? acc : acc_min;
                acc_max = acc > acc_max ? acc : acc_max;
                mult_max = mult > mult_max ? mult : mult_max;
            }
        }
        // warp merge, then one atomic per statistic
        for (int o = 16; o > 0; o >>= 1) {
            acc_min = min(acc_min, __shfl_xor_sync(0xFFFFFFFFu, acc_min, o));
            acc_max = max(acc_max, __shfl_xor_sync(0xFFFFFFFFu, acc_max, o));
            sat += __shfl_xor_sync(0xFFFFFFFFu, sat, o);
            mult_max = max(mult_max, __shfl_xor_sync(0xFFFFFFFFu, mult_max, o));
        }
        if (ctx.lane == 0 && p.stats && acc_min <= acc_max) {
            atomicMin(p.stats, acc_min);
            atomicMax(p.stats + 1, acc_max);
            atomicAdd(reinterpret_cast<unsigned long long*>(p.stats + 2), static_cast<unsigned long long>(sat));
            atomicMax(p.stats + 3, mult_max);
        }
    }
    static DH_DEVINL void tile_end(const Params&, TileState&, const EpiCtx&) {}
};

// The RTL Q5.10 GELU (fixed_mlp.hardware_gelu_q10, fixed_mlp.py:227-247):
// lut[clamp((q + 8192) >> 4, 0, 1023)], 0 at or below -8192, q itself at or
// above 8192.  The 1024-entry table comes from the caller.
__global__ void gelu_q10_kernel(const int32_t* __restrict__ in, int32_t* __restrict__ out, uint64_t count,
                                const int32_t* __restrict__ lut) {
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const int32_t q = in[i];
        int32_t r;
        if (q <= -8192) r = 0;
        else if (q >= 8192) r = q;
        else r = lut[(q + 8192) >> 4];
        out[i] = r;
    }
}

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
                                     const float* rope_sin, const float* v_scale, uint32_t m, uint32_t seq_len,
                                     uint32_t pos_offset, uint32_t kv_stride, uint32_t kv_offset,
                                     void* q, void* k, void* vt, const uint32_t* run_rows,
                                     void* stream) {
    if (!a_scale || !w_scale || !bias || !rope_cos || !rope_sin || !q || !k || !vt)
        return DH_ERR_NULL_POINTER;
    if (seq_len == 0 || m % seq_len != 0 || kv_offset + seq_len > kv_stride)
        return DH_ERR_INVALID_ARGUMENT;
    // a warp's 32 rows must lie in one sequence
    if (seq_len % 32 != 0) return DH_ERR_UNSUPPORTED_SHAPE;
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
         reinterpret_cast<uintptr_t>(w_scale) | reinterpret_cast<uintptr_t>(bias) |
         reinterpret_cast<uintptr_t>(rope_cos) | reinterpret_cast<uintptr_t>(rope_sin) |
         reinterpret_cast<uintptr_t>(v_scale)) & 15u)
        return DH_ERR_ALIGNMENT;
    // 128 x 128 tiles when they fit one wave of the SMs (a forward of one
    // sequence: 144 tiles instead of 72), else 128 x 256
    int sms = kNumSMs, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t bn = ((m + 127) / 128) * (2304 / 128) <= static_cast<uint32_t>(sms) ? 128u : 256u;
    CUtensorMap ta, tb;
    uint32_t st = make_i8_operand_maps(&ta, &tb, a, 768, w, 768, m, 2304, 768, bn);
    if (st != DH_OK) return st;
    const uint64_t bh = static_cast<uint64_t>(m / seq_len) * 12;
    EpiQKV::Params p{};
    if (!make_tmap_2d(&p.q_map, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, bh * seq_len, 64, 128, 32, 64) ||
        !make_tmap_2d(&p.k_map, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, bh * kv_stride, 64, 128, 32, 64))
        return DH_ERR_CUDA;
    p.a_scale = a_scale;
    p.w_scale = w_scale;
    p.bias = bias;
    p.rope_cos = rope_cos;
    p.rope_sin = rope_sin;
    p.v_scale = v_scale;
    p.seq_len = seq_len;
    p.pos_offset = pos_offset;
    p.kv_stride = kv_stride;
    p.kv_offset = kv_offset;
    p.q = static_cast<__nv_bfloat16*>(q);
    p.k = static_cast<__nv_bfloat16*>(k);
    p.vt = static_cast<__half*>(vt);
    GemmShape shape{m, 2304, 768, run_rows};
    const uint32_t tiles = ((m + 127) / 128) * (2304 / bn);
    const cudaError_t e = bn == 128
        ? launch_gemm_i8<128, EpiQKVNarrow>(ta, tb, shape, p, tiles, static_cast<cudaStream_t>(stream))
        : launch_gemm_i8<256, EpiQKV>(ta, tb, shape, p, tiles, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return DH_ERR_CUDA;
    return DH_OK;
}

extern "C" uint32_t dh_gemm_residual(const int8_t* a, const float* a_scale, const int8_t* w,
                                     const float* w_scale, const float* bias, float* x, uint32_t m,
                                     uint32_t n, uint32_t k, const uint32_t* run_rows,
                                     void* stream) {
    if (!a_scale || !w_scale || !x) return DH_ERR_NULL_POINTER;
    if (n % 192 != 0 && n % 256 != 0) return DH_ERR_UNSUPPORTED_SHAPE;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w_scale) |
         reinterpret_cast<uintptr_t>(bias)) & 15u)
        return DH_ERR_ALIGNMENT;
    uint32_t bn = n % 192 == 0 ? 192u : 256u;
    // when even the 128 x 64 tiles fit one wave of the SMs, they spread the
    // rows over three (or four) times as many SMs (one 1,024-row sequence:
    // 96 tiles instead of 32, 853 -> 737 us per forward); with more rows the
    // wide tiles' shorter epilogue per byte wins (4 sequences: 1,282 against
    // 1,375 us with narrow tiles)
    int sms = kNumSMs, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (((m + 127) / 128) * (n / 64) <= static_cast<uint32_t>(sms)) bn = 64;
    CUtensorMap ta, tb;
    uint32_t st = make_i8_operand_maps(&ta, &tb, a, k, w, k, m, n, k, bn);
    if (st != DH_OK) return st;
    GemmShape shape{m, n, k, run_rows};
    const uint32_t tiles = ((m + 127) / 128) * (n / bn);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (bn == 64) {
        if (k > 1024)
            e = launch_gemm_i8<64, EpiResidualNarrowDeep>(ta, tb, shape, {a_scale, w_scale, bias, x, n}, tiles, s);
        else
            e = launch_gemm_i8<64, EpiResidualNarrow>(ta, tb, shape, {a_scale, w_scale, bias, x, n}, tiles, s);
    } else if (bn == 256) {
        e = launch_gemm_i8<256, EpiResidual256>(ta, tb, shape, {a_scale, w_scale, bias, x, n}, tiles, s);
    } else if (k > 1024) {
        e = launch_gemm_i8<192, EpiResidualDeep>(ta, tb, shape, {a_scale, w_scale, bias, x, n}, tiles, s);
    } else {
        e = launch_gemm_i8<192, EpiResidual>(ta, tb, shape, {a_scale, w_scale, bias, x, n}, tiles, s);
    }
    if (e != cudaSuccess) return DH_ERR_CUDA;
    return DH_OK;
}

extern "C" uint32_t dh_gemm_gelu(const int8_t* a, const float* a_scale, const int8_t* w,
                                 const float* w_scale, const float* bias, const float* out_scale,
                                 void* out, uint32_t* row_amax, uint32_t m,
                                 uint32_t n, uint32_t k, const uint32_t* run_rows, void* stream) {
    if (!a_scale || !w_scale || !bias || !out) return DH_ERR_NULL_POINTER;
    if (n % 256 != 0 || n > EpiGelu::kMaxCols) return DH_ERR_UNSUPPORTED_SHAPE;
    if ((reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(w_scale) |
         reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(out_scale)) & 15u)
        return DH_ERR_ALIGNMENT;
    // when 128 x 128 tiles give every CTA at most one tile per epilogue
    // group (one 1,024-row sequence: 192 tiles on 148 SMs), the two groups
    // drain them side by side where 128 x 256 tiles leave one group idle
    int sms = kNumSMs, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t bn = ((m + 127) / 128) * (n / 128) <= 2u * static_cast<uint32_t>(sms) ? 128u : 256u;
    CUtensorMap ta, tb;
    uint32_t st = make_i8_operand_maps(&ta, &tb, a, k, w, k, m, n, k, bn);
    if (st != DH_OK) return st;
    EpiGelu::Params p{};
    if (!make_tmap_2d_sw64(&p.out_map, out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m, n,
                           static_cast<uint64_t>(n) * 2, 32, 32))
        return DH_ERR_CUDA;
    p.a_scale = a_scale;
    p.w_scale = w_scale;
    p.bias = bias;
    p.out_scale = out_scale;
    p.out = static_cast<__nv_bfloat16*>(out);
    p.n = n;
    p.row_amax = row_amax;
    GemmShape shape{m, n, k, run_rows};
    const uint32_t tiles = ((m + 127) / 128) * (n / bn);
    const cudaError_t e = bn == 128
        ? launch_gemm_i8<128, EpiGeluNarrow>(ta, tb, shape, p, tiles, static_cast<cudaStream_t>(stream))
        : launch_gemm_i8<256, EpiGelu>(ta, tb, shape, p, tiles, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return DH_ERR_CUDA;
    return DH_OK;
}

extern "C" uint32_t dh_gemm_i8_requant(const int8_t* a, const int8_t* w, uint32_t m, uint32_t n, uint32_t k,
                                      uint32_t mode, const float* a_scale, uint32_t a_scale_stride,
                                      const float* w_scale, const int32_t* token_factor,
                                      const int32_t* output_factor, uint32_t factor_shift, const int32_t* bias_q,
                                      uint32_t right_shift, uint32_t frac_bits, uint32_t output_width,
                                      int32_t* out, int64_t* stats, void* stream) {
    if (!out || !bias_q) return DH_ERR_NULL_POINTER;
    if (mode == 0 && (!a_scale || !w_scale)) return DH_ERR_NULL_POINTER;
    if (mode == 1 && (!token_factor || !output_factor)) return DH_ERR_NULL_POINTER;
    if (mode > 1 || a_scale_stride > 1 || right_shift == 0 || right_shift > 40 || output_width > 32 ||
        output_width <= frac_bits + 1 || (mode == 1 && (factor_shift == 0 || factor_shift > 40)))
        return DH_ERR_INVALID_ARGUMENT;
    if (right_shift + frac_bits > 62) return DH_ERR_INVALID_ARGUMENT;
    CUtensorMap ta, tb;
    uint32_t st = make_i8_operand_maps(&ta, &tb, a, k, w, k, m, n, k, 256);
    if (st != DH_OK) return st;
    EpiRequantQ::Params p{mode, a_scale, a_scale_stride, w_scale, token_factor, output_factor, factor_shift,
                          bias_q, static_cast<double>(1ull << (right_shift + frac_bits)), right_shift,
                          -(1ll << (output_width - 1)), (1ll << (output_width - 1)) - 1, out, n,
                          reinterpret_cast<long long*>(stats)};
    GemmShape shape{m, n, k, nullptr};
    const uint32_t tiles = ((m + 127) / 128) * ((n + 255) / 256);
    if (launch_gemm_i8<256, EpiRequantQ>(ta, tb, shape, p, tiles, static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return DH_ERR_CUDA;
    return DH_OK;
}

extern "C" uint32_t dh_gelu_q10(const int32_t* in, int32_t* out, uint64_t count, const int32_t* lut, void* stream) {
    if (!in || !out || !lut) return DH_ERR_NULL_POINTER;
    if (count == 0) return DH_OK;
    const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((count + 255) / 256, 148ull * 8));
    gelu_q10_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(in, out, count, lut);
    DH_LAUNCH_CHECK();
    return DH_OK;
}
