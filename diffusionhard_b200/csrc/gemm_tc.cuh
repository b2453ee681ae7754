// gemm_tc.cuh -- persistent warp-specialised int8 GEMM on tcgen05 (sm_100a).
//
//   C[M, N] = A[M, K] . B[N, K]^T   int8 x int8 -> int32 accumulators in TMEM
//
// Both operands are K-major (rows of K bytes) and staged by TMA into 128-byte
// swizzled shared-memory tiles (BM=128 rows x BK=128 bytes for A, BN rows x
// 128 bytes for B), STAGES deep.  One CTA per SM loops over output tiles:
//   warp 0      TMA producer (one elected lane)
//   warp 1      MMA issuer (one elected lane), owns the TMEM allocation
//   warps 2..9  epilogue: 8 warps = 2 per TMEM lane quadrant, each thread owns
//               one output row and half of the tile's columns.
// The accumulator is double-buffered in TMEM (2 x BN columns) so the
// epilogue of tile i overlaps the MMAs of tile i+1.  The epilogue is a policy
// class (Epi) that receives each thread's row and kChunk consecutive int32
// accumulators; it fuses dequantisation and whatever follows the GEMM.
//
// Every mbarrier wait is bounded; on expiry the kernel records an error in
// tc::g_device_error, drains its own TMA copies and MMAs, frees TMEM, exits.
#pragma once

#include <cuda.h>

#include "tc_ptx.cuh"

namespace dh {

// Default hooks for epilogue policies: extra shared memory (bytes, placed
// after the pipeline stages) initialised once per CTA by the epilogue threads
// (thread `tid` of `count`), while the TMA and MMA warps already start the
// first tile's pipeline.
struct EpiBase {
    static constexpr uint32_t kStages = 4;          // TMA pipeline depth
    // epilogue warp groups of 8: with 2, group g takes the tiles accumulated
    // in TMEM buffer g, so two tiles' epilogues run at once (4 warps per
    // scheduler instead of 2), at a register cap of ~112 per thread
    static constexpr uint32_t kGroups = 1;
    static constexpr uint32_t kExtraSmem = 0;      // shared by the CTA
    static constexpr uint32_t kStagingPerWarp = 0;  // private to each epilogue warp
    // Few-row mode: when a launch has at most 32 valid rows, its A rows are
    // loaded into all four 32-row quarters of the tile, so every TMEM lane
    // quadrant holds them; the four warps of a column half then split its
    // columns four ways instead of one quadrant's warps doing all the work
    // (needs (BN / 8) % kChunk == 0).
    static constexpr bool kReplicateRows = false;
    template <class P>
    static DH_DEVINL void init_smem(const P&, uint8_t*, uint32_t /*tid*/, uint32_t /*count*/) {}
    // after the warp's last tile (e.g. drain asynchronous stores that read
    // shared memory before the CTA exits)
    static DH_DEVINL void finish(uint32_t /*lane*/) {}
};

// What an epilogue thread knows about its place in the tile.  All 32 lanes of
// an epilogue warp call chunk() together (rows past m_eff included), so a
// policy may use warp-cooperative stores through its staging buffer.
struct EpiCtx {
    uint32_t row;      // this thread's output row
    bool row_ok;       // row < m_eff
    uint32_t row0;     // first row of this warp (32 consecutive rows)
    uint32_t m_eff;    // number of valid rows
    uint32_t lane;
    uint8_t* stage;    // kStagingPerWarp bytes private to this warp
    uint8_t* extra;    // kExtraSmem bytes shared by the CTA
    bool first_tile;   // this is the warp's first tile
    bool has_next;     // this warp has another tile after this one:
    uint32_t next_row0;  // its first row
    uint32_t next_col;   // and first column (the warp's half of that tile)
    // Bounded rendezvous of the two warps that cover this warp's lane
    // quadrant in its group (an mbarrier of count 64, for
    // tc::mbar_arrive_wait).  A policy that needs the pair in step uses it
    // instead of a named barrier, so a partner that gave up cannot hang it.
    uint64_t* pair_bar;
};

struct GemmShape {
    uint32_t M, N, K;            // K in int8 elements
    const uint32_t* m_count;     // optional device row count (M_eff = min(M, *m_count))
};

template <uint32_t BN_, uint32_t STAGES_ = 4, uint32_t GROUPS_ = 1>
struct GemmCfg {
    static constexpr uint32_t BM = 128, BN = BN_, BK = 128;
    static constexpr uint32_t STAGES = STAGES_;
    static constexpr uint32_t A_BYTES = BM * BK;
    static constexpr uint32_t B_BYTES = BN * BK;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    // two accumulator buffers of BN columns; the allocation is a power of 2
    static constexpr uint32_t TMEM_COLS = 2 * BN <= 256 ? 256u : 512u;
    static constexpr uint32_t GROUPS = GROUPS_;
    static constexpr uint32_t EPI_WARPS = 8 * GROUPS;
    static constexpr uint32_t EPI_THREADS = 32 * EPI_WARPS;
    static constexpr uint32_t THREADS = 64 + EPI_THREADS;
    // barriers + TMEM address, rounded so the epilogue buffers after it stay
    // 128-byte aligned
    // rounded to 1 KB so the epilogue region that follows can hold swizzled
    // TMA store sources
    static constexpr uint32_t BAR_BYTES = ((8 * (2 * STAGES + 5) + 16) + 1023) / 1024 * 1024;
    // the epilogue pair barriers (2 groups x 4 lane quadrants) sit in the
    // upper half of the barrier region
    static constexpr uint32_t PAIR_BAR_OFFSET = 512;
    static_assert(8 * (2 * STAGES + 5) + 16 <= PAIR_BAR_OFFSET && PAIR_BAR_OFFSET + 64 <= BAR_BYTES,
                  "barrier region layout");
    static constexpr uint32_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
    template <class Epi>
    static constexpr uint32_t smem_bytes() {
        return SMEM_BYTES + Epi::kExtraSmem + EPI_WARPS * Epi::kStagingPerWarp;
    }
    static constexpr uint32_t IDESC = tc::idesc_i8_s32<BM, BN>();
};

template <uint32_t BN, class Epi>
__global__ void __launch_bounds__(GemmCfg<BN, Epi::kStages, Epi::kGroups>::THREADS, 1)
gemm_i8_tc_kernel(const __grid_constant__ CUtensorMap tmap_a,
                  const __grid_constant__ CUtensorMap tmap_b,
                  const __grid_constant__ CUtensorMap tmap_a32,  // A, 32-row box (few-row mode)
                  GemmShape shape,
                  const __grid_constant__ typename Epi::Params ep) {
    using Cfg = GemmCfg<BN, Epi::kStages, Epi::kGroups>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    uint8_t* a_smem = smem;
    uint8_t* b_smem = smem + Cfg::STAGES * Cfg::A_BYTES;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(b_smem + Cfg::STAGES * Cfg::B_BYTES);
    uint64_t* empty_bar = full_bar + Cfg::STAGES;
    uint64_t* accf_bar = empty_bar + Cfg::STAGES;  // [2]
    uint64_t* acce_bar = accf_bar + 2;             // [2]
    uint64_t* drain_bar = acce_bar + 2;            // [1]
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain_bar + 1);
    uint64_t* pair_bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(full_bar) + Cfg::PAIR_BAR_OFFSET);
    uint8_t* extra_smem = smem + Cfg::STAGES * Cfg::STAGE_BYTES + Cfg::BAR_BYTES;

    const uint32_t warp = warp_id();
    const uint32_t lane = lane_id();
    if (warp == 0 && lane == 0) {
        for (uint32_t s = 0; s < Cfg::STAGES; ++s) {
            tc::mbar_init(&full_bar[s], 1);
            tc::mbar_init(&empty_bar[s], 1);
        }
        for (uint32_t b = 0; b < 2; ++b) {
            tc::mbar_init(&accf_bar[b], 1);
            tc::mbar_init(&acce_bar[b], 8 * 32);  // one group of 8 warps drains a buffer
        }
        tc::mbar_init(drain_bar, 1);
        for (uint32_t q = 0; q < 8; ++q) tc::mbar_init(&pair_bars[q], 64);
        tc::fence_barrier_init();
        tc::prefetch_tmap(&tmap_a);
        tc::prefetch_tmap(&tmap_b);
        if (Epi::kReplicateRows) tc::prefetch_tmap(&tmap_a32);
    }
    if (warp == 1) tc::tmem_alloc(tmem_holder, Cfg::TMEM_COLS);
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    uint32_t m_eff = shape.M;
    if (shape.m_count) m_eff = min(m_eff, *shape.m_count);
    const uint32_t m_tiles = (m_eff + Cfg::BM - 1) / Cfg::BM;
    const uint32_t n_tiles = (shape.N + BN - 1) / BN;
    const uint32_t k_blocks = (shape.K + Cfg::BK - 1) / Cfg::BK;
    const uint32_t total = m_tiles * n_tiles;
    // few-row mode (one row tile): the 32-row A box lands in every quarter
    const bool replicate = Epi::kReplicateRows && m_eff <= 32;

    if (warp == 0) {
        // ------------------------------------------------------ TMA producer
        if (tc::elect_one()) {
            uint32_t stage = 0, phase = 0;
            uint32_t issued_parity[Cfg::STAGES];
            uint32_t issued = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                const uint32_t m0 = (tile / n_tiles) * Cfg::BM;
                const uint32_t n0 = (tile % n_tiles) * BN;
                for (uint32_t kb = 0; kb < k_blocks; ++kb) {
                    if (!tc::mbar_wait(&empty_bar[stage], phase ^ 1, tc::kErrTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
                    if (replicate) {
#pragma unroll
                        for (uint32_t q = 0; q < 4; ++q)  // 4 KB quarters, 1 KB-aligned for the swizzle
                            tc::tma_load_2d(a_smem + stage * Cfg::A_BYTES + q * (Cfg::A_BYTES / 4), &tmap_a32,
                                            &full_bar[stage], static_cast<int32_t>(kb * Cfg::BK),
                                            static_cast<int32_t>(m0));
                    } else {
                        tc::tma_load_2d(a_smem + stage * Cfg::A_BYTES, &tmap_a, &full_bar[stage],
                                        static_cast<int32_t>(kb * Cfg::BK), static_cast<int32_t>(m0));
                    }
                    tc::tma_load_2d(b_smem + stage * Cfg::B_BYTES, &tmap_b, &full_bar[stage],
                                    static_cast<int32_t>(kb * Cfg::BK), static_cast<int32_t>(n0));
                    issued_parity[stage] = phase;
                    ++issued;
                    if (++stage == Cfg::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Drain: every copy this CTA issued has landed before it may exit.
            const uint32_t last = issued < Cfg::STAGES ? issued : Cfg::STAGES;
            for (uint32_t i = 0; i < last; ++i) {
                const uint32_t s = (stage + Cfg::STAGES - 1 - i) % Cfg::STAGES;
                tc::mbar_wait(&full_bar[s], issued_parity[s], tc::kErrTimeoutFull);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------- MMA issuer
        if (tc::elect_one()) {
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true;
            for (uint32_t tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
                if (!tc::mbar_wait(&acce_bar[acc], acc_phase ^ 1, tc::kErrTimeoutAccEmpty)) break;
                tc::tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (uint32_t kb = 0; kb < k_blocks; ++kb) {
                    if (!tc::mbar_wait(&full_bar[stage], phase, tc::kErrTimeoutFull)) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint64_t a_desc = tc::smem_desc_sw128(a_smem + stage * Cfg::A_BYTES);
                    const uint64_t b_desc = tc::smem_desc_sw128(b_smem + stage * Cfg::B_BYTES);
#pragma unroll
                    for (uint32_t kk = 0; kk < Cfg::BK / 32; ++kk)
                        tc::mma_i8(d_tmem, tc::desc_advance(a_desc, kk * 32),
                                   tc::desc_advance(b_desc, kk * 32), Cfg::IDESC,
                                   (kb | kk) != 0u);
                    tc::mma_commit(&empty_bar[stage]);
                    if (++stage == Cfg::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (!ok) break;
                tc::mma_commit(&accf_bar[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1;
                }
            }
            // Drain: all MMAs issued by this thread complete before TMEM is freed.
            tc::mma_commit(drain_bar);
            tc::mbar_wait(drain_bar, 0, tc::kErrTimeoutAccFull);
        }
    } else {
        // --------------------------------------------------------- epilogue
        const uint32_t ew = warp - 2;  // epilogue warp index
        // the policy's per-CTA tables, filled by the epilogue warps alone
        // (named barrier 1 counts exactly them; no wait precedes it, so every
        // epilogue thread arrives) while the first tile's loads and MMAs run
        Epi::init_smem(ep, extra_smem, threadIdx.x - 64u, Cfg::EPI_THREADS);
        asm volatile("bar.sync 1, %0;" ::"r"(Cfg::EPI_THREADS) : "memory");
        const uint32_t group = ew / 8u;
        const uint32_t quad = warp & 3u;
        const uint32_t half = (ew >> 2) & 1u;
        // few-row mode: every quadrant holds rows 0-31, and the quadrant's
        // warps take a quarter of their half's columns each
        const uint32_t quad_row = replicate ? 0u : quad * 32;
        const uint32_t row_in_tile = quad_row + lane;
        constexpr uint32_t kHalf = BN / 2;
        constexpr uint32_t kChunk = Epi::kChunk;
        static_assert(kHalf % kChunk == 0, "chunk must divide the half tile");
        static_assert(!Epi::kReplicateRows || (kHalf / 4) % kChunk == 0, "few-row mode: a chunk per quarter");
        const uint32_t c_begin = replicate ? quad * (kHalf / 4) : 0u;
        const uint32_t c_end = replicate ? c_begin + kHalf / 4 : kHalf;
        // tile k of this CTA is accumulated in TMEM buffer k % 2
        uint32_t acc = group, acc_phase = 0;
        for (uint32_t tile = blockIdx.x + group * gridDim.x; tile < total; tile += Cfg::GROUPS * gridDim.x) {
            const uint32_t m0 = (tile / n_tiles) * Cfg::BM;
            const uint32_t n0 = (tile % n_tiles) * BN;
            const uint32_t row = m0 + row_in_tile;
            const bool row_ok = row < m_eff;
            const uint32_t next = tile + Cfg::GROUPS * gridDim.x;
            const EpiCtx ctx{row, row_ok, m0 + quad_row, m_eff, lane,
                             extra_smem + Epi::kExtraSmem + ew * Epi::kStagingPerWarp,
                             extra_smem, tile == blockIdx.x + group * gridDim.x, next < total,
                             (next / n_tiles) * Cfg::BM + quad_row, (next % n_tiles) * BN + half * kHalf,
                             &pair_bars[group * 4 + quad]};
            typename Epi::TileState st;
            // tile_begin runs before the accumulator is ready: a policy may
            // start loads that do not depend on it (row metadata, residual).
            // It returns false when one of its own bounded waits gave up.
            if (!Epi::tile_begin(ep, st, ctx, n0 + half * kHalf)) break;
            if (!tc::mbar_wait(&accf_bar[acc], acc_phase, tc::kErrTimeoutAccFull)) break;
            tc::tc_fence_after();
#pragma unroll 1
            for (uint32_t c = c_begin; c < c_end; c += kChunk) {
                const uint32_t col_in_tile = half * kHalf + c;
                const uint32_t taddr =
                    tmem_base + ((quad * 32u) << 16) + acc * BN + col_in_tile;
                uint32_t v[kChunk];
#pragma unroll
                for (uint32_t j = 0; j < kChunk / 32; ++j)
                    tc::tmem_ld_32x32b_x32(taddr + 32 * j,
                                           *reinterpret_cast<uint32_t(*)[32]>(&v[32 * j]));
                tc::tmem_ld_wait();
                Epi::chunk(ep, st, ctx, n0 + col_in_tile, &v[0]);
            }
            Epi::tile_end(ep, st, ctx);
            tc::tc_fence_before();
            tc::mbar_arrive(&acce_bar[acc]);
            if (Cfg::GROUPS == 2) {
                acc_phase ^= 1;
            } else if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1;
            }
        }
        Epi::finish(lane);
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
    }
}

// Host launch helper: persistent grid of min(tiles, SMs) CTAs (or `max_ctas`).
template <uint32_t BN, class Epi>
inline cudaError_t launch_gemm_i8(const CUtensorMap& ta, const CUtensorMap& tb,
                                  const GemmShape& shape, const typename Epi::Params& ep,
                                  uint32_t tiles_hint, cudaStream_t stream,
                                  const CUtensorMap* ta32 = nullptr) {
    using Cfg = GemmCfg<BN, Epi::kStages, Epi::kGroups>;
    auto kernel = gemm_i8_tc_kernel<BN, Epi>;
    static std::atomic<uint64_t> configured{0};
    cudaError_t e = smem_optin_once(kernel, Cfg::template smem_bytes<Epi>(), configured);
    if (e != cudaSuccess) return e;
    int sms = kNumSMs;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
            sms = v;
    }
    const uint32_t grid = tiles_hint == 0 ? 1u : (tiles_hint < static_cast<uint32_t>(sms) ? tiles_hint : sms);
    if (Epi::kReplicateRows && !ta32) return cudaErrorInvalidValue;
    kernel<<<grid, Cfg::THREADS, Cfg::template smem_bytes<Epi>(), stream>>>(ta, tb, ta32 ? *ta32 : ta, shape, ep);
    return cudaGetLastError();
}

}  // namespace dh
