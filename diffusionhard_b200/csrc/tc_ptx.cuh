// tc_ptx.cuh -- thin inline-PTX wrappers for the sm_100a tensor-core path:
// mbarriers, TMA tile loads, tcgen05 TMEM allocation / loads / MMA, and the
// shared-memory and instruction descriptors (layouts per the PTX ISA
// "tcgen05 matrix descriptors" and "instruction descriptor" tables).
//
// No multicast anywhere: every TMA load is issued by the CTA that consumes it
// and reads this GPU's own memory.
#pragma once

#include "dh_common.cuh"

namespace dh {
namespace tc {

// ------------------------------------------------------------------ errors

// Device error word (bounded waits that expire set it; the host reads it with
// dh_device_error).
extern __device__ uint32_t g_device_error;

constexpr uint32_t kErrTimeoutFull = 1;
constexpr uint32_t kErrTimeoutEmpty = 2;
constexpr uint32_t kErrTimeoutAccFull = 3;
constexpr uint32_t kErrTimeoutAccEmpty = 4;
constexpr uint32_t kErrTimeoutPair = 5;  // epilogue warp-pair rendezvous

DH_DEVINL void report_error(uint32_t code) { atomicCAS(&g_device_error, 0u, code); }

// --------------------------------------------------------------- mbarrier

DH_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

DH_DEVINL void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

DH_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

DH_DEVINL void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

DH_DEVINL bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wall-clock bound of the suspending waits below.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

DH_DEVINL uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete is
// suspended until it completes (or 1 ms passes) instead of returning at once
// to poll again.
DH_DEVINL bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}

// Bounded wait for pipelines whose waiting threads share schedulers with the
// threads doing the work: the waiter sleeps instead of taking issue slots.
// Gives up (records `code`, returns false) after limit_ns of wall time.
DH_DEVINL bool mbar_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t code,
                                 uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait_suspend(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait_suspend(bar, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) {
            report_error(code);
            return false;
        }
    }
}

// Bounded wait: returns false (and records `code`) when the spin limit expires.
DH_DEVINL bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t code) {
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    report_error(code);
    return false;
}

// Bounded rendezvous: arrive on `bar` and wait for the phase this arrival
// belongs to (identified by the arrival's state token, so the caller keeps no
// parity).  Every participant of the barrier's count must call it.  Returns
// false (and records `code`) when the spin limit expires, e.g. because a
// participant gave up earlier and will never arrive.
DH_DEVINL bool mbar_arrive_wait(uint64_t* bar, uint32_t code) {
    uint64_t token;
    asm volatile("mbarrier.arrive.shared::cta.b64 %0, [%1];" : "=l"(token) : "r"(smem_u32(bar)) : "memory");
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "l"(token)
            : "memory");
        if (ok) return true;
    }
    report_error(code);
    return false;
}

// ------------------------------------------------------------------- TMA

// Tiled store shared -> global (bulk-group completion, no multicast).  x is
// the innermost coordinate; x * element size must be a multiple of 16 bytes
// and no coordinate may be negative.
DH_DEVINL void tma_store_2d(const void* tmap, const void* smem_src, int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(tmap)),
                 "r"(smem_u32(smem_src)), "r"(x), "r"(y)
                 : "memory");
}
DH_DEVINL void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed store groups still read their shared source.
template <int N>
DH_DEVINL void tma_store_wait_read() { asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory"); }
// Wait until every committed store group completed.
DH_DEVINL void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

DH_DEVINL void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar, int32_t x, int32_t y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

DH_DEVINL void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int32_t x, int32_t y,
                           int32_t z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

DH_DEVINL void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// ------------------------------------------------------------------ TMEM

// Allocate `ncols` TMEM columns (power of two >= 32); the base address is
// written to *smem_result.  Whole warp.
DH_DEVINL void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

DH_DEVINL void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

DH_DEVINL void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DH_DEVINL void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives the
// 32 columns of TMEM lane (warp quadrant base + t).
DH_DEVINL void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

DH_DEVINL uint32_t tmem_ld_32x32b_x1(uint32_t taddr) {
    uint32_t r;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
    return r;
}

DH_DEVINL void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 consecutive columns (stores) -- used to stage P for attention.
DH_DEVINL void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15])
        : "memory");
}
DH_DEVINL void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

DH_DEVINL void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------ descriptors

// Shared-memory matrix descriptor, K-major operand staged by TMA with
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart (SBO).
// Bits: [0,14) start>>4, [16,30) LBO>>4, [32,46) SBO>>4, [46,48) version 1,
// [49,52) base offset 0, [61,64) layout 2 = SWIZZLE_128B.
DH_DEVINL uint64_t smem_desc_sw128(const void* smem_ptr) {
    const uint32_t addr = smem_u32(smem_ptr);
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(1u) << 16;             // LBO (unused for swizzled K-major)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;     // SBO
    d |= static_cast<uint64_t>(1u) << 46;             // descriptor version (sm100)
    d |= static_cast<uint64_t>(2u) << 61;             // SWIZZLE_128B
    return d;
}

// Advance the start address of a descriptor by `bytes` (multiple of 16) --
// the K step inside one 128-byte swizzle atom.
DH_DEVINL uint64_t desc_advance(uint64_t desc, uint32_t bytes) { return desc + (bytes >> 4); }

// Instruction descriptor, dense, K-major A and B.
//   [4,6) D format (1 = F32, 2 = S32), [7,10) A format, [10,13) B format,
//   [15] A major, [16] B major, [17,23) N>>3, [24,29) M>>4.
// kind::i8: A/B format 1 = signed int8.  kind::f16: A/B format 1 = bf16.
template <uint32_t M, uint32_t N>
__host__ __device__ constexpr uint32_t idesc_i8_s32() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}
template <uint32_t M, uint32_t N>
__host__ __device__ constexpr uint32_t idesc_bf16_f32() {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// kind::f16 with f16 A and B, f32 accumulate.
template <uint32_t M, uint32_t N>
__host__ __device__ constexpr uint32_t idesc_f16_f32() {
    return (1u << 4) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, one instruction (M x N x 32 for i8,
// M x N x 16 for bf16).  Issued by a single thread.
DH_DEVINL void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                      uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

DH_DEVINL void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` when all previously issued tcgen05 ops of this thread finish.
// D[tmem] (+)= A[tmem] * B[smem]^T (kind::f16): A is M x 16 with row m in
// TMEM lane m and its 16 elements packed two per column in 8 consecutive
// columns starting at a_tmem.  Issued by a single thread.
DH_DEVINL void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

DH_DEVINL void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

DH_DEVINL bool elect_one() {
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "elect.sync _|p, 0xFFFFFFFF;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

}  // namespace tc
}  // namespace dh
