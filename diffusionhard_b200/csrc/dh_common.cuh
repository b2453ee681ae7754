// dh_common.cuh -- shared device helpers for the sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/dh_b200.h"

#define DH_DEVINL __device__ __forceinline__

#define DH_CUDA_RETURN(expr)                                   \
    do {                                                       \
        cudaError_t _e = (expr);                               \
        if (_e != cudaSuccess) return DH_ERR_CUDA;             \
    } while (0)

#define DH_LAUNCH_CHECK()                                      \
    do {                                                       \
        cudaError_t _e = cudaGetLastError();                   \
        if (_e != cudaSuccess) return DH_ERR_CUDA;             \
    } while (0)

namespace dh {

constexpr int kNumSMs = 148;

// Bounded spin limit for every device-side wait (mbarrier polls).  A wait that
// exceeds it records DH_DEVERR_TIMEOUT in the kernel's status word and gives up
// instead of hanging the GPU.
constexpr uint32_t kSpinLimit = 1u << 26;

// Host: opt `kernel` into `bytes` of dynamic shared memory on the current
// device, once per device.  The attribute is per device, so a process that
// launches on several GPUs sets it on each; `done` holds one bit per device
// ordinal (the kernel's own static flag word).  Two threads that race set the
// same value twice, which is harmless.
template <class Kernel>
inline cudaError_t smem_optin_once(Kernel kernel, uint32_t bytes, std::atomic<uint64_t>& done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev >= 0 && dev < 64 ? (1ull << dev) : 0ull;
    if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_release);
    return e;
}

DH_DEVINL uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

DH_DEVINL uint32_t lane_id() { return threadIdx.x & 31u; }
DH_DEVINL uint32_t warp_id() { return threadIdx.x >> 5; }

// Score packing for the (max score, lowest id) argmax reduction: the high word
// is the score with the sign bit flipped (order-preserving for int32), the low
// word is ~id so that, on equal scores, the lower id compares larger.
DH_DEVINL uint64_t pack_score_id(int32_t score, uint32_t id) {
    return (static_cast<uint64_t>(static_cast<uint32_t>(score) ^ 0x80000000u) << 32) |
           static_cast<uint64_t>(0xFFFFFFFFu - id);
}
DH_DEVINL uint32_t packed_id(uint64_t p) { return 0xFFFFFFFFu - static_cast<uint32_t>(p); }
DH_DEVINL int32_t packed_score(uint64_t p) {
    return static_cast<int32_t>(static_cast<uint32_t>(p >> 32) ^ 0x80000000u);
}
// Float keys: order-preserving map of IEEE bits to uint32.
DH_DEVINL uint32_t float_order_key(float f) {
    uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
DH_DEVINL uint64_t pack_float_id(float score, uint32_t id) {
    return (static_cast<uint64_t>(float_order_key(score)) << 32) |
           static_cast<uint64_t>(0xFFFFFFFFu - id);
}

DH_DEVINL uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        uint64_t other = __shfl_xor_sync(0xFFFFFFFFu, v, o);
        v = other > v ? other : v;
    }
    return v;
}

DH_DEVINL float warp_sum_f32(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}
DH_DEVINL float warp_max_f32(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}

}  // namespace dh
