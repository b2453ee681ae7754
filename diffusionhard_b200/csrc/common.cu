// common.cu -- library-wide device state: the device error word written by
// bounded waits that expire (see tc_ptx.cuh), and its host accessor.
#include "tc_ptx.cuh"

namespace dh {
namespace tc {
__device__ uint32_t g_device_error = 0;
}  // namespace tc
}  // namespace dh

extern "C" uint32_t dh_device_error(uint32_t* out, uint32_t clear) {
    if (!out) return DH_ERR_NULL_POINTER;
    uint32_t v = 0;
    DH_CUDA_RETURN(cudaMemcpyFromSymbol(&v, dh::tc::g_device_error, sizeof(v)));
    if (clear) {
        const uint32_t zero = 0;
        DH_CUDA_RETURN(cudaMemcpyToSymbol(dh::tc::g_device_error, &zero, sizeof(zero)));
    }
    *out = v;
    return DH_OK;
}

namespace dh {
namespace {

// One thread waits on a shared-memory mbarrier that receives its single
// arrival only when `arrive` is set.  The wait polls at most `spin_limit`
// times, then records kErrTimeoutFull in the device error word and returns --
// the same give-up path as the pipeline waits of the GEMM, attention and head
// kernels -- so a wait that can never complete ends the kernel instead of
// hanging the GPU.
__global__ void wait_selftest_kernel(uint32_t spin_limit, uint32_t arrive, uint32_t* completed) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
    if (arrive) tc::mbar_arrive(&bar);
    bool ok = false;
    for (uint32_t i = 0; i < spin_limit && !ok; ++i) ok = tc::mbar_try_wait(&bar, 0);
    if (!ok) tc::report_error(tc::kErrTimeoutFull);
    *completed = ok ? 1u : 0u;
}

__global__ void wait_suspend_selftest_kernel(uint64_t limit_ns, uint32_t arrive, uint32_t* completed) {
    __shared__ uint64_t bar;
    if (threadIdx.x != 0) return;
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
    if (arrive) tc::mbar_arrive(&bar);
    *completed = tc::mbar_wait_suspend(&bar, 0, tc::kErrTimeoutFull, limit_ns) ? 1u : 0u;
}

}  // namespace
}  // namespace dh

extern "C" uint32_t dh_wait_suspend_selftest(uint64_t limit_ns, uint32_t arrive, uint32_t* completed, void* stream) {
    if (!completed) return DH_ERR_NULL_POINTER;
    if (limit_ns == 0 || limit_ns > dh::tc::kWaitLimitNs) return DH_ERR_INVALID_ARGUMENT;
    dh::wait_suspend_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, arrive, completed);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

extern "C" uint32_t dh_wait_selftest(uint32_t spin_limit, uint32_t arrive, uint32_t* completed, void* stream) {
    if (!completed) return DH_ERR_NULL_POINTER;
    if (spin_limit == 0 || spin_limit > (1u << 16)) return DH_ERR_INVALID_ARGUMENT;
    dh::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(spin_limit, arrive, completed);
    DH_LAUNCH_CHECK();
    return DH_OK;
}
