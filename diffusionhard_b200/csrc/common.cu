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
