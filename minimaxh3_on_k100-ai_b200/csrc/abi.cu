// Library-wide C-ABI entry points: version, status strings, device error word.
#include "h3_abi_util.h"
#include "sm100_ptx.cuh"

extern "C" unsigned int h3_attention_device_error_read_and_clear(void);
extern "C" unsigned int h3_gemm_device_error_read_and_clear(void);
extern "C" unsigned int h3_model_ops_device_error_read_and_clear(void);
extern "C" unsigned int h3_exchange_device_error_read_and_clear(void);

extern "C" int h3_abi_version(void) { return H3_ABI_VERSION; }

extern "C" const char *h3_status_string(int status) {
    switch (status) {
        case H3_OK: return "ok";
        case H3_ERR_NULL: return "null descriptor or data pointer";
        case H3_ERR_BAD_SHAPE: return "bad shape";
        case H3_ERR_BAD_DTYPE: return "bad dtype";
        case H3_ERR_BAD_LAYOUT: return "bad layout (strides or alignment)";
        case H3_ERR_UNSUPPORTED: return "unsupported configuration";
        case H3_ERR_LAUNCH: return "CUDA launch error";
        case H3_ERR_DRIVER: return "driver entry point unavailable";
        case H3_ERR_TIMEOUT: return "bounded device wait timed out";
        case H3_ERR_INDEX: return "row index outside the indexed tensor";
        case H3_ERR_TOO_LARGE: return "request exceeds the library's static scratch capacity";
        default: return "unknown status";
    }
}

// Synchronises the current device, then reads and clears the device error words
// of the kernels with bounded waits or index checks.  Returns H3_ERR_TIMEOUT if
// any wait expired since the last call, else H3_ERR_INDEX if a row index was out
// of range, H3_ERR_LAUNCH if the device reports an error, else H3_OK.
extern "C" int h3_device_error(void) {
    if (cudaDeviceSynchronize() != cudaSuccess) return H3_ERR_LAUNCH;
    unsigned int own = 0, zero = 0;
    cudaMemcpyFromSymbol(&own, h3::g_h3_device_error, sizeof(own));
    cudaMemcpyToSymbol(h3::g_h3_device_error, &zero, sizeof(zero));
    const unsigned int w = own | h3_attention_device_error_read_and_clear() | h3_gemm_device_error_read_and_clear() |
                           h3_model_ops_device_error_read_and_clear() | h3_exchange_device_error_read_and_clear();
    if (w & 1u) return H3_ERR_TIMEOUT;
    return (w & 2u) ? H3_ERR_INDEX : H3_OK;
}

namespace {
// One thread waits on an mbarrier that nothing ever arrives at, with a short
// limit: the bounded-wait path must give up, record the expiry in the device
// error word and let the kernel finish, leaving the context usable.
__global__ void wait_timeout_selftest_kernel(uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        h3::mbar_init(&bar, 1);
        h3::fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) h3::mbar_wait_ns(&bar, 0, nullptr, limit_ns);
    __syncthreads();
}
}  // namespace

extern "C" int h3_selftest_wait_timeout(uint64_t limit_ns, void *stream) {
    if (limit_ns == 0 || limit_ns > 1000000000ull) return H3_ERR_UNSUPPORTED;
    wait_timeout_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(limit_ns);
    return h3::launch_status();
}
