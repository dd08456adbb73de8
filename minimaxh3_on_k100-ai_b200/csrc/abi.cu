// Library-wide C-ABI entry points: version, status strings, device error word.
#include "h3_abi_util.h"

extern "C" unsigned int h3_attention_device_error_read_and_clear(void);
extern "C" unsigned int h3_gemm_device_error_read_and_clear(void);

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
        default: return "unknown status";
    }
}

// Synchronises the current device, then reads and clears the device error words
// of the kernels with bounded waits.  Returns H3_ERR_TIMEOUT if any wait expired
// since the last call, H3_ERR_LAUNCH if the device reports an error, else H3_OK.
extern "C" int h3_device_error(void) {
    if (cudaDeviceSynchronize() != cudaSuccess) return H3_ERR_LAUNCH;
    const unsigned int w = h3_attention_device_error_read_and_clear() | h3_gemm_device_error_read_and_clear();
    return w ? H3_ERR_TIMEOUT : H3_OK;
}
