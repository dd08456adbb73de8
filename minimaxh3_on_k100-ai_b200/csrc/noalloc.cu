// The out-projection fused with the gated residual + RMSNorm + AdaLN, for callers
// that cannot allocate device memory where they call this library.
//
// h3_linear_gated_residual_rms_modulate passes the per-tile sums of squares from
// the projection's epilogue to the norm pass through a caller-owned workspace.
// Some callers have no way to provide one at the call site: a host framework that
// owns every device allocation through a pool planned ahead of time (it hands out
// the tensors it planned and nothing else), or a plugin boundary whose host side
// has no device allocator at all.  This entry point runs the same two kernels with
// that scratch in a fixed array compiled into the library's device image:
// H3_NOALLOC_SQ_FLOATS floats (4 MiB), present on every GPU that loads the library
// until the process exits.  It calls no cudaMalloc, cudaFree or allocating library
// routine.
//
// The array's name in host code stands for a host-side shadow, not device memory,
// so host code never hands it to a kernel: the first call on each device asks the
// runtime for the array's device address (cudaGetSymbolAddress, with that device
// current) and caches it per device.  That first call should come before any
// stream capture.  All calls share the one array and it keeps whatever the last
// call wrote; nothing needs clearing, because the projection writes every partial
// sum that the norm pass of the same call reads.  Calls that can overlap on the
// GPU (other streams, other host threads on the same device) race on the array
// and must be serialised by the caller.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>

#include "h3_abi_util.h"

namespace {

constexpr int64_t kTileColumns = 256;   // columns per partial sum: the projection's output tile width

// Scratch of h3_linear_gated_residual_rms_modulate_noalloc (see above).
static __device__ __align__(256) float g_noalloc_sq[H3_NOALLOC_SQ_FLOATS];

std::atomic<float *> g_scratch_addr[64];   // device address of g_noalloc_sq per device ordinal
std::mutex g_scratch_mutex;

// The device address of the scratch array on the current device (looked up once per device).
int scratch_address(float **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return H3_ERR_UNSUPPORTED;
    float *p = g_scratch_addr[dev].load(std::memory_order_acquire);
    if (!p) {
        std::lock_guard<std::mutex> lock(g_scratch_mutex);
        p = g_scratch_addr[dev].load(std::memory_order_relaxed);
        if (!p) {
            void *addr = nullptr;
            if (cudaGetSymbolAddress(&addr, g_noalloc_sq) != cudaSuccess || !addr) return H3_ERR_DRIVER;
            p = static_cast<float *>(addr);
            g_scratch_addr[dev].store(p, std::memory_order_release);
        }
    }
    *out = p;
    return H3_OK;
}

}  // namespace

extern "C" int h3_linear_gated_residual_rms_modulate_noalloc(const h3_tensor *residual_out, const h3_tensor *out,
                                                             const h3_tensor *x, const h3_tensor *w,
                                                             const h3_tensor *residual, const h3_tensor *gate,
                                                             const h3_tensor *weight, const h3_tensor *scale,
                                                             const h3_tensor *shift, float eps, void *stream) {
    if (!residual_out || !w) return H3_ERR_NULL;
    if (residual_out->ndim != 2 || w->ndim != 2 || residual_out->shape[0] < 0 || w->shape[0] < 0)
        return H3_ERR_BAD_SHAPE;
    const int64_t rows = residual_out->shape[0];
    const int64_t tiles = (w->shape[0] + kTileColumns - 1) / kTileColumns;
    if (rows * tiles > (int64_t)H3_NOALLOC_SQ_FLOATS) return H3_ERR_TOO_LARGE;
    float *sq = nullptr;
    H3_CHECK(scratch_address(&sq));
    h3_tensor scratch{};
    scratch.data = sq;
    scratch.ndim = 2;
    scratch.dtype = H3_F32;
    scratch.shape[0] = rows;
    scratch.shape[1] = tiles;
    scratch.strides[0] = tiles;
    scratch.strides[1] = 1;
    return h3_linear_gated_residual_rms_modulate(residual_out, out, x, w, residual, gate, weight, scale, shift, eps,
                                                 &scratch, stream);
}
