// Peer-memory exchange for the Ulysses all-to-alls (patches/InfiniLM.patch:895-1137,
// all_to_all_* InfiniCore.patch:526-577): the producing kernels (the QKV
// projection's epilogue, or the q/k RMSNorm + RoPE and row-copy kernels, and the
// attention's scatter epilogue) store straight into the peers' receive buffers
// over NVLink, then one thread per rank raises an epoch flag in
// every peer's flag array and the receiver waits for its peers' flags before the
// next kernel reads the data.  Receive buffers are plain cudaMalloc allocations
// shared through CUDA IPC handles (no multicast objects, no NVLS).
//
// Flag array of a rank: uint64 flags[slot][H3_EXCHANGE_MAX_RANKS]; flags[s][q] is
// written only by rank q.  Every rank also keeps uint64 epoch[slot] locally: the
// signal kernel increments it and sends the new value, the wait kernel waits
// until every peer's flag has reached the local value.  All ranks run the same
// sequence of exchanges, so their epochs advance together; a peer can be at
// most one exchange ahead (it needs this rank's next message to go further),
// hence the >= test.
//
// Buffer reuse needs no extra flags: a rank writes a peer's q/k/v receive buffer
// for block i+1 only after it has received that peer's attention output of block i
// (sent after the peer's attention read the buffer), and a peer writes this rank's
// output-return buffer for block i+1 only after receiving this rank's q/k/v of
// block i+1 (sent after this rank consumed block i's returns).
#include <stdint.h>
#include <string.h>

#include <cuda_bf16.h>

#include "h3_abi_util.h"
#include "sm100_ptx.cuh"

namespace h3 {
namespace xchg {

struct PeerFlags {
    uint64_t *flags[H3_EXCHANGE_MAX_RANKS];  // flag array of every rank (own entry included)
};

__device__ __forceinline__ void st_release_sys(uint64_t *p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void signal_kernel(PeerFlags peers, uint64_t *epoch, int slot, int rank, int world) {
    if (threadIdx.x != 0) return;
    const uint64_t e = epoch[slot] + 1;
    epoch[slot] = e;
    // the data stores of the preceding kernels on this stream are complete; order
    // the flag after them for every observer in the system
    __threadfence_system();
    for (int p = 0; p < world; ++p)
        if (p != rank) st_release_sys(peers.flags[p] + slot * H3_EXCHANGE_MAX_RANKS + rank, e);
}

__global__ void wait_kernel(const uint64_t *flags, const uint64_t *epoch, int slot, int rank, int world,
                            uint64_t timeout_ns) {
    const int q = threadIdx.x;
    bool ok = true;
    if (q < world && q != rank) {
        const uint64_t target = epoch[slot];
        const uint64_t *f = flags + slot * H3_EXCHANGE_MAX_RANKS + q;
        const uint64_t start = globaltimer();
        while (ld_acquire_sys(f) < target) {
            if (globaltimer() - start > timeout_ns) {
                ok = false;
                break;
            }
            __nanosleep(64);
        }
    }
    if (!ok) atomicOr(&g_h3_device_error, 1u);
    __syncwarp();
    __threadfence_system();
}

// All-reduce step of the tensor-parallel block (the reference's allreduce_on_stream_
// after the row-parallel projections, InfiniLM.patch:1432-1436, 1455-1459): this
// rank owns rows [r0, r0 + R) of the sum; it reads those rows of every rank's
// partial (peer loads), adds them in fp32 in rank order, rounds once to BF16 and
// stores the result into every rank's sum buffer (peer stores).  The fixed order
// makes the sum identical on every rank and independent of timing.
struct ReduceArgs {
    const __nv_bfloat16 *src[H3_EXCHANGE_MAX_RANKS];
    __nv_bfloat16 *dst[H3_EXCHANGE_MAX_RANKS];
    int64_t s_row, d_row;   // row strides (elements), shared by all blocks
    int64_t rows, vec_per_row;
    int n;
};

__global__ void __launch_bounds__(256) reduce_rows_kernel(ReduceArgs a) {
    const int64_t total = a.rows * a.vec_per_row;
    for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < total; i += (int64_t)gridDim.x * 256) {
        const int64_t r = i / a.vec_per_row, c = (i - r * a.vec_per_row) * 8;
        float acc[8] = {};
        for (int p = 0; p < a.n; ++p) {
            const uint4 v = *reinterpret_cast<const uint4 *>(a.src[p] + r * a.s_row + c);
            const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&v);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __bfloat1622float2(h[k]);
                acc[2 * k] = __fadd_rn(acc[2 * k], f.x);
                acc[2 * k + 1] = __fadd_rn(acc[2 * k + 1], f.y);
            }
        }
        uint4 o;
        __nv_bfloat162 *oh = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k) oh[k] = __floats2bfloat162_rn(acc[2 * k], acc[2 * k + 1]);
        for (int p = 0; p < a.n; ++p) *reinterpret_cast<uint4 *>(a.dst[p] + r * a.d_row + c) = o;
    }
}

}  // namespace xchg
}  // namespace h3

using namespace h3;

extern "C" int h3_ipc_alloc(uint64_t bytes, void **ptr, void *handle) {
    if (!ptr || !handle) return H3_ERR_NULL;
    *ptr = nullptr;
    if (bytes == 0) return H3_ERR_BAD_SHAPE;
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return H3_ERR_LAUNCH;
    if (cudaMemset(p, 0, bytes) != cudaSuccess) {
        cudaFree(p);
        return H3_ERR_LAUNCH;
    }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaFree(p);
        return H3_ERR_DRIVER;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == H3_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    *ptr = p;
    return H3_OK;
}

extern "C" int h3_ipc_open(const void *handle, void **ptr) {
    if (!ptr || !handle) return H3_ERR_NULL;
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void *p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return H3_ERR_DRIVER;
    *ptr = p;
    return H3_OK;
}

extern "C" int h3_ipc_close(void *ptr) {
    if (!ptr) return H3_ERR_NULL;
    return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? H3_OK : H3_ERR_DRIVER;
}

extern "C" int h3_ipc_free(void *ptr) {
    if (!ptr) return H3_ERR_NULL;
    return cudaFree(ptr) == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}

extern "C" int h3_exchange_signal(void *const *peer_flags, uint64_t *epoch, int32_t slot, int32_t rank,
                                  int32_t world, void *stream) {
    if (!peer_flags || !epoch) return H3_ERR_NULL;
    if (world < 1 || world > H3_EXCHANGE_MAX_RANKS || rank < 0 || rank >= world) return H3_ERR_BAD_SHAPE;
    if (slot < 0 || slot >= H3_EXCHANGE_SLOTS) return H3_ERR_BAD_SHAPE;
    xchg::PeerFlags pf{};
    for (int p = 0; p < world; ++p) {
        if (!peer_flags[p]) return H3_ERR_NULL;
        pf.flags[p] = static_cast<uint64_t *>(peer_flags[p]);
    }
    xchg::signal_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(pf, epoch, slot, rank, world);
    return launch_status();
}

extern "C" int h3_exchange_wait(const void *flags, const uint64_t *epoch, int32_t slot, int32_t rank, int32_t world,
                                uint64_t timeout_ns, void *stream) {
    if (!flags || !epoch) return H3_ERR_NULL;
    if (world < 1 || world > H3_EXCHANGE_MAX_RANKS || rank < 0 || rank >= world) return H3_ERR_BAD_SHAPE;
    if (slot < 0 || slot >= H3_EXCHANGE_SLOTS) return H3_ERR_BAD_SHAPE;
    if (timeout_ns == 0 || timeout_ns > 60000000000ull) return H3_ERR_UNSUPPORTED;
    xchg::wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(static_cast<const uint64_t *>(flags), epoch, slot, rank,
                                                          world, timeout_ns);
    return launch_status();
}

extern "C" int h3_peer_reduce_rows(const h3_tensor *dsts, const h3_tensor *srcs, int32_t n, void *stream) {
    if (!dsts || !srcs) return H3_ERR_NULL;
    if (n < 1 || n > H3_EXCHANGE_MAX_RANKS) return H3_ERR_BAD_SHAPE;
    const int64_t R = srcs[0].shape[0], C = srcs[0].ndim == 2 ? srcs[0].shape[1] : 0;
    xchg::ReduceArgs a;
    for (int i = 0; i < n; ++i) {
        for (const h3_tensor *t : {&srcs[i], &dsts[i]}) {
            H3_CHECK(check_bf16(t));
            if (t->ndim != 2 || t->shape[0] != R || t->shape[1] != C) return H3_ERR_BAD_SHAPE;
            if ((t->strides[1] != 1 && C > 1) || !aligned16(t->data) || t->strides[0] % 8 != 0) return H3_ERR_BAD_LAYOUT;
        }
        if (srcs[i].strides[0] != srcs[0].strides[0] || dsts[i].strides[0] != dsts[0].strides[0]) return H3_ERR_BAD_LAYOUT;
        a.src[i] = static_cast<const __nv_bfloat16 *>(srcs[i].data);
        a.dst[i] = static_cast<__nv_bfloat16 *>(dsts[i].data);
    }
    if (C % 8 != 0) return H3_ERR_BAD_SHAPE;
    if (R == 0 || C == 0) return H3_OK;
    a.s_row = srcs[0].strides[0];
    a.d_row = dsts[0].strides[0];
    a.rows = R;
    a.vec_per_row = C / 8;
    a.n = n;
    const int64_t total = R * a.vec_per_row;
    const int64_t blocks = (total + 255) / 256;
    xchg::reduce_rows_kernel<<<(unsigned)(blocks < 4 * 148 * 8 ? blocks : 4 * 148 * 8), 256, 0, (cudaStream_t)stream>>>(a);
    return launch_status();
}

// device error word of this translation unit (exchange waits that gave up)
extern "C" unsigned int h3_exchange_device_error_read_and_clear(void) {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, h3::g_h3_device_error, sizeof(v));
    cudaMemcpyToSymbol(h3::g_h3_device_error, &zero, sizeof(zero));
    return v;
}
