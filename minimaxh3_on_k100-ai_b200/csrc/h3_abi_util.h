// Host-side validation and launch helpers shared by the C-ABI entry points.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "../../include/h3_b200.h"

#define H3_CHECK(expr)              \
    do {                            \
        const int _h3_s = (expr);   \
        if (_h3_s != H3_OK) return _h3_s; \
    } while (0)

namespace h3 {

inline int64_t numel(const h3_tensor *t) {
    int64_t n = 1;
    for (int i = 0; i < t->ndim; ++i) n *= t->shape[i];
    return n;
}

// A descriptor must exist; its data pointer may be null only when it is empty.
inline int check_desc(const h3_tensor *t, int dtype) {
    if (!t) return H3_ERR_NULL;
    if (t->dtype != dtype) return H3_ERR_BAD_DTYPE;
    if (t->ndim < 1 || t->ndim > H3_MAX_DIMS) return H3_ERR_BAD_SHAPE;
    for (int i = 0; i < t->ndim; ++i)
        if (t->shape[i] < 0) return H3_ERR_BAD_SHAPE;
    if (!t->data && numel(t) != 0) return H3_ERR_NULL;
    return H3_OK;
}
inline int check_bf16(const h3_tensor *t) { return check_desc(t, H3_BF16); }

inline int check_rank(const h3_tensor *t, int lo, int hi) {
    if (!t) return H3_ERR_NULL;
    return (t->ndim >= lo && t->ndim <= hi) ? H3_OK : H3_ERR_BAD_SHAPE;
}

inline int check_same_shape(const h3_tensor *a, const h3_tensor *b) {
    if (!a || !b) return H3_ERR_NULL;
    if (a->ndim != b->ndim) return H3_ERR_BAD_SHAPE;
    for (int i = 0; i < a->ndim; ++i)
        if (a->shape[i] != b->shape[i]) return H3_ERR_BAD_SHAPE;
    return H3_OK;
}

// [S, C] -> (n0 = 1, n1 = S); [B, S, C] -> (n0 = B, n1 = S); rows = n0 * n1
inline void lead_dims(const h3_tensor *t, int64_t *rows, int64_t *n1) {
    if (t->ndim == 3) {
        *rows = t->shape[0] * t->shape[1];
        *n1 = t->shape[1] > 0 ? t->shape[1] : 1;
    } else {
        *rows = t->shape[0];
        *n1 = t->shape[0] > 0 ? t->shape[0] : 1;
    }
}
inline void lead_strides(const h3_tensor *t, int64_t *s0, int64_t *s1) {
    if (t->ndim == 3) {
        *s0 = t->strides[0];
        *s1 = t->strides[1];
    } else {
        *s0 = 0;
        *s1 = t->strides[0];
    }
}

inline bool aligned_to(const void *p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }
inline bool aligned16(const void *p) { return aligned_to(p, 16); }

// every row starts 16-byte aligned, the inner stride is 1 and C is a multiple of `vec`
inline bool rows_vectorizable(const h3_tensor *t, int64_t vec) {
    const int64_t C = t->shape[t->ndim - 1];
    if (t->strides[t->ndim - 1] != 1 || C % vec != 0 || !aligned16(t->data)) return false;
    for (int i = 0; i < t->ndim - 1; ++i)
        if (t->strides[i] % vec != 0) return false;
    return true;
}

inline int launch_status() {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? H3_OK : H3_ERR_LAUNCH;
}

// SM count of the current device, cached per device ordinal.
inline int num_sms() {
    static std::atomic<int> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int v = cache[dev].load(std::memory_order_relaxed);
    if (v == 0) {
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        cache[dev].store(v, std::memory_order_relaxed);
    }
    return v;
}

}  // namespace h3
