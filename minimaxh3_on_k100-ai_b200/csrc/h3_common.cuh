// Shared device/host helpers for the H3 sm_100a kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/h3_b200.h"

namespace h3 {

// ---------------------------------------------------------------------------
// BF16 rounding helpers.  Every product/sum is written with the _rn intrinsics
// so the compiler cannot contract a multiply and an add into one FMA: the
// reference rounds the fp32 product to BF16 before the add.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf(float v) {  // round to BF16 and back
    return __bfloat162float(__float2bfloat16_rn(v));
}
// Round two values to BF16 and back with one paired conversion (cvt.rn.bf16x2.f32):
// the same round-to-nearest-even as bf() on each value, at half the conversions.
__device__ __forceinline__ void bf2(float &a, float &b) {
    const float2 f = __bfloat1622float2(__floats2bfloat162_rn(a, b));
    a = f.x;
    b = f.y;
}
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }

__device__ __forceinline__ void unpack8(const uint4 &v, float f[8]) {
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __bfloat1622float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}
__device__ __forceinline__ uint4 pack8(const float f[8]) {
    uint4 v;
    __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    return v;
}
__device__ __forceinline__ void unpack4(const uint2 &v, float f[4]) {
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&v);
    float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
}
__device__ __forceinline__ uint2 pack4(const float f[4]) {
    uint2 v;
    __nv_bfloat162 *h = reinterpret_cast<__nv_bfloat162 *>(&v);
    h[0] = __floats2bfloat162_rn(f[0], f[1]);
    h[1] = __floats2bfloat162_rn(f[2], f[3]);
    return v;
}

// Reciprocal square root with the same two roundings as torch's CPU rsqrt
// (1 / sqrt(x): a correctly rounded sqrt, then a correctly rounded division).
__device__ __forceinline__ float rsqrt_torch(float v) { return __fdiv_rn(1.0f, __fsqrt_rn(v)); }

// ---------------------------------------------------------------------------
// Row views: a tensor seen as [n0, n1, C] rows of C elements.  Leading dims of
// a 2-D tensor collapse to n0 = 1.  Strides in elements; stride 0 broadcasts.
// ---------------------------------------------------------------------------
struct RowView {
    const __nv_bfloat16 *p;
    int64_t s0, s1, sc;
};
struct RowViewMut {
    __nv_bfloat16 *p;
    int64_t s0, s1, sc;
};

__device__ __forceinline__ int64_t row_offset(int64_t s0, int64_t s1, int64_t row, int64_t n1) {
    if (row < n1) return row * s1;  // 2-D views (n0 == 1) and the first batch: no division
    const int64_t i0 = row / n1, i1 = row - i0 * n1;
    return i0 * s0 + i1 * s1;
}

}  // namespace h3
