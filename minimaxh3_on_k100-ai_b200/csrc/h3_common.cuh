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

// Packed BF16x2 arithmetic.  For BF16 operands a, b: bf16(fp32(a*b)) is the
// correctly rounded BF16 product (the fp32 product is exact), and
// bf16(fp32(a+b)) is the correctly rounded BF16 sum (the fp32 sum is exact
// unless the smaller term is below 2^-16 of the larger, where both roundings
// return the larger term).  So one mul.rn.bf16x2 / add.rn.bf16x2 reproduces
// the reference's "fp32 op, then .to(bf16)" step bit for bit, two lanes at a time.
// The .rn modifier is explicit: without it ptxas may contract a mul followed by
// an add into one fma (one rounding instead of the reference's two).
__device__ __forceinline__ __nv_bfloat162 u2bf(uint32_t u) { return *reinterpret_cast<__nv_bfloat162 *>(&u); }
__device__ __forceinline__ uint32_t bf2u(__nv_bfloat162 b) { return *reinterpret_cast<uint32_t *>(&b); }
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t badd2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t bneg2(uint32_t a) { return a ^ 0x80008000u; }
__device__ __forceinline__ uint32_t bsplat(float v) { return bf2u(__float2bfloat162_rn(v)); }  // v BF16-valued
__device__ __forceinline__ float blo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bhi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ uint32_t &w32(uint4 &v, int i) { return reinterpret_cast<uint32_t *>(&v)[i]; }
__device__ __forceinline__ uint32_t w32(const uint4 &v, int i) { return reinterpret_cast<const uint32_t *>(&v)[i]; }
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
// Unsigned 32-bit division by a run-time invariant divisor with one multiply-high
// (Granlund & Montgomery, "Division by invariant integers using multiplication",
// PLDI 1994, round-up method): for d > 1, l = ceil(log2 d),
// m = floor(2^32 (2^l - d) / d) + 1, q = (t + ((n - t) >> 1)) >> (l - 1) with
// t = umulhi(n, m).  Exact for every 32-bit n; d == 1 is handled separately.
struct FastDiv {
    uint32_t d, m, l;
    __host__ static FastDiv make(uint32_t d) {
        FastDiv f;
        f.d = d;
        uint32_t l = 0;
        while ((1ull << l) < d) ++l;
        f.l = l;
        f.m = d > 1 ? (uint32_t)((((1ull << 32) * ((1ull << l) - d)) / d) + 1) : 0;
        return f;
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        if (d == 1) return n;
        const uint32_t t = __umulhi(n, m);
        return (t + ((n - t) >> 1)) >> (l - 1);
    }
};

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
