// Fused pointwise kernels of the H3 DiT block (sm_100a), with the reference's
// BF16 rounding at every step (tools/h3_pointwise.py; torch compositions in
// tools/bench_h3_ops.py:81-258), plus their C-ABI entry points.
//
// Design: HBM-bound; every kernel reads its inputs once and writes its outputs
// once with 16-byte accesses and enough independent loads in flight per thread.
//  * Row ops (RMSNorm / AdaLN family, LayerNorm variant): one warp per row, the
//    row held in registers as packed BF16 (it is BF16 anyway), sum of squares
//    reduced serially per lane in column order then by an xor-shuffle tree: no
//    shared memory, no block barrier, and a row's result never depends on which
//    warp, CTA or rank computes it.
//  * Per-head ops (q/k norm + RoPE): a half-warp per 128-wide head row (16 lanes x
//    8 elements), two rows in flight per half-warp, RoPE partners exchanged by
//    shuffle, output written straight into the (permuted) all-to-all send layout.
//  * Element-wise ops (gated residual, SwiGLU): flat grid over (row, column
//    vector), one 16-byte vector of each operand per thread, no 64-bit division.
// Launch shapes (rows per task, vectors per thread, occupancy) were chosen by
// timing CUDA-graph-replayed launches on B200 at the reference's benchmark shapes
// ([8192, 1792], [8192, 4864], q/k [8192, 14, 128]) and at the DiT step's: many
// resident warps with little work each beat fewer warps with deeper pipelines.
// Each kernel has a vectorised path (inner stride 1, 16-byte aligned rows) and a
// strided path with the same arithmetic and summation order (identical bits).
#include <math.h>

#include "h3_abi_util.h"
#include "h3_common.cuh"

namespace h3 {

template <bool VEC>
__device__ __forceinline__ uint4 load8p(const __nv_bfloat16 *base, int64_t sc, int64_t col, int64_t C) {
    if (VEC) return *reinterpret_cast<const uint4 *>(base + col);
    float f[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = (col + i < C) ? __bfloat162float(base[(col + i) * sc]) : 0.f;
    return pack8(f);
}
template <bool VEC>
__device__ __forceinline__ void store8p(__nv_bfloat16 *base, int64_t sc, int64_t col, int64_t C, uint4 v) {
    if (VEC) {
        *reinterpret_cast<uint4 *>(base + col) = v;
    } else {
        float f[8];
        unpack8(v, f);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (col + i < C) base[(col + i) * sc] = __float2bfloat16_rn(f[i]);
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = add_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ===========================================================================
// element-wise ops: gated residual, SwiGLU
// ===========================================================================
struct EwArgs {
    RowView a, b, c;     // gated residual: a=x, b=gate, c=y ; swiglu: a=up, b=gate
    RowViewMut o;
    int64_t rows, n1, C;
};

enum { EW_GATED_RESIDUAL = 0, EW_SWIGLU = 1 };
#ifndef H3_EW_VPT
#define H3_EW_VPT 1
#endif
constexpr int EW_THREADS = 256, EW_VPT = H3_EW_VPT;   // vectors of 8 per thread

// 8 elements (one 16-byte vector) of either op
template <int OP>
__device__ __forceinline__ uint4 ew_apply8(uint4 a, uint4 b, uint4 c) {
    uint4 o;
    if (OP == EW_GATED_RESIDUAL) {           // bf16(x + bf16(gate * y))
#pragma unroll
        for (int i = 0; i < 4; ++i) w32(o, i) = badd2(w32(a, i), bmul2(w32(b, i), w32(c, i)));
    } else {                                 // bf16(up * bf16(g / (1 + exp(-g))))
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float g0 = blo(w32(b, i)), g1 = bhi(w32(b, i));
            float a0 = __fdiv_rn(g0, add_rn(1.0f, expf(-g0)));
            float a1 = __fdiv_rn(g1, add_rn(1.0f, expf(-g1)));
            w32(o, i) = bmul2(w32(a, i), bf2u(__floats2bfloat162_rn(a0, a1)));
        }
    }
    return o;
}

// Flat index over the rows x vectors of the tensor (row = v / nvec by an
// invariant-integer division), EW_VPT vectors per thread with all loads issued
// before any arithmetic; narrow rows no longer leave most of a CTA idle.
template <int OP, bool VEC>
__global__ void __launch_bounds__(EW_THREADS) ew_kernel(EwArgs args, FastDiv div_nvec, uint32_t total) {
    const int64_t nvec = (args.C + 7) >> 3;
    uint4 va[EW_VPT], vb[EW_VPT], vc[EW_VPT];
    uint32_t rows[EW_VPT], cols[EW_VPT];
    const uint32_t base = blockIdx.x * (uint32_t)(EW_THREADS * EW_VPT) + threadIdx.x;
#pragma unroll
    for (int k = 0; k < EW_VPT; ++k) {
        const uint32_t v = base + k * EW_THREADS;
        const uint32_t row = div_nvec.div(v);
        rows[k] = row;
        cols[k] = v - row * (uint32_t)nvec;
        vc[k] = make_uint4(0, 0, 0, 0);
        if (v < total) {
            const int64_t col = (int64_t)cols[k] * 8;
            va[k] = load8p<VEC>(args.a.p + row_offset(args.a.s0, args.a.s1, row, args.n1), args.a.sc, col, args.C);
            vb[k] = load8p<VEC>(args.b.p + row_offset(args.b.s0, args.b.s1, row, args.n1), args.b.sc, col, args.C);
            if (OP == EW_GATED_RESIDUAL)
                vc[k] = load8p<VEC>(args.c.p + row_offset(args.c.s0, args.c.s1, row, args.n1), args.c.sc, col, args.C);
        }
    }
#pragma unroll
    for (int k = 0; k < EW_VPT; ++k) {
        if (base + k * EW_THREADS < total)
            store8p<VEC>(args.o.p + row_offset(args.o.s0, args.o.s1, rows[k], args.n1), args.o.sc,
                         (int64_t)cols[k] * 8, args.C, ew_apply8<OP>(va[k], vb[k], vc[k]));
    }
}

// ===========================================================================
// row ops: RMSNorm, RMSNorm+AdaLN, gated residual + RMSNorm+AdaLN, LN+AdaLN
// ===========================================================================
// ROW_RMS_MOD_SQ: ROW_RMS_MOD with the row's sum of squares taken from per-256-column
// partial sums (written by a projection epilogue) instead of reduced here.
enum { ROW_RMS = 0, ROW_RMS_MOD = 1, ROW_RES_RMS_MOD = 2, ROW_LN_MOD = 3, ROW_RMS_MOD_SQ = 4 };

struct RowArgs {
    RowView x, gate, y, scale, shift;   // gate/y only for ROW_RES_RMS_MOD
    const __nv_bfloat16 *weight;        // [C], stride wsc
    int64_t wsc;
    RowViewMut out, residual;           // residual only for ROW_RES_RMS_MOD
    int64_t rows, n1, C;
    const float *sq;                    // ROW_RMS_MOD_SQ: [rows, nt] partial sums, row stride ldsq
    int64_t ldsq;
    int nt;
    // per-segment modulation rows (nseg > 0): rows [seg_end[s-1], seg_end[s]) use the
    // contiguous scale / shift rows seg_scale[s] / seg_shift[s]
    int nseg;
    int64_t seg_end[H3_MAX_SEGMENTS];
    const __nv_bfloat16 *seg_scale[H3_MAX_SEGMENTS], *seg_shift[H3_MAX_SEGMENTS];
    float eps;
};

#ifndef H3_ROW_WARPS
#define H3_ROW_WARPS 4
#endif
constexpr int ROW_WARPS = H3_ROW_WARPS;  // rows per CTA (one warp each)
#ifndef H3_ROW_PIPE_MAXV
#define H3_ROW_PIPE_MAXV 8              // rows of at most this many 16-byte vectors per lane are pipelined
#endif
#ifndef H3_ROW_PIPE_RPW
#define H3_ROW_PIPE_RPW 1               // ... H3_ROW_PIPE_RPW rows per warp (1: one row per warp; deeper
                                        // pipelines measured slower, e.g. AdaLN at [8192, 1792] 3560 GB/s
                                        // with 4 rows per warp against 4300 with 1)
#endif

// Phase 1 of a row: its input vectors into registers (for the fused residual
// op, the residual itself, which is also written out).
template <int MODE, bool VEC, int VPT>
__device__ __forceinline__ void row_load(const RowArgs &args, int64_t row, int lane, uint4 (&v)[VPT]) {
    const int64_t C = args.C;
    const int64_t nvec = (C + 7) >> 3;
    const __nv_bfloat16 *xrow = args.x.p + row_offset(args.x.s0, args.x.s1, row, args.n1);
    if (MODE == ROW_RES_RMS_MOD) {
        // residual = bf16(x + bf16(gate * y)), written out and normalised
        const __nv_bfloat16 *grow = args.gate.p + row_offset(args.gate.s0, args.gate.s1, row, args.n1);
        const __nv_bfloat16 *yrow = args.y.p + row_offset(args.y.s0, args.y.s1, row, args.n1);
        __nv_bfloat16 *rrow = args.residual.p + row_offset(args.residual.s0, args.residual.s1, row, args.n1);
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const int64_t vi = lane + 32 * k;
            v[k] = make_uint4(0, 0, 0, 0);
            if (vi < nvec) {
                const uint4 x = load8p<VEC>(xrow, args.x.sc, vi * 8, C);
                const uint4 g = load8p<VEC>(grow, args.gate.sc, vi * 8, C);
                const uint4 y = load8p<VEC>(yrow, args.y.sc, vi * 8, C);
#pragma unroll
                for (int i = 0; i < 4; ++i) w32(v[k], i) = badd2(w32(x, i), bmul2(w32(g, i), w32(y, i)));
                store8p<VEC>(rrow, args.residual.sc, vi * 8, C, v[k]);
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const int64_t vi = lane + 32 * k;
            v[k] = vi < nvec ? load8p<VEC>(xrow, args.x.sc, vi * 8, C) : make_uint4(0, 0, 0, 0);
        }
    }

}

// Phase 2: statistics, normalise, weight, modulate, store.
template <int MODE, bool VEC, int VPT>
__device__ __forceinline__ void row_finish(const RowArgs &args, int64_t row, int lane, const uint4 (&v)[VPT]) {
    const int64_t C = args.C;
    const int64_t nvec = (C + 7) >> 3;
    // ---- statistics (padding lanes hold zeros) ----
    float r = 0.f, shift_ln = 0.f;
    if (MODE == ROW_LN_MOD) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < VPT; ++k)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                s = add_rn(s, blo(w32(v[k], i)));
                s = add_rn(s, bhi(w32(v[k], i)));
            }
        const float mean = __fdiv_rn(warp_sum(s), (float)C);
        float q = 0.f;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
            const int64_t vi = lane + 32 * k;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (vi * 8 + 2 * i < C) {
                    const float d = __fsub_rn(blo(w32(v[k], i)), mean);
                    q = __fmaf_rn(d, d, q);
                }
                if (vi * 8 + 2 * i + 1 < C) {
                    const float d = __fsub_rn(bhi(w32(v[k], i)), mean);
                    q = __fmaf_rn(d, d, q);
                }
            }
        }
        const float var = __fdiv_rn(warp_sum(q), (float)C);
        r = rsqrt_torch(add_rn(var, args.eps));
        shift_ln = -mul_rn(r, mean);  // y = x * rstd + (-rstd * mean), fused
    } else {
        float s = 0.f;
        if (MODE == ROW_RMS_MOD_SQ) {
            // lane l adds partials l, l + 32, ... in order; then the xor tree
            const float *sqrow = args.sq + row * args.ldsq;
            for (int i = lane; i < args.nt; i += 32) s = add_rn(s, sqrow[i]);
        } else {
#pragma unroll
            for (int k = 0; k < VPT; ++k)
#pragma unroll
                for (int i = 0; i < 4; ++i) {   // bf16(x^2), summed in fp32 in column order
                    const uint32_t sq = bmul2(w32(v[k], i), w32(v[k], i));
                    s = add_rn(s, blo(sq));
                    s = add_rn(s, bhi(sq));
                }
        }
        const float mean = bf(__fdiv_rn(warp_sum(s), (float)C));
        const float var = bf(add_rn(mean, args.eps));
        r = bf(rsqrt_torch(var));
    }

    // ---- normalise, weight, modulate, store ----
    const __nv_bfloat16 *srow = nullptr, *hrow = nullptr;
    if (MODE != ROW_RMS) {
        if (args.nseg > 0) {
            int s = 0;
            while (s + 1 < args.nseg && row >= args.seg_end[s]) ++s;
            srow = args.seg_scale[s];
            hrow = args.seg_shift[s];
        } else {
            srow = args.scale.p + row_offset(args.scale.s0, args.scale.s1, row, args.n1);
            hrow = args.shift.p + row_offset(args.shift.s0, args.shift.s1, row, args.n1);
        }
    }
    __nv_bfloat16 *orow = args.out.p + row_offset(args.out.s0, args.out.s1, row, args.n1);
    const uint32_t r2 = bsplat(r);
    const uint32_t one2 = 0x3f803f80u;                       // (1.0, 1.0) in BF16
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
        const int64_t vi = lane + 32 * k;
        if (vi >= nvec) continue;
        uint4 o;
        if (MODE == ROW_LN_MOD) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                w32(o, i) = bf2u(__floats2bfloat162_rn(__fmaf_rn(blo(w32(v[k], i)), r, shift_ln),
                                                       __fmaf_rn(bhi(w32(v[k], i)), r, shift_ln)));
        } else {
            uint4 w;
            if (VEC && args.wsc == 1) {
                w = *reinterpret_cast<const uint4 *>(args.weight + vi * 8);
            } else {
                float f[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    f[i] = (vi * 8 + i < C) ? __bfloat162float(args.weight[(vi * 8 + i) * args.wsc]) : 0.f;
                w = pack8(f);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) w32(o, i) = bmul2(bmul2(w32(v[k], i), r2), w32(w, i));  // bf(bf(x*r)*w)
        }
        if (MODE != ROW_RMS) {
            const uint4 sc = load8p<VEC>(srow, args.scale.sc, vi * 8, C);
            const uint4 sh = load8p<VEC>(hrow, args.shift.sc, vi * 8, C);
#pragma unroll
            for (int i = 0; i < 4; ++i)     // bf(bf(o * bf(1 + scale)) + shift)
                w32(o, i) = badd2(bmul2(w32(o, i), badd2(w32(sc, i), one2)), w32(sh, i));
        }
        store8p<VEC>(orow, args.out.sc, vi * 8, C, o);
    }
}

// One warp per row; with RPW > 1, RPW consecutive rows per warp, software-
// pipelined (row u+1's loads issued before row u is normalised and stored).
template <int MODE, bool VEC, int VPT, int RPW>
__global__ void __launch_bounds__(ROW_WARPS * 32) row_kernel(RowArgs args) {
    const int lane = threadIdx.x & 31;
    const int64_t row0 = ((int64_t)blockIdx.x * ROW_WARPS + (threadIdx.x >> 5)) * RPW;
    if (row0 >= args.rows) return;  // whole warp leaves together
    uint4 v[2][VPT];   // the second buffer is dead (and not allocated) when RPW == 1
    row_load<MODE, VEC, VPT>(args, row0, lane, v[0]);
#pragma unroll
    for (int u = 0; u < RPW; ++u) {
        if (u + 1 < RPW && row0 + u + 1 < args.rows)
            row_load<MODE, VEC, VPT>(args, row0 + u + 1, lane, v[(u + 1) & 1]);
        if (row0 + u < args.rows) row_finish<MODE, VEC, VPT>(args, row0 + u, lane, v[u & 1]);
    }
}

// Per-256-column partial sums of squares for ROW_RMS_MOD_SQ (h3_rms_modulate_sq):
// sq[row][n] = fp32 sum, in column order, of bf16(x^2) over columns
// [256 n, 256 n + 256) of the row, as a projection epilogue writes them
// (gemm EPI_GATED_RES_SQ).  The row's total: lane l adds partials l, l + 32, ...
// in order, then the xor-16/8/4/2/1 tree.
constexpr int SQ_TILE = 256;

// ===========================================================================
// per-head q/k RMSNorm + RoPE: a half-warp per 128-wide head row
// ===========================================================================
struct HeadArgs {
    const __nv_bfloat16 *x;
    int64_t xs[4];                 // [T, P, Hs, D] strides
    __nv_bfloat16 *out;
    int64_t os[4];
    __nv_bfloat16 *outs[H3_EXCHANGE_MAX_RANKS];  // per-block outputs (nouts > 0): block p at outs[p]
    int nouts;
    const __nv_bfloat16 *weight;   // [128] (norm only)
    int64_t wsc;
    const __nv_bfloat16 *cos, *sin;
    int64_t cs0, cs1, ss0, ss1;
    int64_t T, P, Hs;
    FastDiv div_chunks, div_hs;    // by the head-row chunks per token and by Hs
    uint32_t chunks;               // ceil(P*Hs / HEAD_ROWS_PER_HW)
    int half;                      // rotated pairs (48 or 64); 0 = no rotation
    float eps;
};

#ifndef H3_HEAD_ROWS
#define H3_HEAD_ROWS 2
#endif
#ifndef H3_HEAD_MINB
#define H3_HEAD_MINB 12   // resident CTAs per SM the register allocation must allow (40 registers)
#endif
constexpr int HEAD_THREADS = 128;                                      // 8 half-warps
constexpr int HEAD_ROWS_PER_HW = H3_HEAD_ROWS;                         // rows in flight per half-warp

// A half-warp task is a chunk of up to HEAD_ROWS_PER_HW consecutive head rows
// ph = p * Hs + h of one token t: the token's cos/sin are loaded once per task,
// and all the chunk's rows are loaded before the first is used, so a half-warp
// keeps HEAD_ROWS_PER_HW x 256 B of q/k in flight.
template <bool NORM, bool VEC>
__global__ void __launch_bounds__(HEAD_THREADS, H3_HEAD_MINB) head_kernel(HeadArgs a) {
    const int lane = threadIdx.x & 31;
    const int hl = lane & 15;                    // lane within the half-warp: elements [8hl, 8hl+8)
    const int hw_base = lane & 16;
    const int hw = threadIdx.x >> 4;             // half-warp index in the CTA
    const uint32_t PH = (uint32_t)(a.P * a.Hs), Hs = (uint32_t)a.Hs;
    const int d = a.half >> 3;                   // lanes per rotated half
    const int partner = hl < d ? hl + d : (hl < 2 * d ? hl - d : hl);
    const bool rot_lane = a.half > 0 && hl < 2 * d;

    const uint32_t task = blockIdx.x * (uint32_t)(HEAD_THREADS / 16) + hw;
    const uint32_t t = a.div_chunks.div(task), c = task - t * a.chunks;
    const bool task_ok = t < (uint32_t)a.T;
    uint4 cv = make_uint4(0, 0, 0, 0), sv = make_uint4(0, 0, 0, 0);
    if (task_ok && rot_lane) {
        const int j = 8 * (hl < d ? hl : hl - d);
        cv = load8p<VEC>(a.cos + t * a.cs0 + j * a.cs1, a.cs1, 0, 8);
        sv = load8p<VEC>(a.sin + t * a.ss0 + j * a.ss1, a.ss1, 0, 8);
    }
    uint4 xv[HEAD_ROWS_PER_HW];
    uint32_t pp[HEAD_ROWS_PER_HW], hh[HEAD_ROWS_PER_HW];
    bool ok[HEAD_ROWS_PER_HW];
#pragma unroll
    for (int u = 0; u < HEAD_ROWS_PER_HW; ++u) {
        const uint32_t ph = c * (uint32_t)HEAD_ROWS_PER_HW + u;
        const uint32_t p = a.div_hs.div(ph), h = ph - p * Hs;
        pp[u] = p;
        hh[u] = h;
        ok[u] = task_ok && ph < PH;
        xv[u] = make_uint4(0, 0, 0, 0);
        if (ok[u]) xv[u] = load8p<VEC>(a.x + t * a.xs[0] + p * a.xs[1] + h * a.xs[2], a.xs[3], 8 * hl, 128);
    }
    uint4 w = make_uint4(0, 0, 0, 0);
    if (NORM) {
        if (VEC && a.wsc == 1) {
            w = *reinterpret_cast<const uint4 *>(a.weight + 8 * hl);
        } else {
            float f[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = __bfloat162float(a.weight[(8 * hl + i) * a.wsc]);
            w = pack8(f);
        }
    }
#pragma unroll
    for (int u = 0; u < HEAD_ROWS_PER_HW; ++u) {
        uint4 v = xv[u];
        if (NORM) {
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {        // bf16(x^2), fp32 sum in column order
                const uint32_t sq = bmul2(w32(v, i), w32(v, i));
                s = add_rn(s, blo(sq));
                s = add_rn(s, bhi(sq));
            }
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) s = add_rn(s, __shfl_xor_sync(0xffffffffu, s, o));  // within the half
            const float mean = bf(__fmul_rn(s, 0.0078125f));   // s / 128, exact (power of two)
            const float var = bf(add_rn(mean, a.eps));
            const uint32_t r2 = bsplat(bf(rsqrt_torch(var)));
#pragma unroll
            for (int i = 0; i < 4; ++i) w32(v, i) = bmul2(bmul2(w32(v, i), r2), w32(w, i));  // bf(bf(x*r)*w)
        }
        uint4 o = v;
        if (a.half > 0) {
            uint4 pv;                            // the RoPE partner's values (same row)
            const int src = hw_base | partner;
#pragma unroll
            for (int i = 0; i < 4; ++i) w32(pv, i) = __shfl_sync(0xffffffffu, w32(v, i), src);
            if (rot_lane) {
                // first half:  y0 = bf(bf(a*c) + bf(-b*s));  second half: y1 = bf(bf(b*c) + bf(a*s))
                const bool first = hl < d;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t other = first ? bneg2(w32(pv, i)) : w32(pv, i);
                    w32(o, i) = badd2(bmul2(w32(v, i), w32(cv, i)), bmul2(other, w32(sv, i)));
                }
            }
        }
        if (ok[u]) {
            __nv_bfloat16 *dst = a.nouts > 0 ? a.outs[pp[u]] + t * a.os[0] + hh[u] * a.os[2]
                                             : a.out + t * a.os[0] + pp[u] * a.os[1] + hh[u] * a.os[2];
            store8p<VEC>(dst, a.os[3], 8 * hl, 128, o);
        }
    }
}

// ===========================================================================
// RoPE table and timestep embedding
// ===========================================================================
struct RopeCacheArgs {
    const double *pos;
    int64_t ps0, ps1;
    const float *power[3];  // per-axis power arrays (all equal for the reference table)
    int64_t pws;            // power element stride
    __nv_bfloat16 *out;
    int64_t os0, os1;
    int64_t T;
    int f[3];
    int ftot;
};

__global__ void __launch_bounds__(256) rope_cache_kernel(RopeCacheArgs a) {
    const int64_t total = a.T * a.ftot;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = idx / a.ftot;
        const int j = (int)(idx - t * a.ftot);
        const int axis = j < a.f[0] ? 0 : (j < a.f[0] + a.f[1] ? 1 : 2);
        const int k = j - (axis > 0 ? a.f[0] : 0) - (axis > 1 ? a.f[1] : 0);
        const float position = __double2float_rn(a.pos[t * a.ps0 + axis * a.ps1]);
        const float inverse = __fdiv_rn(1.0f, a.power[axis][k * a.pws]);
        const float angle = __fmul_rn(position, inverse);
        // cos/sin evaluated in double and rounded once to fp32: the correctly
        // rounded fp32 value, which the CPU reference's fp32 cos/sin match to 1 ulp.
        const float c = (float)cos((double)angle);
        const float s = (float)sin((double)angle);
        a.out[t * a.os0 + j * a.os1] = __float2bfloat16_rn(c);
        a.out[t * a.os0 + (a.ftot + j) * a.os1] = __float2bfloat16_rn(s);
    }
}

__global__ void __launch_bounds__(256) timestep_embedding_kernel(float *out, int64_t os0, int64_t os1,
                                                                 const float *t, int64_t ts, int64_t n,
                                                                 int64_t dim, float log_max_period) {
    const int64_t total = n * dim;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = idx / dim, c = idx - i * dim;
        const int64_t half = dim / 2;
        const int64_t k = c < half ? c : c - half;
        // exp / cos / sin evaluated in double and rounded once: the correctly
        // rounded fp32 values, so large timesteps (t * f up to ~1e3 rad) do not
        // amplify a 1-ulp frequency difference
        const float expo = __fdiv_rn(__fmul_rn(-log_max_period, (float)k), (float)half);
        const float freq = (float)exp((double)expo);
        const float angle = __fmul_rn(t[i * ts], freq);
        out[i * os0 + c * os1] = c < half ? (float)cos((double)angle) : (float)sin((double)angle);
    }
}

// ===========================================================================
// host-side launchers
// ===========================================================================
static int grid_for(int64_t work, int threads) {
    int64_t blocks = (work + threads - 1) / threads;
    const int64_t cap = (int64_t)num_sms() * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

static RowView rowview(const h3_tensor *t) {
    RowView r;
    r.p = static_cast<const __nv_bfloat16 *>(t->data);
    lead_strides(t, &r.s0, &r.s1);
    r.sc = t->strides[t->ndim - 1];
    return r;
}
static RowViewMut rowview_mut(const h3_tensor *t) {
    RowViewMut r;
    r.p = static_cast<__nv_bfloat16 *>(t->data);
    lead_strides(t, &r.s0, &r.s1);
    r.sc = t->strides[t->ndim - 1];
    return r;
}

template <int OP>
static int launch_ew(const h3_tensor *o, const h3_tensor *a, const h3_tensor *b, const h3_tensor *c,
                     cudaStream_t stream) {
    EwArgs args;
    args.a = rowview(a);
    args.b = rowview(b);
    args.c = c ? rowview(c) : args.b;
    args.o = rowview_mut(o);
    lead_dims(o, &args.rows, &args.n1);
    args.C = o->shape[o->ndim - 1];
    if (args.rows == 0 || args.C == 0) return H3_OK;
    const bool vec = rows_vectorizable(o, 8) && rows_vectorizable(a, 8) && rows_vectorizable(b, 8) &&
                     (!c || rows_vectorizable(c, 8));
    const int64_t nvec = (args.C + 7) / 8;
    const int64_t total = args.rows * nvec;
    if (total > 0x7fffffffLL) return H3_ERR_UNSUPPORTED;
    const unsigned grid = (unsigned)((total + EW_THREADS * EW_VPT - 1) / (EW_THREADS * EW_VPT));
    const FastDiv dn = FastDiv::make((uint32_t)nvec);
    if (vec) ew_kernel<OP, true><<<grid, EW_THREADS, 0, stream>>>(args, dn, (uint32_t)total);
    else ew_kernel<OP, false><<<grid, EW_THREADS, 0, stream>>>(args, dn, (uint32_t)total);
    return launch_status();
}

template <int MODE>
static int launch_row(RowArgs &args, bool vec, cudaStream_t stream) {
    if (args.rows == 0 || args.C == 0) return H3_OK;
    const int64_t nvec = (args.C + 7) / 8;
    const int vpt = (int)((nvec + 31) / 32);
    // rows per warp follow the instantiated width bucket: H3_ROW_PIPE_RPW for buckets
    // <= H3_ROW_PIPE_MAXV vectors per lane, else 1; the grid is sized from the same constant
#define H3_ROW_LAUNCH(VEC_, V)                                                              \
    {                                                                                       \
        constexpr int R = (V) <= H3_ROW_PIPE_MAXV ? H3_ROW_PIPE_RPW : 1;                    \
        const int64_t blocks = (args.rows + ROW_WARPS * R - 1) / (ROW_WARPS * R);           \
        if (blocks > 0x7fffffffLL) return H3_ERR_UNSUPPORTED;                               \
        row_kernel<MODE, VEC_, V, R><<<(unsigned)blocks, ROW_WARPS * 32, 0, stream>>>(args); \
        return launch_status();                                                             \
    }
#define H3_ROW_VEC(V) \
    if (vec && vpt <= V) H3_ROW_LAUNCH(true, V)
#define H3_ROW_STRIDED(V) \
    if (!vec && vpt <= V) H3_ROW_LAUNCH(false, V)
    H3_ROW_VEC(1)
    H3_ROW_VEC(2)
    H3_ROW_VEC(4)
    H3_ROW_VEC(8)
    H3_ROW_VEC(12)
    H3_ROW_VEC(16)
    H3_ROW_VEC(20)
    H3_ROW_VEC(24)
    H3_ROW_VEC(32)
    H3_ROW_STRIDED(4)
    H3_ROW_STRIDED(16)
    H3_ROW_STRIDED(32)
#undef H3_ROW_VEC
#undef H3_ROW_STRIDED
#undef H3_ROW_LAUNCH
    return H3_ERR_UNSUPPORTED;  // rows wider than 8192 elements
}

}  // namespace h3

using namespace h3;

// ===========================================================================
// C-ABI
// ===========================================================================
extern "C" int h3_gated_residual(const h3_tensor *out, const h3_tensor *x, const h3_tensor *gate,
                                 const h3_tensor *y, void *stream) {
    H3_CHECK(check_bf16(out) ?: check_bf16(x) ?: check_bf16(gate) ?: check_bf16(y));
    H3_CHECK(check_rank(out, 2, 3) ?: check_same_shape(out, x) ?: check_same_shape(out, gate) ?:
             check_same_shape(out, y));
    return launch_ew<EW_GATED_RESIDUAL>(out, x, gate, y, (cudaStream_t)stream);
}

extern "C" int h3_swiglu(const h3_tensor *y, const h3_tensor *up, const h3_tensor *gate, void *stream) {
    H3_CHECK(check_bf16(y) ?: check_bf16(up) ?: check_bf16(gate));
    H3_CHECK(check_rank(y, 2, 3) ?: check_same_shape(y, up) ?: check_same_shape(y, gate));
    return launch_ew<EW_SWIGLU>(y, up, gate, nullptr, (cudaStream_t)stream);
}

static int fill_row_args(RowArgs &a, const h3_tensor *out, const h3_tensor *x, const h3_tensor *weight,
                         const h3_tensor *scale, const h3_tensor *shift, float eps, bool *vec) {
    a.x = rowview(x);
    a.out = rowview_mut(out);
    a.gate = a.y = a.x;
    a.residual = a.out;
    a.scale = scale ? rowview(scale) : a.x;
    a.shift = shift ? rowview(shift) : a.x;
    a.weight = weight ? static_cast<const __nv_bfloat16 *>(weight->data) : nullptr;
    a.wsc = weight ? weight->strides[0] : 1;
    lead_dims(out, &a.rows, &a.n1);
    a.C = out->shape[out->ndim - 1];
    a.eps = eps;
    a.sq = nullptr;
    a.ldsq = 0;
    a.nt = 0;
    a.nseg = 0;
    *vec = rows_vectorizable(out, 8) && rows_vectorizable(x, 8) && (!scale || rows_vectorizable(scale, 8)) &&
           (!shift || rows_vectorizable(shift, 8)) &&
           (!weight || (weight->strides[0] == 1 && aligned16(weight->data)));
    return H3_OK;
}

static int check_weight(const h3_tensor *w, int64_t C) {
    H3_CHECK(check_bf16(w));
    if (w->ndim != 1 || w->shape[0] != C) return H3_ERR_BAD_SHAPE;
    return H3_OK;
}

extern "C" int h3_rms_norm(const h3_tensor *y, const h3_tensor *x, const h3_tensor *weight, float eps,
                           void *stream) {
    H3_CHECK(check_bf16(y) ?: check_bf16(x));
    H3_CHECK(check_rank(x, 2, 3) ?: check_same_shape(y, x));
    H3_CHECK(check_weight(weight, x->shape[x->ndim - 1]));
    RowArgs a;
    bool vec;
    fill_row_args(a, y, x, weight, nullptr, nullptr, eps, &vec);
    return launch_row<ROW_RMS>(a, vec, (cudaStream_t)stream);
}

extern "C" int h3_rms_modulate(const h3_tensor *y, const h3_tensor *x, const h3_tensor *weight,
                               const h3_tensor *scale, const h3_tensor *shift, float eps, void *stream) {
    H3_CHECK(check_bf16(y) ?: check_bf16(x) ?: check_bf16(scale) ?: check_bf16(shift));
    H3_CHECK(check_rank(x, 2, 3) ?: check_same_shape(y, x) ?: check_same_shape(scale, x) ?:
             check_same_shape(shift, x));
    H3_CHECK(check_weight(weight, x->shape[x->ndim - 1]));
    RowArgs a;
    bool vec;
    fill_row_args(a, y, x, weight, scale, shift, eps, &vec);
    return launch_row<ROW_RMS_MOD>(a, vec, (cudaStream_t)stream);
}

extern "C" int h3_ln_modulate(const h3_tensor *y, const h3_tensor *x, const h3_tensor *scale,
                              const h3_tensor *shift, float eps, void *stream) {
    H3_CHECK(check_bf16(y) ?: check_bf16(x) ?: check_bf16(scale) ?: check_bf16(shift));
    H3_CHECK(check_rank(x, 2, 3) ?: check_same_shape(y, x) ?: check_same_shape(scale, x) ?:
             check_same_shape(shift, x));
    RowArgs a;
    bool vec;
    fill_row_args(a, y, x, nullptr, scale, shift, eps, &vec);
    return launch_row<ROW_LN_MOD>(a, vec, (cudaStream_t)stream);
}

extern "C" int h3_gated_residual_rms_modulate(const h3_tensor *residual, const h3_tensor *out,
                                              const h3_tensor *x, const h3_tensor *gate, const h3_tensor *y,
                                              const h3_tensor *weight, const h3_tensor *scale,
                                              const h3_tensor *shift, float eps, void *stream) {
    H3_CHECK(check_bf16(residual) ?: check_bf16(out) ?: check_bf16(x) ?: check_bf16(gate) ?: check_bf16(y) ?:
             check_bf16(scale) ?: check_bf16(shift));
    H3_CHECK(check_rank(x, 2, 3) ?: check_same_shape(out, x) ?: check_same_shape(residual, x) ?:
             check_same_shape(gate, x) ?: check_same_shape(y, x) ?: check_same_shape(scale, x) ?:
             check_same_shape(shift, x));
    H3_CHECK(check_weight(weight, x->shape[x->ndim - 1]));
    RowArgs a;
    bool vec;
    fill_row_args(a, out, x, weight, scale, shift, eps, &vec);
    a.gate = rowview(gate);
    a.y = rowview(y);
    a.residual = rowview_mut(residual);
    vec = vec && rows_vectorizable(gate, 8) && rows_vectorizable(y, 8) && rows_vectorizable(residual, 8);
    return launch_row<ROW_RES_RMS_MOD>(a, vec, (cudaStream_t)stream);
}

extern "C" int h3_rms_modulate_sq(const h3_tensor *y, const h3_tensor *x, const h3_tensor *sq,
                                  const h3_tensor *weight, const h3_tensor *scale, const h3_tensor *shift, float eps,
                                  void *stream) {
    H3_CHECK(check_bf16(y) ?: check_bf16(x) ?: check_bf16(scale) ?: check_bf16(shift) ?: check_desc(sq, H3_F32));
    H3_CHECK(check_rank(x, 2, 3) ?: check_same_shape(y, x) ?: check_same_shape(scale, x) ?:
             check_same_shape(shift, x));
    const int64_t C = x->shape[x->ndim - 1];
    H3_CHECK(check_weight(weight, C));
    RowArgs a;
    bool vec;
    fill_row_args(a, y, x, weight, scale, shift, eps, &vec);
    a.nt = (int)((C + SQ_TILE - 1) / SQ_TILE);
    if (sq->ndim != 2 || sq->shape[0] != a.rows || sq->shape[1] != a.nt) return H3_ERR_BAD_SHAPE;
    if ((a.nt > 1 && sq->strides[1] != 1) || (a.rows > 1 && sq->strides[0] < a.nt)) return H3_ERR_BAD_LAYOUT;
    a.sq = static_cast<const float *>(sq->data);
    a.ldsq = sq->strides[0];
    return launch_row<ROW_RMS_MOD_SQ>(a, vec, (cudaStream_t)stream);
}

extern "C" int h3_rms_modulate_segmented(const h3_tensor *y, const h3_tensor *x, const h3_tensor *sq,
                                         const h3_tensor *weight, const h3_tensor *scales, const h3_tensor *shifts,
                                         const int64_t *seg_rows, int32_t nseg, float eps, void *stream) {
    H3_CHECK(check_bf16(y) ?: check_bf16(x));
    H3_CHECK(check_rank(x, 2, 2) ?: check_same_shape(y, x));
    if (!scales || !shifts || !seg_rows) return H3_ERR_NULL;
    if (nseg < 1) return H3_ERR_BAD_SHAPE;
    if (nseg > H3_MAX_SEGMENTS) return H3_ERR_UNSUPPORTED;
    const int64_t C = x->shape[1];
    H3_CHECK(check_weight(weight, C));
    RowArgs a;
    bool vec;
    fill_row_args(a, y, x, weight, nullptr, nullptr, eps, &vec);
    int64_t end = 0;
    for (int i = 0; i < nseg; ++i) {
        for (const h3_tensor *t : {&scales[i], &shifts[i]}) {
            H3_CHECK(check_bf16(t));
            if (t->ndim != 1 || t->shape[0] != C) return H3_ERR_BAD_SHAPE;
            if ((C > 1 && t->strides[0] != 1) || !aligned16(t->data)) return H3_ERR_BAD_LAYOUT;
        }
        if (seg_rows[i] < 0) return H3_ERR_BAD_SHAPE;
        end += seg_rows[i];
        a.seg_end[i] = end;
        a.seg_scale[i] = static_cast<const __nv_bfloat16 *>(scales[i].data);
        a.seg_shift[i] = static_cast<const __nv_bfloat16 *>(shifts[i].data);
    }
    if (end != a.rows) return H3_ERR_BAD_SHAPE;
    a.nseg = nseg;
    // the segment rows are contiguous: the strided load path reads them with stride 1
    a.scale.p = a.seg_scale[0];
    a.shift.p = a.seg_shift[0];
    a.scale.s0 = a.scale.s1 = a.shift.s0 = a.shift.s1 = 0;
    a.scale.sc = a.shift.sc = 1;
    if (!sq) return launch_row<ROW_RMS_MOD>(a, vec, (cudaStream_t)stream);
    H3_CHECK(check_desc(sq, H3_F32));
    a.nt = (int)((C + SQ_TILE - 1) / SQ_TILE);
    if (sq->ndim != 2 || sq->shape[0] != a.rows || sq->shape[1] != a.nt) return H3_ERR_BAD_SHAPE;
    if ((a.nt > 1 && sq->strides[1] != 1) || (a.rows > 1 && sq->strides[0] < a.nt)) return H3_ERR_BAD_LAYOUT;
    a.sq = static_cast<const float *>(sq->data);
    a.ldsq = sq->strides[0];
    return launch_row<ROW_RMS_MOD_SQ>(a, vec, (cudaStream_t)stream);
}

static int head_launch(const h3_tensor *out, const h3_tensor *x, const h3_tensor *weight,
                       const h3_tensor *cos, const h3_tensor *sin, float eps, bool norm, cudaStream_t stream,
                       const h3_tensor *outs = nullptr, int nouts = 0) {
    // x/out are [T, P, Hs, 128] (4-D) or [S, H, 128] (3-D, seen as P = 1); with nouts > 0,
    // x is [T, nouts, Hs, 128] and block p goes to outs[p], each [T, Hs, 128]
    HeadArgs a;
    a.nouts = nouts;
    for (int i = 0; i < H3_EXCHANGE_MAX_RANKS; ++i) a.outs[i] = nullptr;
    int64_t shp[4], xs[4], os[4];
    if (x->ndim == 4) {
        for (int i = 0; i < 4; ++i) { shp[i] = x->shape[i]; xs[i] = x->strides[i]; os[i] = out ? out->strides[i] : 0; }
    } else {
        shp[0] = x->shape[0]; shp[1] = 1; shp[2] = x->shape[1]; shp[3] = x->shape[2];
        xs[0] = x->strides[0]; xs[1] = 0; xs[2] = x->strides[1]; xs[3] = x->strides[2];
        if (!out) return H3_ERR_NULL;
        os[0] = out->strides[0]; os[1] = 0; os[2] = out->strides[1]; os[3] = out->strides[2];
    }
    if (nouts > 0) {
        // per-block outputs: strides of outs[0] ([T, Hs, 128]) as (t, -, h, d)
        os[0] = outs[0].strides[0]; os[1] = 0; os[2] = outs[0].strides[1]; os[3] = outs[0].strides[2];
        for (int i = 0; i < nouts; ++i) a.outs[i] = static_cast<__nv_bfloat16 *>(outs[i].data);
    }
    a.x = static_cast<const __nv_bfloat16 *>(x->data);
    a.out = nouts > 0 ? a.outs[0] : static_cast<__nv_bfloat16 *>(out->data);
    for (int i = 0; i < 4; ++i) { a.xs[i] = xs[i]; a.os[i] = os[i]; }
    a.weight = weight ? static_cast<const __nv_bfloat16 *>(weight->data) : nullptr;
    a.wsc = weight ? weight->strides[0] : 1;
    a.cos = static_cast<const __nv_bfloat16 *>(cos->data);
    a.sin = static_cast<const __nv_bfloat16 *>(sin->data);
    a.cs0 = cos->strides[0]; a.cs1 = cos->strides[1];
    a.ss0 = sin->strides[0]; a.ss1 = sin->strides[1];
    a.T = shp[0]; a.P = shp[1]; a.Hs = shp[2];
    if (a.P * a.Hs <= 0 || a.P * a.Hs > 0x7fffffffLL) return a.T == 0 || a.P * a.Hs == 0 ? H3_OK : H3_ERR_UNSUPPORTED;
    a.chunks = (uint32_t)((a.P * a.Hs + HEAD_ROWS_PER_HW - 1) / HEAD_ROWS_PER_HW);
    a.div_chunks = FastDiv::make(a.chunks);
    a.div_hs = FastDiv::make((uint32_t)a.Hs);
    a.half = (int)cos->shape[1];
    a.eps = eps;
    const int64_t rows = a.T * a.P * a.Hs;
    if (rows == 0) return H3_OK;
    bool vec = xs[3] == 1 && os[3] == 1 && a.cs1 == 1 && a.ss1 == 1 && aligned16(x->data) &&
               aligned16(a.out) && aligned16(cos->data) && aligned16(sin->data);
    for (int i = 0; i < nouts; ++i) vec = vec && aligned16(a.outs[i]);
    for (int i = 0; i < 3; ++i) vec = vec && (xs[i] % 8 == 0) && (os[i] % 8 == 0);
    vec = vec && a.cs0 % 8 == 0 && a.ss0 % 8 == 0;
    const int64_t tasks = a.T * (int64_t)a.chunks;
    if (rows > 0x7fffffffLL || tasks > 0x7fffffffLL) return H3_ERR_UNSUPPORTED;
    const unsigned g = (unsigned)((tasks + HEAD_THREADS / 16 - 1) / (HEAD_THREADS / 16));
    if (norm) {
        if (vec) head_kernel<true, true><<<g, HEAD_THREADS, 0, stream>>>(a);
        else head_kernel<true, false><<<g, HEAD_THREADS, 0, stream>>>(a);
    } else {
        if (vec) head_kernel<false, true><<<g, HEAD_THREADS, 0, stream>>>(a);
        else head_kernel<false, false><<<g, HEAD_THREADS, 0, stream>>>(a);
    }
    return launch_status();
}

static int check_angles(const h3_tensor *cos, const h3_tensor *sin, int64_t T) {
    H3_CHECK(check_bf16(cos) ?: check_bf16(sin));
    if (cos->ndim != 2 || cos->shape[0] != T) return H3_ERR_BAD_SHAPE;
    H3_CHECK(check_same_shape(cos, sin));
    const int64_t half = cos->shape[1];
    if (half <= 0 || half % 8 != 0 || 2 * half > 128) return H3_ERR_BAD_SHAPE;
    return H3_OK;
}

extern "C" int h3_rope(const h3_tensor *y, const h3_tensor *x, const h3_tensor *cos, const h3_tensor *sin,
                       void *stream) {
    H3_CHECK(check_bf16(y) ?: check_bf16(x));
    if (x->ndim != 3 || x->shape[2] != 128) return H3_ERR_BAD_SHAPE;
    H3_CHECK(check_same_shape(y, x));
    H3_CHECK(check_angles(cos, sin, x->shape[0]));
    return head_launch(y, x, nullptr, cos, sin, 0.f, false, (cudaStream_t)stream);
}

// One launch for every destination block of the sequence-parallel exchange:
// x [T, n, Hs, 128], outs[p] [T, Hs, 128] (all the same shape and strides).
extern "C" int h3_qk_norm_rope_multi(const h3_tensor *outs, int32_t n, const h3_tensor *x, const h3_tensor *weight,
                                     const h3_tensor *cos, const h3_tensor *sin, float eps, void *stream) {
    if (!outs) return H3_ERR_NULL;
    H3_CHECK(check_bf16(x));
    if (n < 1 || n > H3_EXCHANGE_MAX_RANKS) return H3_ERR_BAD_SHAPE;
    if (x->ndim != 4 || x->shape[1] != n || x->shape[3] != 128) return H3_ERR_BAD_SHAPE;
    for (int i = 0; i < n; ++i) {
        H3_CHECK(check_bf16(&outs[i]));
        if (outs[i].ndim != 3 || outs[i].shape[0] != x->shape[0] || outs[i].shape[1] != x->shape[2] ||
            outs[i].shape[2] != 128)
            return H3_ERR_BAD_SHAPE;
        for (int j = 0; j < 3; ++j)
            if (outs[i].strides[j] != outs[0].strides[j]) return H3_ERR_BAD_LAYOUT;
    }
    H3_CHECK(check_weight(weight, 128));
    H3_CHECK(check_angles(cos, sin, x->shape[0]));
    return head_launch(nullptr, x, weight, cos, sin, eps, true, (cudaStream_t)stream, outs, n);
}

extern "C" int h3_qk_norm_rope(const h3_tensor *out, const h3_tensor *x, const h3_tensor *weight,
                               const h3_tensor *cos, const h3_tensor *sin, float eps, void *stream) {
    H3_CHECK(check_bf16(out) ?: check_bf16(x));
    if (x->ndim != 4 || x->shape[3] != 128) return H3_ERR_BAD_SHAPE;
    H3_CHECK(check_same_shape(out, x));
    H3_CHECK(check_weight(weight, 128));
    H3_CHECK(check_angles(cos, sin, x->shape[0]));
    return head_launch(out, x, weight, cos, sin, eps, true, (cudaStream_t)stream);
}

static int rope_cache_launch(const h3_tensor *out, const h3_tensor *position, const float *p0, const float *p1,
                             const float *p2, int64_t pws, int f0, int f1, int f2, cudaStream_t stream) {
    RopeCacheArgs a;
    a.pos = static_cast<const double *>(position->data);
    a.ps0 = position->strides[0];
    a.ps1 = position->strides[1];
    a.power[0] = p0; a.power[1] = p1; a.power[2] = p2;
    a.pws = pws;
    a.out = static_cast<__nv_bfloat16 *>(out->data);
    a.os0 = out->strides[0];
    a.os1 = out->strides[1];
    a.T = position->shape[0];
    a.f[0] = f0; a.f[1] = f1; a.f[2] = f2;
    a.ftot = f0 + f1 + f2;
    if (a.T == 0) return H3_OK;
    rope_cache_kernel<<<grid_for(a.T * a.ftot, 256), 256, 0, stream>>>(a);
    return launch_status();
}

extern "C" int h3_rope_cache(const h3_tensor *out, const h3_tensor *position, const h3_tensor *power,
                             void *stream) {
    H3_CHECK(check_desc(out, H3_BF16));
    H3_CHECK(check_desc(position, H3_F64));
    H3_CHECK(check_desc(power, H3_F32));
    if (position->ndim != 2 || position->shape[1] != 3 || power->ndim != 1 || power->shape[0] != 16)
        return H3_ERR_BAD_SHAPE;
    if (out->ndim != 2 || out->shape[0] != position->shape[0] || out->shape[1] != 96) return H3_ERR_BAD_SHAPE;
    const float *p = static_cast<const float *>(power->data);
    return rope_cache_launch(out, position, p, p, p, power->strides[0], 16, 16, 16, (cudaStream_t)stream);
}

extern "C" int h3_rope_cache_sectioned(const h3_tensor *out, const h3_tensor *position, const h3_tensor *power,
                                       int32_t f0, int32_t f1, int32_t f2, void *stream) {
    H3_CHECK(check_desc(out, H3_BF16));
    H3_CHECK(check_desc(position, H3_F64));
    H3_CHECK(check_desc(power, H3_F32));
    if (f0 <= 0 || f1 <= 0 || f2 <= 0) return H3_ERR_BAD_SHAPE;
    const int ftot = f0 + f1 + f2;
    if (position->ndim != 2 || position->shape[1] != 3 || power->ndim != 1 || power->shape[0] != ftot)
        return H3_ERR_BAD_SHAPE;
    if (out->ndim != 2 || out->shape[0] != position->shape[0] || out->shape[1] != 2 * ftot) return H3_ERR_BAD_SHAPE;
    const float *p = static_cast<const float *>(power->data);
    const int64_t s = power->strides[0];
    return rope_cache_launch(out, position, p, p + f0 * s, p + (f0 + f1) * s, s, f0, f1, f2,
                             (cudaStream_t)stream);
}

extern "C" int h3_timestep_embedding(const h3_tensor *out, const h3_tensor *t, float max_period, void *stream) {
    H3_CHECK(check_desc(out, H3_F32));
    H3_CHECK(check_desc(t, H3_F32));
    if (t->ndim != 1 || out->ndim != 2 || out->shape[0] != t->shape[0] || out->shape[1] % 2 != 0 ||
        out->shape[1] <= 0)
        return H3_ERR_BAD_SHAPE;
    const int64_t n = t->shape[0], dim = out->shape[1];
    if (n == 0) return H3_OK;
    timestep_embedding_kernel<<<grid_for(n * dim, 256), 256, 0, (cudaStream_t)stream>>>(
        static_cast<float *>(out->data), out->strides[0], out->strides[1], static_cast<const float *>(t->data),
        t->strides[0], n, dim, logf(max_period));
    return launch_status();
}
