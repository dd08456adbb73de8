// Model-wrapper ops around the block stack: fp32 linears (patch and audio
// projections in and out, the time MLP), row gather / scatter for packing the
// joint sequence, and SiLU.  None is on the per-block path; together they are
// well under 1 % of a denoising step.
//
//   h3_linear_f32      linear_forward on the F32 modules of MiniMaxH3Transformer
//                      (proj_in / audio_proj_in InfiniLM.patch:1662-1664, proj_out /
//                      audio_proj_out :1812-1814, time embedder :1501-1517)
//   h3_gather_rows     gather_rows -> embedding(indices, table) :587-590, used by
//                      OutputNorm (:1530-1538) and the final output gather (:1822-1823)
//   h3_index_copy_rows index_copy of text/video/audio embeddings into the packed
//                      sequence :1685-1690
//   h3_silu            op::silu (fp32) followed by cast_to :1267-1268, 1511, 1535
//   h3_adaln_projection MiniMaxH3AdaLNProjection::forward's linear + bias
//                      (:1260-1279) for its few conditioning rows
#include <math.h>
#include <stdint.h>

#include "h3_abi_util.h"
#include "h3_common.cuh"
#include "sm100_ptx.cuh"

namespace h3 {
namespace mops {

// ---------------------------------------------------------------------------
// fp32 linear: y[M,N] = x[M,K] w[N,K]^T (+ b[N]); x BF16 or F32, w/b F32, y F32
// or BF16 (the fp32 result rounded once, as cast_to after an F32 linear).
// 64x64 output tile per 256-thread CTA, 4x4 outputs per thread, K in steps of 16
// through shared memory (transposed so the inner loop reads are conflict-free).
// Each output accumulates its K products in increasing k with fmaf.  For at most
// GEMV_ROWS rows (the time MLP runs on one timestep) a warp per output column
// streams its weight row instead: lane-strided partial sums, then a fixed
// butterfly reduction.  Either way the result of a row depends only on M's path,
// not on the other rows.
// ---------------------------------------------------------------------------
constexpr int LT = 64, LK = 16;

struct LinArgs {
    const void *x;
    const float *w, *b;
    void *y;
    int64_t M, N, K, sx, sw, sy;  // row strides in elements
    int x_bf16, y_bf16;
};

__global__ void __launch_bounds__(256) linear_f32_kernel(LinArgs a) {
    __shared__ float xs[LK][LT + 4];
    __shared__ float ws[LK][LT + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t m0 = (int64_t)blockIdx.y * LT, n0 = (int64_t)blockIdx.x * LT;
    float acc[4][4] = {};
    for (int64_t k0 = 0; k0 < a.K; k0 += LK) {
        // 64 rows x 16 k of x and of w: 1024 elements each, 4 per thread
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int e = threadIdx.x + 256 * i;
            const int r = e >> 4, kk = e & 15;
            const int64_t m = m0 + r, n = n0 + r, k = k0 + kk;
            float xv = 0.f, wv = 0.f;
            if (m < a.M && k < a.K) {
                xv = a.x_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16 *>(a.x)[m * a.sx + k])
                              : static_cast<const float *>(a.x)[m * a.sx + k];
            }
            if (n < a.N && k < a.K) wv = a.w[n * a.sw + k];
            xs[kk][r] = xv;
            ws[kk][r] = wv;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < LK; ++kk) {
            float xr[4], wr[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                xr[i] = xs[kk][ty + 16 * i];
                wr[i] = ws[kk][tx + 16 * i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xr[i], wr[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t m = m0 + ty + 16 * i;
        if (m >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t n = n0 + tx + 16 * j;
            if (n >= a.N) continue;
            const float v = a.b ? __fadd_rn(acc[i][j], a.b[n]) : acc[i][j];
            if (a.y_bf16) static_cast<__nv_bfloat16 *>(a.y)[m * a.sy + n] = __float2bfloat16_rn(v);
            else static_cast<float *>(a.y)[m * a.sy + n] = v;
        }
    }
}

constexpr int GEMV_ROWS = 8;

__global__ void __launch_bounds__(256) linear_f32_gemv_kernel(LinArgs a) {
    const int64_t n = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (n >= a.N) return;
    float acc[GEMV_ROWS] = {};
    const float *wr = a.w + n * a.sw;
    for (int64_t k = lane; k < a.K; k += 32) {
        const float wv = wr[k];
#pragma unroll
        for (int m = 0; m < GEMV_ROWS; ++m) {
            if (m < a.M) {
                const float xv = a.x_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16 *>(a.x)[m * a.sx + k])
                                          : static_cast<const float *>(a.x)[m * a.sx + k];
                acc[m] = fmaf(xv, wv, acc[m]);
            }
        }
    }
#pragma unroll
    for (int m = 0; m < GEMV_ROWS; ++m) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[m] = __fadd_rn(acc[m], __shfl_xor_sync(0xffffffffu, acc[m], o));
    }
    if (lane == 0) {
        for (int m = 0; m < GEMV_ROWS && m < a.M; ++m) {
            const float v = a.b ? __fadd_rn(acc[m], a.b[n]) : acc[m];
            if (a.y_bf16) static_cast<__nv_bfloat16 *>(a.y)[m * a.sy + n] = __float2bfloat16_rn(v);
            else static_cast<float *>(a.y)[m * a.sy + n] = v;
        }
    }
}

// ---------------------------------------------------------------------------
// AdaLN projection: y[M,N] = bf16(bf16(x[M,K] w[N,K]^T) + b[N]), all BF16, M <=
// ADALN_ROWS.  The weight (6 x modalities x Hd rows of Hd) is read once and is
// the whole cost, so this is a streaming kernel: a warp per weight row, each
// lane 16-byte chunks lane, lane + 32, ... of it (512 contiguous bytes per warp
// load, ADALN_UNROLL loads in flight per lane), fp32 products accumulated in
// chunk order per lane, then a xor-16/8/4/2/1 tree.  The grid covers every SM
// however the rows are split across ranks (a GEMM tile grid over 11520 rows,
// one rank's share on 8 GPUs, fills 45 SMs).
// ---------------------------------------------------------------------------
constexpr int ADALN_ROWS = 4;
constexpr int ADALN_UNROLL = 5;

struct AdaArgs {
    const __nv_bfloat16 *x, *w, *b;
    __nv_bfloat16 *y;
    int64_t M, N, K, sx, sw, sy;
};

__global__ void __launch_bounds__(256) adaln_projection_kernel(AdaArgs a) {
    const int64_t n = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (n >= a.N) return;
    const uint4 *wr = reinterpret_cast<const uint4 *>(a.w + n * a.sw);
    const int64_t chunks = a.K / 8;
    float acc[ADALN_ROWS] = {};
    for (int64_t c0 = lane; c0 < chunks; c0 += 32 * ADALN_UNROLL) {
        uint4 wv[ADALN_UNROLL];
#pragma unroll
        for (int u = 0; u < ADALN_UNROLL; ++u) {
            const int64_t c = c0 + 32 * u;
            if (c < chunks) wv[u] = __ldcs(wr + c);   // streamed once: keep it out of L2's way
        }
#pragma unroll
        for (int u = 0; u < ADALN_UNROLL; ++u) {
            const int64_t c = c0 + 32 * u;
            if (c >= chunks) break;
            const __nv_bfloat16 *we = reinterpret_cast<const __nv_bfloat16 *>(&wv[u]);
#pragma unroll
            for (int m = 0; m < ADALN_ROWS; ++m) {
                if (m < a.M) {
                    const uint4 xv = __ldg(reinterpret_cast<const uint4 *>(a.x + m * a.sx) + c);
                    const __nv_bfloat16 *xe = reinterpret_cast<const __nv_bfloat16 *>(&xv);
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        acc[m] = fmaf(__bfloat162float(xe[e]), __bfloat162float(we[e]), acc[m]);
                }
            }
        }
    }
#pragma unroll
    for (int m = 0; m < ADALN_ROWS; ++m) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc[m] = __fadd_rn(acc[m], __shfl_xor_sync(0xffffffffu, acc[m], o));
    }
    if (lane == 0) {
        for (int m = 0; m < ADALN_ROWS && m < a.M; ++m) {
            float v = __bfloat162float(__float2bfloat16_rn(acc[m]));   // the linear's BF16 output
            if (a.b) v = __fadd_rn(v, __bfloat162float(a.b[n]));        // + bias, one BF16 rounding
            a.y[m * a.sy + n] = __float2bfloat16_rn(v);
        }
    }
}

// ---------------------------------------------------------------------------
// Row gather / scatter.  One warp per row; 16-byte vectors when every row start
// is 16-byte aligned, else elements.  An index outside [0, rows) of the indexed
// tensor leaves that row untouched and raises the device error word.
// ---------------------------------------------------------------------------
struct RowMoveArgs {
    const uint8_t *src;
    uint8_t *dst;
    const int64_t *idx;
    int64_t rows;        // number of indices
    int64_t limit;       // rows of the indexed tensor
    int64_t row_bytes;
    int64_t s_src, s_dst;  // row strides in bytes
    int scatter;           // 0: dst[r] = src[idx[r]]; 1: dst[idx[r]] = src[r]
    int vec16;
};

__global__ void __launch_bounds__(256) row_move_kernel(RowMoveArgs a) {
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= a.rows) return;
    const int64_t i = a.idx[r];
    if (i < 0 || i >= a.limit) {
        if (lane == 0) atomicOr(&g_h3_device_error, 2u);
        return;
    }
    const uint8_t *s = a.src + (a.scatter ? r : i) * a.s_src;
    uint8_t *d = a.dst + (a.scatter ? i : r) * a.s_dst;
    if (a.vec16) {
        for (int64_t o = (int64_t)lane * 16; o < a.row_bytes; o += 32 * 16)
            *reinterpret_cast<uint4 *>(d + o) = *reinterpret_cast<const uint4 *>(s + o);
    } else {
        for (int64_t o = (int64_t)lane * 2; o < a.row_bytes; o += 32 * 2)
            *reinterpret_cast<uint16_t *>(d + o) = *reinterpret_cast<const uint16_t *>(s + o);
    }
}

// ---------------------------------------------------------------------------
// Block copy: src [n, R, C] (strided) -> dst[b] [R, C], one launch for all n
// blocks (the v and attention-output legs of the sequence-parallel exchange).
// ---------------------------------------------------------------------------
struct BlockCopyArgs {
    const uint8_t *src;
    uint8_t *dst[H3_EXCHANGE_MAX_RANKS];
    int64_t n, rows, row_bytes;
    int64_t s_blk, s_row, d_row;   // bytes
    int vec16;
};

__global__ void __launch_bounds__(256) block_copy_kernel(BlockCopyArgs a) {
    const int64_t g = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);   // global row = b * rows + r
    const int lane = threadIdx.x & 31;
    if (g >= a.n * a.rows) return;
    const int64_t b = g / a.rows, r = g - b * a.rows;
    const uint8_t *s = a.src + b * a.s_blk + r * a.s_row;
    uint8_t *d = a.dst[b] + r * a.d_row;
    if (a.vec16) {
        for (int64_t o = (int64_t)lane * 16; o < a.row_bytes; o += 32 * 16)
            *reinterpret_cast<uint4 *>(d + o) = *reinterpret_cast<const uint4 *>(s + o);
    } else {
        for (int64_t o = (int64_t)lane * 2; o < a.row_bytes; o += 32 * 2)
            *reinterpret_cast<uint16_t *>(d + o) = *reinterpret_cast<const uint16_t *>(s + o);
    }
}

// ---------------------------------------------------------------------------
// SiLU in fp32, written as F32 or rounded to BF16: y = x / (1 + e^-x).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) silu_kernel(const float *x, void *y, int64_t n, int y_bf16) {
    for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (int64_t)gridDim.x * 256) {
        const float v = x[i];
        const float s = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
        if (y_bf16) static_cast<__nv_bfloat16 *>(y)[i] = __float2bfloat16_rn(s);
        else static_cast<float *>(y)[i] = s;
    }
}

}  // namespace mops
}  // namespace h3

using namespace h3;

namespace {

int elem_bytes(int dtype) { return dtype == H3_BF16 ? 2 : (dtype == H3_F32 ? 4 : 0); }

bool dense_rows_2d(const h3_tensor *t) { return t->ndim == 2 && t->strides[1] == 1 && t->strides[0] >= t->shape[1]; }

}  // namespace

extern "C" int h3_linear_f32(const h3_tensor *y, const h3_tensor *x, const h3_tensor *w, const h3_tensor *bias,
                             void *stream) {
    if (!y) return H3_ERR_NULL;
    if (y->dtype != H3_BF16 && y->dtype != H3_F32) return H3_ERR_BAD_DTYPE;
    H3_CHECK(check_desc(y, y->dtype));
    H3_CHECK(check_desc(w, H3_F32));
    if (!x) return H3_ERR_NULL;
    if (x->dtype != H3_BF16 && x->dtype != H3_F32) return H3_ERR_BAD_DTYPE;
    H3_CHECK(check_desc(x, x->dtype));
    if (x->ndim != 2 || w->ndim != 2 || y->ndim != 2) return H3_ERR_BAD_SHAPE;
    const int64_t M = x->shape[0], K = x->shape[1], N = w->shape[0];
    if (w->shape[1] != K || y->shape[0] != M || y->shape[1] != N) return H3_ERR_BAD_SHAPE;
    if (bias) {
        H3_CHECK(check_desc(bias, H3_F32));
        if (bias->ndim != 1 || bias->shape[0] != N) return H3_ERR_BAD_SHAPE;
        if (bias->strides[0] != 1 && N > 1) return H3_ERR_BAD_LAYOUT;
    }
    if (!dense_rows_2d(x) || !dense_rows_2d(w) || !dense_rows_2d(y)) return H3_ERR_BAD_LAYOUT;
    if (M == 0 || N == 0) return H3_OK;
    if (M / mops::LT >= 65535) return H3_ERR_UNSUPPORTED;
    mops::LinArgs a{x->data, static_cast<const float *>(w->data), bias ? static_cast<const float *>(bias->data) : nullptr,
                    y->data, M, N, K, x->strides[0], w->strides[0], y->strides[0],
                    x->dtype == H3_BF16, y->dtype == H3_BF16};
    if (M <= mops::GEMV_ROWS) {
        if ((N + 7) / 8 > 0x7fffffff) return H3_ERR_UNSUPPORTED;
        mops::linear_f32_gemv_kernel<<<(unsigned)((N + 7) / 8), 256, 0, (cudaStream_t)stream>>>(a);
        return launch_status();
    }
    const dim3 grid((unsigned)((N + mops::LT - 1) / mops::LT), (unsigned)((M + mops::LT - 1) / mops::LT));
    mops::linear_f32_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(a);
    return launch_status();
}

extern "C" int h3_adaln_projection(const h3_tensor *y, const h3_tensor *x, const h3_tensor *w,
                                   const h3_tensor *bias, void *stream) {
    H3_CHECK(check_desc(y, H3_BF16));
    H3_CHECK(check_desc(x, H3_BF16));
    H3_CHECK(check_desc(w, H3_BF16));
    if (x->ndim != 2 || w->ndim != 2 || y->ndim != 2) return H3_ERR_BAD_SHAPE;
    const int64_t M = x->shape[0], K = x->shape[1], N = w->shape[0];
    if (w->shape[1] != K || y->shape[0] != M || y->shape[1] != N) return H3_ERR_BAD_SHAPE;
    if (M > mops::ADALN_ROWS) return H3_ERR_UNSUPPORTED;
    if (bias) {
        H3_CHECK(check_desc(bias, H3_BF16));
        if (bias->ndim != 1 || bias->shape[0] != N) return H3_ERR_BAD_SHAPE;
        if (bias->strides[0] != 1 && N > 1) return H3_ERR_BAD_LAYOUT;
    }
    if (!dense_rows_2d(x) || !dense_rows_2d(w) || !dense_rows_2d(y)) return H3_ERR_BAD_LAYOUT;
    // 16-byte chunks of every weight and input row
    if (K % 8 != 0 || !aligned16(x->data) || !aligned16(w->data)) return H3_ERR_BAD_LAYOUT;
    if ((M > 1 && x->strides[0] % 8 != 0) || (N > 1 && w->strides[0] % 8 != 0)) return H3_ERR_BAD_LAYOUT;
    if (M == 0 || N == 0) return H3_OK;
    if ((N + 7) / 8 > 0x7fffffff) return H3_ERR_UNSUPPORTED;
    mops::AdaArgs a{static_cast<const __nv_bfloat16 *>(x->data), static_cast<const __nv_bfloat16 *>(w->data),
                    bias ? static_cast<const __nv_bfloat16 *>(bias->data) : nullptr,
                    static_cast<__nv_bfloat16 *>(y->data), M, N, K,
                    M > 1 ? x->strides[0] : K, N > 1 ? w->strides[0] : K, M > 1 ? y->strides[0] : N};
    mops::adaln_projection_kernel<<<(unsigned)((N + 7) / 8), 256, 0, (cudaStream_t)stream>>>(a);
    return launch_status();
}

namespace {

int row_move(const h3_tensor *dst, const h3_tensor *src, const h3_tensor *indices, bool scatter, void *stream) {
    if (!dst || !src || !indices) return H3_ERR_NULL;
    const int eb = elem_bytes(src->dtype);
    if (eb == 0 || dst->dtype != src->dtype) return H3_ERR_BAD_DTYPE;
    H3_CHECK(check_desc(src, src->dtype));
    H3_CHECK(check_desc(dst, dst->dtype));
    H3_CHECK(check_desc(indices, H3_I64));
    if (src->ndim != 2 || dst->ndim != 2 || indices->ndim != 1) return H3_ERR_BAD_SHAPE;
    if (src->shape[1] != dst->shape[1]) return H3_ERR_BAD_SHAPE;
    const int64_t n = indices->shape[0];
    // gather: dst [n, C] from src rows; scatter: src [n, C] into dst rows
    if ((scatter ? src->shape[0] : dst->shape[0]) != n) return H3_ERR_BAD_SHAPE;
    if (!dense_rows_2d(src) || !dense_rows_2d(dst)) return H3_ERR_BAD_LAYOUT;
    if (indices->strides[0] != 1 && n > 1) return H3_ERR_BAD_LAYOUT;
    if (n == 0 || src->shape[1] == 0) return H3_OK;
    mops::RowMoveArgs a;
    a.src = static_cast<const uint8_t *>(src->data);
    a.dst = static_cast<uint8_t *>(dst->data);
    a.idx = static_cast<const int64_t *>(indices->data);
    a.rows = n;
    a.limit = scatter ? dst->shape[0] : src->shape[0];
    a.row_bytes = src->shape[1] * eb;
    a.s_src = src->strides[0] * eb;
    a.s_dst = dst->strides[0] * eb;
    a.scatter = scatter ? 1 : 0;
    a.vec16 = (a.row_bytes % 16 == 0 && a.s_src % 16 == 0 && a.s_dst % 16 == 0 && aligned16(src->data) &&
               aligned16(dst->data))
                  ? 1
                  : 0;
    const int64_t blocks = (n + 7) / 8;
    if (blocks > 0x7fffffff) return H3_ERR_UNSUPPORTED;
    mops::row_move_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(a);
    return launch_status();
}

}  // namespace

extern "C" int h3_gather_rows(const h3_tensor *out, const h3_tensor *table, const h3_tensor *indices, void *stream) {
    return row_move(out, table, indices, false, stream);
}

extern "C" int h3_index_copy_rows(const h3_tensor *out, const h3_tensor *indices, const h3_tensor *src,
                                  void *stream) {
    return row_move(out, src, indices, true, stream);
}

extern "C" int h3_copy_blocks(const h3_tensor *dsts, int32_t n, const h3_tensor *src, void *stream) {
    if (!dsts || !src) return H3_ERR_NULL;
    const int eb = elem_bytes(src->dtype);
    if (eb == 0) return H3_ERR_BAD_DTYPE;
    H3_CHECK(check_desc(src, src->dtype));
    if (n < 1 || n > H3_EXCHANGE_MAX_RANKS) return H3_ERR_BAD_SHAPE;
    if (src->ndim != 3 || src->shape[0] != n) return H3_ERR_BAD_SHAPE;
    if (src->strides[2] != 1 && src->shape[2] > 1) return H3_ERR_BAD_LAYOUT;
    const int64_t rows = src->shape[1], C = src->shape[2];
    mops::BlockCopyArgs a;
    for (int i = 0; i < H3_EXCHANGE_MAX_RANKS; ++i) a.dst[i] = nullptr;
    bool aligned = aligned16(src->data);
    for (int i = 0; i < n; ++i) {
        const h3_tensor *d = &dsts[i];
        if (d->dtype != src->dtype) return H3_ERR_BAD_DTYPE;
        H3_CHECK(check_desc(d, d->dtype));
        if (d->ndim != 2 || d->shape[0] != rows || d->shape[1] != C) return H3_ERR_BAD_SHAPE;
        if (!dense_rows_2d(d) || d->strides[0] != dsts[0].strides[0]) return H3_ERR_BAD_LAYOUT;
        a.dst[i] = static_cast<uint8_t *>(d->data);
        aligned = aligned && aligned16(d->data);
    }
    if (rows == 0 || C == 0) return H3_OK;
    a.src = static_cast<const uint8_t *>(src->data);
    a.n = n;
    a.rows = rows;
    a.row_bytes = C * eb;
    a.s_blk = src->strides[0] * eb;
    a.s_row = src->strides[1] * eb;
    a.d_row = dsts[0].strides[0] * eb;
    a.vec16 = (aligned && a.row_bytes % 16 == 0 && a.s_blk % 16 == 0 && a.s_row % 16 == 0 && a.d_row % 16 == 0) ? 1 : 0;
    const int64_t blocks = (n * rows + 7) / 8;
    if (blocks > 0x7fffffff) return H3_ERR_UNSUPPORTED;
    mops::block_copy_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(a);
    return launch_status();
}

extern "C" int h3_silu(const h3_tensor *y, const h3_tensor *x, void *stream) {
    H3_CHECK(check_desc(x, H3_F32));
    if (!y) return H3_ERR_NULL;
    if (y->dtype != H3_F32 && y->dtype != H3_BF16) return H3_ERR_BAD_DTYPE;
    H3_CHECK(check_desc(y, y->dtype));
    H3_CHECK(check_same_shape(y, x));
    // contiguous only (the op runs on small fp32 vectors such as temb)
    int64_t expect = 1;
    for (int i = x->ndim - 1; i >= 0; --i) {
        if (x->shape[i] > 1 && (x->strides[i] != expect || y->strides[i] != expect)) return H3_ERR_BAD_LAYOUT;
        expect *= x->shape[i];
    }
    const int64_t n = numel(x);
    if (n == 0) return H3_OK;
    const int64_t blocks = (n + 255) / 256;
    mops::silu_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, (cudaStream_t)stream>>>(
        static_cast<const float *>(x->data), y->data, n, y->dtype == H3_BF16);
    return launch_status();
}

// device error word of this translation unit (index checks of the row moves)
extern "C" unsigned int h3_model_ops_device_error_read_and_clear(void) {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, h3::g_h3_device_error, sizeof(v));
    cudaMemcpyToSymbol(h3::g_h3_device_error, &zero, sizeof(zero));
    return v;
}
