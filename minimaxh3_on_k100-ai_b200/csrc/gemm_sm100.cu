// BF16 projections of the H3 DiT block on tcgen05 / TMEM, fed by TMA (sm_100a),
// with the block's pointwise ops fused into the epilogue.
//
//   y = x W^T                                       (QKV, out-proj; reference linear,
//                                                     patches/InfiniCore.patch:1231-1292)
//   y = swiglu(x Wup^T, x Wgate^T)                   (gate_up + h3_swiglu,
//                                                     patches/InfiniLM.patch:1172-1179)
//   y = bf16(res + bf16(gate * bf16(x W^T)))         (down-proj + h3_gated_residual,
//                                                     patches/InfiniLM.patch:1391-1394)
//   q, k, v = x Wqkv^T with q/k RMSNorm + RoPE        (QKV projection + h3_qk_norm_rope_,
//             stored per head into destination         patches/InfiniLM.patch:744-839, and the
//             buffers (local, or a peer's receive      Ulysses send of gather_sequence :895-910)
//             buffer over NVLink)
// The epilogues round the accumulator to BF16 first, exactly where the unfused
// reference materialises the linear's BF16 output, then apply the pointwise op
// with its staged rounding, so fused == unfused bit for bit.
//
// Persistent kernel, one CTA per SM, 128x256 output tiles, K in steps of 64
// (one 128-byte swizzle span) through a 4-slot TMA ring.  Warp 0 loads (TMA, no
// multicast), warp 1 issues tcgen05.mma (M=128, N=256, K=16) into one of two
// TMEM accumulators (2 x 256 columns), warps 4..7 drain the other accumulator
// (tcgen05.ld, one output row per thread) while the next tile accumulates.
// Tiles are rasterised in column groups of 8: the 148 tiles in flight then span
// ~18 row tiles x 8 column tiles, whose A rows and W rows (~24 + 21 MB at K = 5120)
// are the smallest working set per wave on 148 SMs; measured on B200 at config 3,
// groups of 8 / 16 / 32 / 64 ran the four projections at 1291 / 1268 / 1150 /
// 1024 TFLOP/s.
#include <math.h>
#include <stdint.h>

#include "h3_abi_util.h"
#include "h3_common.cuh"
#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace h3 {
namespace gemm {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int THREADS = 256;
constexpr uint32_t TMEM_COLS = 512;
#ifndef H3_GEMM_GROUP_N
#define H3_GEMM_GROUP_N 8
#endif
constexpr int GROUP_N = H3_GEMM_GROUP_N;   // column tiles per raster group
// EPI_QKV stages each epilogue warp's 32 head rows (8 KB) in shared memory, so that
// the stores to the destination (often a peer's receive buffer over NVLink) go out
// as whole 256-byte rows, 16 lanes per row, instead of 16-byte pieces of 32 rows
constexpr int QKV_STAGE_WARP = 32 * 256;

// Shared-memory layout of one CTA.  PAIR: a CTA pair (cluster of 2, tcgen05
// cta_group::2) owns a 256 x 256 output tile; each CTA loads its own 128 A rows
// and half (128) of the tile's 256 W rows per K step -- 32 KB instead of 48 KB
// per CTA, which leaves room for 6 ring slots (H3_GEMM_PAIR_STAGES without the QKV
// epilogue's staging rows; 7 measured the same) -- and keeps its 128 output rows in
// its own TMEM.
#ifndef H3_GEMM_PAIR_STAGES
#define H3_GEMM_PAIR_STAGES 6
#endif
template <bool PAIR, bool QKV = false>
struct Cfg {
    static constexpr int STAGES = PAIR ? (QKV ? 6 : H3_GEMM_PAIR_STAGES) : 4;
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;   // W rows this CTA loads per K step
    static constexpr int STAGE_BYTES = A_BYTES + B_ROWS * BK * 2;
    static constexpr int ROWS = PAIR ? 2 * BM : BM;     // output rows per tile
    static constexpr int OFF_BAR = STAGES * STAGE_BYTES;
    static constexpr int NUM_BARS = 2 * STAGES + 4;
    static constexpr int SMEM = OFF_BAR + NUM_BARS * 8 + 16 + 1024;
    static constexpr int OFF_QKV_STAGE = (OFF_BAR + NUM_BARS * 8 + 16 + 127) / 128 * 128;
    static constexpr int SMEM_QKV = OFF_QKV_STAGE + 4 * QKV_STAGE_WARP + 1024;
    static_assert((QKV ? SMEM_QKV : SMEM) <= 232448, "shared memory over the sm_100 per-block limit");
};
__host__ __device__ constexpr bool is_qkv(int epi) { return epi == 3 || epi == 5; }
template <bool PAIR>
__host__ __device__ constexpr int smem_bytes(int epi) {
    return is_qkv(epi) ? Cfg<PAIR, true>::SMEM_QKV : Cfg<PAIR, false>::SMEM;
}

// EPI_GATED_RES_SQ: EPI_GATED_RES, plus the tile's share of the output row's sum
// of squares for the RMSNorm that follows (sq[row][n] = fp32 sum over the tile's
// columns, in column order, of bf16(out^2)), so the norm pass needs no reduction.
// EPI_QKV64: EPI_QKV for 64 rotated pairs (the full-D 44/42/42 RoPE layout).
enum Epi { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_GATED_RES = 2, EPI_QKV = 3, EPI_GATED_RES_SQ = 4, EPI_QKV64 = 5 };
constexpr int QKV_HALF = 48;              // rotated pairs per head (3 axes x 16 frequencies)

struct Params {
    int M, N, K;            // N: accumulator columns (weight rows)
    int num_m, num_n, num_tiles;
    __nv_bfloat16 *out;
    int64_t ldo;
    const __nv_bfloat16 *res;
    int64_t ldr;
    const __nv_bfloat16 *gate;
    int64_t ldg;            // 0 broadcasts one gate row
    float *sq;              // EPI_GATED_RES_SQ: [M, ceil(N / BN)] fp32 partial sums of squares
    int64_t ldsq;
    // gated residual with per-segment gate rows (nseg > 0): rows [seg_end[s-1], seg_end[s])
    // use the gate row gates[s] (one modulation row per segment, as the block applies them)
    int nseg;
    int seg_end[H3_MAX_SEGMENTS];
    const __nv_bfloat16 *gates[H3_MAX_SEGMENTS];
    // EPI_QKV: accumulator column c = part * hcols + head * 128 + d (part 0/1/2 = q/k/v);
    // head h goes to destination h / hpd, head slot h % hpd
    int hcols, hpd;
    __nv_bfloat16 *dst[3][H3_EXCHANGE_MAX_RANKS];
    int64_t drow, dhead;    // destination strides: token, head (elements)
    const __nv_bfloat16 *norm_q, *norm_k;
    const __nv_bfloat16 *cos, *sin;
    int64_t cs0, ss0;
    float eps;
};

__device__ __forceinline__ void tile_coords(const Params &p, int tile, int &m, int &n) {
    const int span = GROUP_N * p.num_m;
    const int g = tile / span;
    const int r = tile - g * span;
    const int n0 = g * GROUP_N;
    const int gw = min(GROUP_N, p.num_n - n0);
    m = r / gw;
    n = n0 + (r - m * gw);
}

__device__ __forceinline__ void st_global_v4(void *ptr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

template <int EPI, bool PAIR>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, Params p) {
    using C = Cfg<PAIR, is_qkv(EPI)>;
    constexpr int STAGES = C::STAGES;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::OFF_BAR);
    uint64_t *full = bars;
    uint64_t *empty = bars + STAGES;
    uint64_t *acc_full = bars + 2 * STAGES;
    uint64_t *acc_empty = acc_full + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + C::NUM_BARS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kblocks = p.K / BK;
    // PAIR: CTA `rank` of the pair; tiles are dealt to pairs.  The leader (rank 0)
    // holds the ring's full barriers (both CTAs' TMA bytes count there) and the
    // accumulator-empty barriers (both CTAs' epilogue warps arrive there) and
    // issues the MMAs; each CTA's empty and accumulator-full barriers get the
    // leader's commits.
    const uint32_t rank = PAIR ? cluster_ctarank() : 0;
    const int first_tile = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int tile_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&acc_full[a], 1);
            mbar_init(&acc_empty[a], PAIR ? 8 : 128);   // PAIR: one arrival per epilogue warp of the pair
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        if (PAIR) {
            tmem_alloc_pair(tmem_slot, TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    if (PAIR) cluster_sync();   // the peer's barriers are initialised before any remote arrive
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&ta);
            tma_prefetch_desc(&tb);
            uint32_t it = 0;
            bool ok = true;
            for (int tile = first_tile; tile < p.num_tiles && ok; tile += tile_step) {
                int m, n;
                tile_coords(p, tile, m, n);
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const uint32_t slot = it % STAGES, use = it / STAGES;
                    ok = mbar_wait(&empty[slot], (use & 1) ^ 1, abort_flag);
                    if (!ok) break;
                    uint8_t *sa = smem + slot * C::STAGE_BYTES;
                    if (PAIR) {
                        // both CTAs' bytes complete the leader's barrier, whose arrival
                        // (with the pair's byte count) the leader makes
                        const uint32_t fb = mapa_shared(&full[slot], 0);
                        if (rank == 0) mbar_expect_tx(&full[slot], 2 * C::STAGE_BYTES);
                        tma_load_2d_pair(sa, &ta, fb, kb * BK, m * C::ROWS + (int)rank * BM);
                        tma_load_2d_pair(sa + A_BYTES, &tb, fb, kb * BK, n * BN + (int)rank * C::B_ROWS);
                    } else {
                        mbar_expect_tx(&full[slot], C::STAGE_BYTES);
                        tma_load_2d(sa, &ta, &full[slot], kb * BK, m * BM);
                        tma_load_2d(sa + A_BYTES, &tb, &full[slot], kb * BK, n * BN);
                    }
                }
            }
            // the leader's last commits arrive on this CTA's empty barriers: wait for
            // them, so that none lands after the CTA has exited
            for (uint32_t i = 0; i < STAGES && ok; ++i) {
                if (it < i + 1) break;
                const uint32_t u = it - 1 - i;
                ok = mbar_wait(&empty[u % STAGES], (u / STAGES) & 1, abort_flag);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t IDESC = idesc_bf16_f32(C::ROWS, BN, false);
            const uint32_t base = smem_u32(smem);
            uint32_t it = 0, lt = 0;
            bool ok = true;
            for (int tile = first_tile; tile < p.num_tiles && ok; tile += tile_step, ++lt) {
                const uint32_t acc = lt & 1, use = lt >> 1;
                ok = PAIR ? mbar_wait_cluster(&acc_empty[acc], (use & 1) ^ 1, abort_flag)
                          : mbar_wait(&acc_empty[acc], (use & 1) ^ 1, abort_flag);
                if (!ok) break;
                tc_fence_after();
                const uint32_t d = tmem + acc * BN;
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const uint32_t slot = it % STAGES;
                    ok = mbar_wait(&full[slot], (it / STAGES) & 1, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t sa = base + slot * C::STAGE_BYTES, sb = sa + A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t da = smem_desc_sw128(sa + kk * 32, 16, 1024);
                        const uint64_t db = smem_desc_sw128(sb + kk * 32, 16, 1024);
                        if (PAIR) umma_ss_pair(d, da, db, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
                        else umma_ss(d, da, db, IDESC, (kb > 0 || kk > 0) ? 1u : 0u);
                    }
                    if (PAIR) {
                        umma_commit_pair(smem_u32(&empty[slot]));
                        umma_commit_pair(mapa_shared(&empty[slot], 1));
                    } else {
                        umma_commit(&empty[slot]);
                    }
                }
                if (!ok) break;
                if (PAIR) {
                    umma_commit_pair(smem_u32(&acc_full[acc]));
                    umma_commit_pair(mapa_shared(&acc_full[acc], 1));
                } else {
                    umma_commit(&acc_full[acc]);
                }
            }
            if (!ok) drain_in_flight();
        }
    } else if (warp >= 4) {
        const int wq = warp & 3;
        const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
        uint32_t lt = 0;
        bool ok = true;
        for (int tile = first_tile; tile < p.num_tiles; tile += tile_step, ++lt) {
            int m, n;
            tile_coords(p, tile, m, n);
            const uint32_t acc = lt & 1;
            ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[acc], (lt >> 1) & 1, abort_flag));
            if (!ok) break;
            tc_fence_after();
            const uint32_t tbase = tmem + acc * BN + lane_off;
            const int row0 = m * C::ROWS + (int)rank * BM;   // this CTA's first output row
            const int row = row0 + wq * 32 + lane;
            const bool row_ok = row < p.M;
            if (EPI == EPI_QKV || EPI == EPI_QKV64) {
                // the tile's 256 columns are two heads of one part; this thread owns one token
                constexpr int HW = (EPI == EPI_QKV64 ? 64 : QKV_HALF) / 2;   // rotated pairs as BF16x2 words
                uint32_t cw[HW], sw[HW];
                if (row_ok) {
#pragma unroll
                    for (int q = 0; q < HW / 4; ++q) {
                        const uint4 c4 = *reinterpret_cast<const uint4 *>(p.cos + (int64_t)row * p.cs0 + 8 * q);
                        const uint4 s4 = *reinterpret_cast<const uint4 *>(p.sin + (int64_t)row * p.ss0 + 8 * q);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            cw[4 * q + e] = w32(c4, e);
                            sw[4 * q + e] = w32(s4, e);
                        }
                    }
                }
#pragma unroll 1
                for (int hh = 0; hh < 2; ++hh) {
                    const int col = n * BN + hh * 128;
                    const int part = col / p.hcols;
                    const int head = (col - part * p.hcols) >> 7;
                    const int dp = head / p.hpd, hloc = head - dp * p.hpd;
                    uint32_t xw[64];
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        uint32_t v[32];
                        tmem_ld32(tbase + hh * 128 + cc * 32, v);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 16; ++i)   // the linear's BF16 output
                            xw[16 * cc + i] = pack2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
                    }
                    if (row_ok && part < 2) {
                        // RMSNorm over the head with the exact summation tree of the q/k
                        // kernel (16 partial sums of 8 columns, then a xor-8/4/2/1 tree)
                        float s16[16];
#pragma unroll
                        for (int l = 0; l < 16; ++l) {
                            float sacc = 0.f;
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const uint32_t sq = bmul2(xw[4 * l + i], xw[4 * l + i]);
                                sacc = add_rn(sacc, blo(sq));
                                sacc = add_rn(sacc, bhi(sq));
                            }
                            s16[l] = sacc;
                        }
#pragma unroll
                        for (int o = 8; o > 0; o >>= 1)
#pragma unroll
                            for (int l = 0; l < o; ++l) s16[l] = add_rn(s16[l], s16[l + o]);
                        const float mean = bf(__fmul_rn(s16[0], 0.0078125f));
                        const float var = bf(add_rn(mean, p.eps));
                        const uint32_t r2 = bsplat(bf(rsqrt_torch(var)));
                        const __nv_bfloat16 *nw = part == 0 ? p.norm_q : p.norm_k;
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            const uint4 w4 = *reinterpret_cast<const uint4 *>(nw + 8 * q);
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                xw[4 * q + e] = bmul2(bmul2(xw[4 * q + e], r2), w32(w4, e));  // bf(bf(x*r)*w)
                        }
                        // RoPE: y0 = bf(bf(a*c) + bf(-b*s)), y1 = bf(bf(b*c) + bf(a*s))
#pragma unroll
                        for (int j = 0; j < HW; ++j) {
                            const uint32_t a = xw[j], b = xw[j + HW];
                            xw[j] = badd2(bmul2(a, cw[j]), bmul2(bneg2(b), sw[j]));
                            xw[j + HW] = badd2(bmul2(b, cw[j]), bmul2(a, sw[j]));
                        }
                    }
                    // this lane's row into the warp's staging rows (16-byte chunk c of row r at
                    // chunk c ^ (r & 7): each 8-lane phase of a store or load hits 8 distinct
                    // bank groups), then whole rows out: store q covers rows 2q and 2q + 1 of
                    // the warp, 16 lanes (256 contiguous bytes) per row
                    const uint32_t stage = smem_u32(smem + C::OFF_QKV_STAGE + wq * QKV_STAGE_WARP);
                    if (row_ok) {
#pragma unroll
                        for (int q = 0; q < 16; ++q)
                            st_shared_v4(stage + lane * 256 + ((q ^ (lane & 7)) << 4), xw[4 * q], xw[4 * q + 1],
                                         xw[4 * q + 2], xw[4 * q + 3]);
                    }
                    __syncwarp();
                    const int c = lane & 15;
#pragma unroll 4
                    for (int q = 0; q < 16; ++q) {
                        const int r = 2 * q + (lane >> 4);
                        const int grow = row0 + wq * 32 + r;
                        if (grow < p.M) {
                            const uint4 v = ld_shared_v4(stage + r * 256 + ((c ^ (r & 7)) << 4));
                            st_global_v4(p.dst[part][dp] + (int64_t)grow * p.drow + (int64_t)hloc * p.dhead + 8 * c,
                                         v.x, v.y, v.z, v.w);
                        }
                    }
                    __syncwarp();   // the staging rows are rewritten by the next head
                }
            } else if (EPI == EPI_SWIGLU) {
                // accumulator columns [0,128) = up, [128,256) = gate of features n*128 + c
#pragma unroll 1
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t u[32], g[32];
                    tmem_ld32(tbase + cc * 32, u);
                    tmem_ld32(tbase + 128 + cc * 32, g);
                    tmem_ld_wait();
                    const int col = n * 128 + cc * 32;
                    if (row_ok) {
                        uint32_t w[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            // the linear's BF16 outputs, then bf16(up * bf16(g / (1 + exp(-g))))
                            const uint32_t up2 = pack2(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1]));
                            const uint32_t g2 = pack2(__uint_as_float(g[2 * i]), __uint_as_float(g[2 * i + 1]));
                            const float g0 = blo(g2), g1 = bhi(g2);
                            const float a0 = __fdiv_rn(g0, add_rn(1.0f, expf(-g0)));
                            const float a1 = __fdiv_rn(g1, add_rn(1.0f, expf(-g1)));
                            w[i] = bmul2(up2, pack2(a0, a1));
                        }
                        __nv_bfloat16 *dst = p.out + (int64_t)row * p.ldo + col;
#pragma unroll
                        for (int q = 0; q < 4; ++q) st_global_v4(dst + 8 * q, w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
                    }
                }
            } else {
                float ssq = 0.f;   // EPI_GATED_RES_SQ: this row's sum of bf16(out^2) over the tile
                // this row's gate row: strided view, or its segment's modulation row
                const __nv_bfloat16 *grow_ptr = p.gate + (int64_t)row * p.ldg;
                if (p.nseg > 0) {
                    int s = 0;
                    while (s + 1 < p.nseg && row >= p.seg_end[s]) ++s;
                    grow_ptr = p.gates[s];
                }
#pragma unroll 1
                for (int cc = 0; cc < BN / 32; ++cc) {
                    uint32_t v[32];
                    tmem_ld32(tbase + cc * 32, v);
                    tmem_ld_wait();
                    const int col = n * BN + cc * 32;
                    if (row_ok && col < p.N) {
                        uint32_t w[16];
                        if (EPI == EPI_STORE) {
#pragma unroll
                            for (int i = 0; i < 16; ++i)
                                w[i] = pack2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
                        } else {  // EPI_GATED_RES, EPI_GATED_RES_SQ
                            const __nv_bfloat16 *rp = p.res + (int64_t)row * p.ldr + col;
                            const __nv_bfloat16 *gp = grow_ptr + col;
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const uint4 r4 = *reinterpret_cast<const uint4 *>(rp + 8 * q);
                                const uint4 g4 = *reinterpret_cast<const uint4 *>(gp + 8 * q);
#pragma unroll
                                for (int e = 0; e < 4; ++e) {   // bf16(res + bf16(gate * bf16(acc)))
                                    const int idx = 8 * q + 2 * e;
                                    const uint32_t y2 = pack2(__uint_as_float(v[idx]), __uint_as_float(v[idx + 1]));
                                    w[4 * q + e] = badd2(w32(r4, e), bmul2(w32(g4, e), y2));
                                }
                            }
                            if (EPI == EPI_GATED_RES_SQ) {
#pragma unroll
                                for (int i = 0; i < 16; ++i) {   // columns in order: lo, hi of each word
                                    const uint32_t sq = bmul2(w[i], w[i]);
                                    ssq = add_rn(ssq, blo(sq));
                                    ssq = add_rn(ssq, bhi(sq));
                                }
                            }
                        }
                        __nv_bfloat16 *dst = p.out + (int64_t)row * p.ldo + col;
#pragma unroll
                        for (int q = 0; q < 4; ++q) st_global_v4(dst + 8 * q, w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
                    }
                }
                if (EPI == EPI_GATED_RES_SQ && row_ok) p.sq[(int64_t)row * p.ldsq + n] = ssq;
            }
            tc_fence_before();
            if (PAIR) {
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));
            } else {
                mbar_arrive(&acc_empty[acc]);
            }
        }
        if (!ok) drain_in_flight();
    }

    __syncwarp();
    tc_fence_before();
    if (PAIR) cluster_sync();   // neither CTA leaves while the pair's MMAs or arrivals may touch it
    else __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        if (PAIR) tmem_dealloc_pair(tmem, TMEM_COLS);
        else tmem_dealloc(tmem, TMEM_COLS);
    }
}

// dst rows = 128-row blocks [up_0 | gate_0 | up_1 | gate_1 | ...] of src = [up; gate]
__global__ void pack_gate_up_kernel(__nv_bfloat16 *dst, int64_t lddst, const __nv_bfloat16 *src, int64_t ldsrc,
                                    int64_t F, int64_t K) {
    const int64_t vpr = K / 8;
    const int64_t total = 2 * F * vpr;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = idx / vpr, c = (idx - r * vpr) * 8;
        const int64_t blk = r / 256, within = r - blk * 256;
        const int64_t s = within < 128 ? blk * 128 + within : F + blk * 128 + (within - 128);
        *reinterpret_cast<uint4 *>(dst + r * lddst + c) = *reinterpret_cast<const uint4 *>(src + s * ldsrc + c);
    }
}

}  // namespace gemm
}  // namespace h3

using namespace h3;

namespace {

int check_matrix(const h3_tensor *t) {
    H3_CHECK(check_bf16(t));
    if (t->ndim != 2) return H3_ERR_BAD_SHAPE;
    if (t->strides[1] != 1 || !aligned16(t->data)) return H3_ERR_BAD_LAYOUT;
    if (t->shape[0] > 1 && (t->strides[0] % 8 != 0 || t->strides[0] < t->shape[1])) return H3_ERR_BAD_LAYOUT;
    return H3_OK;
}

int mat_tmap(CUtensorMap *map, const h3_tensor *t, uint32_t box_rows) {
    const cuuint64_t dims[2] = {(cuuint64_t)t->shape[1], (cuuint64_t)t->shape[0]};
    const int64_t ld = t->shape[0] > 1 ? t->strides[0] : ((t->shape[1] + 7) / 8) * 8;
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {gemm::BK, box_rows};
    return make_tmap_bf16(map, t->data, 2, dims, strides, box);
}

// Which tile form the projections use: 0 chooses per launch, 1 forces single-CTA
// 128-row tiles, 2 forces CTA-pair 256-row tiles (h3_gemm_variant).
std::atomic<int> g_gemm_variant{0};

// The pair form halves each SM's W traffic but pads M to 256 rows: chosen unless
// that pads more rows than the single form by over 1/64 of the product.
bool use_pair(int M) {
    const int v = g_gemm_variant.load();
    if (v == 1) return false;
    if (v == 2) return true;
    const int64_t pad2 = (int64_t)(M + 255) / 256 * 256, pad1 = (int64_t)(M + 127) / 128 * 128;
    return pad2 * 64 <= pad1 * 65;
}

template <int EPI, bool PAIR>
int launch_form(const CUtensorMap &ta, const CUtensorMap &tb, gemm::Params &p, cudaStream_t stream) {
    using C = gemm::Cfg<PAIR>;
    constexpr int smem = gemm::smem_bytes<PAIR>(EPI);
    auto kernel = gemm::gemm_kernel<EPI, PAIR>;
    p.num_m = (p.M + C::ROWS - 1) / C::ROWS;
    p.num_n = (p.N + gemm::BN - 1) / gemm::BN;
    p.num_tiles = p.num_m * p.num_n;
    // per device: 0 = not set up yet, else 1 + the number of CTAs (single) or
    // CTA pairs (PAIR) that are resident at once
    static std::atomic<int> resident[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return H3_ERR_UNSUPPORTED;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(gemm::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = PAIR ? attr : nullptr;
    cfg.numAttrs = PAIR ? 1 : 0;
    if (resident[dev].load() == 0) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
            return H3_ERR_LAUNCH;
        int n = num_sms();
        if (PAIR) {
            cfg.gridDim = dim3(2 * (n / 2));
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess || clusters < 1)
                return H3_ERR_LAUNCH;
            n = clusters;
        }
        resident[dev].store(1 + n);
    }
    const int slots = resident[dev].load() - 1;
    const int units = p.num_tiles < slots ? p.num_tiles : slots;
    cfg.gridDim = dim3(PAIR ? 2 * units : units);
    if (cudaLaunchKernelEx(&cfg, kernel, ta, tb, p) != cudaSuccess) return H3_ERR_LAUNCH;
    return launch_status();
}

template <int EPI>
int launch_gemm(const h3_tensor *x, const h3_tensor *w, gemm::Params &p, cudaStream_t stream) {
    // an empty product launches nothing (a tensor map cannot describe a zero extent)
    if (p.M == 0 || p.N == 0) return H3_OK;
    const bool pair = use_pair(p.M);
    CUtensorMap ta, tb;
    H3_CHECK(mat_tmap(&ta, x, gemm::BM));
    H3_CHECK(mat_tmap(&tb, w, pair ? gemm::Cfg<true>::B_ROWS : gemm::Cfg<false>::B_ROWS));
    return pair ? launch_form<EPI, true>(ta, tb, p, stream) : launch_form<EPI, false>(ta, tb, p, stream);
}

int check_gemm_operands(const h3_tensor *y, const h3_tensor *x, const h3_tensor *w) {
    H3_CHECK(check_matrix(y));
    H3_CHECK(check_matrix(x));
    H3_CHECK(check_matrix(w));
    if (x->shape[1] != w->shape[1]) return H3_ERR_BAD_SHAPE;
    if (x->shape[1] % gemm::BK != 0 || x->shape[1] == 0) return H3_ERR_UNSUPPORTED;
    if (x->shape[0] > 0x7fffffffLL || w->shape[0] > 0x7fffffffLL) return H3_ERR_UNSUPPORTED;
    return H3_OK;
}

}  // namespace

extern "C" int h3_linear(const h3_tensor *y, const h3_tensor *x, const h3_tensor *w, void *stream) {
    H3_CHECK(check_gemm_operands(y, x, w));
    if (y->shape[0] != x->shape[0] || y->shape[1] != w->shape[0]) return H3_ERR_BAD_SHAPE;
    if (y->shape[1] % 32 != 0) return H3_ERR_UNSUPPORTED;
    gemm::Params p{};
    p.M = (int)x->shape[0];
    p.N = (int)w->shape[0];
    p.K = (int)x->shape[1];
    p.out = static_cast<__nv_bfloat16 *>(y->data);
    p.ldo = y->strides[0];
    return launch_gemm<gemm::EPI_STORE>(x, w, p, (cudaStream_t)stream);
}

extern "C" int h3_linear_swiglu(const h3_tensor *y, const h3_tensor *x, const h3_tensor *w_packed, void *stream) {
    H3_CHECK(check_gemm_operands(y, x, w_packed));
    const int64_t F = w_packed->shape[0] / 2;
    if (w_packed->shape[0] % 256 != 0) return H3_ERR_BAD_SHAPE;
    if (y->shape[0] != x->shape[0] || y->shape[1] != F) return H3_ERR_BAD_SHAPE;
    gemm::Params p{};
    p.M = (int)x->shape[0];
    p.N = (int)w_packed->shape[0];
    p.K = (int)x->shape[1];
    p.out = static_cast<__nv_bfloat16 *>(y->data);
    p.ldo = y->strides[0];
    return launch_gemm<gemm::EPI_SWIGLU>(x, w_packed, p, (cudaStream_t)stream);
}

namespace {

// out = bf16(residual + bf16(gate * bf16(x w^T))); with sq, also the per-tile
// partial sums of squares of out (EPI_GATED_RES_SQ)
int gated_residual_gemm(const h3_tensor *out, const h3_tensor *x, const h3_tensor *w, const h3_tensor *residual,
                        const h3_tensor *gate, const h3_tensor *sq, cudaStream_t stream,
                        const h3_tensor *gates = nullptr, const int64_t *seg_rows = nullptr, int nseg = 0) {
    H3_CHECK(check_gemm_operands(out, x, w));
    H3_CHECK(check_bf16(residual));
    if (out->shape[0] != x->shape[0] || out->shape[1] != w->shape[0]) return H3_ERR_BAD_SHAPE;
    H3_CHECK(check_same_shape(residual, out));
    if (out->shape[1] % 32 != 0) return H3_ERR_UNSUPPORTED;
    if (residual->strides[1] != 1 || !aligned16(residual->data) || residual->strides[0] % 8 != 0)
        return H3_ERR_BAD_LAYOUT;
    gemm::Params p{};
    p.M = (int)x->shape[0];
    p.N = (int)w->shape[0];
    p.K = (int)x->shape[1];
    if (nseg > 0) {
        // one contiguous gate row [N] per segment of consecutive rows
        if (!gates || !seg_rows) return H3_ERR_NULL;
        if (nseg > H3_MAX_SEGMENTS) return H3_ERR_UNSUPPORTED;
        int64_t end = 0;
        for (int i = 0; i < nseg; ++i) {
            H3_CHECK(check_bf16(&gates[i]));
            if (gates[i].ndim != 1 || gates[i].shape[0] != out->shape[1]) return H3_ERR_BAD_SHAPE;
            if ((out->shape[1] > 1 && gates[i].strides[0] != 1) || !aligned16(gates[i].data)) return H3_ERR_BAD_LAYOUT;
            if (seg_rows[i] < 0) return H3_ERR_BAD_SHAPE;
            end += seg_rows[i];
            p.seg_end[i] = (int)end;
            p.gates[i] = static_cast<const __nv_bfloat16 *>(gates[i].data);
        }
        if (end != out->shape[0]) return H3_ERR_BAD_SHAPE;
        p.nseg = nseg;
        p.gate = p.gates[0];
        p.ldg = 0;
    } else {
        H3_CHECK(check_bf16(gate));
        H3_CHECK(check_same_shape(gate, out));
        if (gate->strides[1] != 1 || !aligned16(gate->data) || gate->strides[0] % 8 != 0) return H3_ERR_BAD_LAYOUT;
        p.gate = static_cast<const __nv_bfloat16 *>(gate->data);
        p.ldg = gate->strides[0];
    }
    p.out = static_cast<__nv_bfloat16 *>(out->data);
    p.ldo = out->strides[0];
    p.res = static_cast<const __nv_bfloat16 *>(residual->data);
    p.ldr = residual->strides[0];
    if (!sq) return launch_gemm<gemm::EPI_GATED_RES>(x, w, p, stream);
    H3_CHECK(check_desc(sq, H3_F32));
    const int64_t nt = (out->shape[1] + gemm::BN - 1) / gemm::BN;
    if (sq->ndim != 2 || sq->shape[0] != out->shape[0] || sq->shape[1] != nt) return H3_ERR_BAD_SHAPE;
    if ((nt > 1 && sq->strides[1] != 1) || (sq->shape[0] > 1 && sq->strides[0] < nt)) return H3_ERR_BAD_LAYOUT;
    p.sq = static_cast<float *>(sq->data);
    p.ldsq = sq->strides[0];
    return launch_gemm<gemm::EPI_GATED_RES_SQ>(x, w, p, stream);
}

}  // namespace

extern "C" int h3_linear_gated_residual(const h3_tensor *out, const h3_tensor *x, const h3_tensor *w,
                                        const h3_tensor *residual, const h3_tensor *gate, void *stream) {
    return gated_residual_gemm(out, x, w, residual, gate, nullptr, (cudaStream_t)stream);
}

extern "C" int h3_linear_gated_residual_segmented(const h3_tensor *out, const h3_tensor *sq, const h3_tensor *x,
                                                  const h3_tensor *w, const h3_tensor *residual,
                                                  const h3_tensor *gates, const int64_t *seg_rows, int32_t nseg,
                                                  void *stream) {
    if (nseg < 1) return H3_ERR_BAD_SHAPE;
    return gated_residual_gemm(out, x, w, residual, nullptr, sq, (cudaStream_t)stream, gates, seg_rows, nseg);
}

extern "C" int h3_linear_gated_residual_sq(const h3_tensor *out, const h3_tensor *sq, const h3_tensor *x,
                                           const h3_tensor *w, const h3_tensor *residual, const h3_tensor *gate,
                                           void *stream) {
    if (!sq) return H3_ERR_NULL;
    return gated_residual_gemm(out, x, w, residual, gate, sq, (cudaStream_t)stream);
}

extern "C" int h3_linear_gated_residual_rms_modulate(const h3_tensor *residual_out, const h3_tensor *out,
                                                     const h3_tensor *x, const h3_tensor *w,
                                                     const h3_tensor *residual, const h3_tensor *gate,
                                                     const h3_tensor *weight, const h3_tensor *scale,
                                                     const h3_tensor *shift, float eps, const h3_tensor *workspace,
                                                     void *stream) {
    if (!workspace || !residual_out) return H3_ERR_NULL;
    H3_CHECK(check_bf16(out));
    H3_CHECK(check_same_shape(out, residual_out));
    H3_CHECK(h3_linear_gated_residual_sq(residual_out, workspace, x, w, residual, gate, stream));
    return h3_rms_modulate_sq(out, residual_out, workspace, weight, scale, shift, eps, stream);
}

// QKV projection with q/k RMSNorm + RoPE in the epilogue, each head row stored to
// its destination: q_dsts/k_dsts/v_dsts are arrays of ndst descriptors [T, hpd, 128]
// (same strides), head h of the projection goes to destination h / hpd.
extern "C" int h3_linear_qkv_norm_rope(const h3_tensor *x, const h3_tensor *w, const h3_tensor *q_dsts,
                                       const h3_tensor *k_dsts, const h3_tensor *v_dsts, int32_t ndst,
                                       const h3_tensor *norm_q, const h3_tensor *norm_k, const h3_tensor *cos,
                                       const h3_tensor *sin, float eps, void *stream) {
    if (!q_dsts || !k_dsts || !v_dsts) return H3_ERR_NULL;
    H3_CHECK(check_matrix(x));
    H3_CHECK(check_matrix(w));
    if (x->shape[1] != w->shape[1]) return H3_ERR_BAD_SHAPE;
    if (x->shape[1] % gemm::BK != 0 || x->shape[1] == 0) return H3_ERR_UNSUPPORTED;
    if (x->shape[0] > 0x7fffffffLL || w->shape[0] > 0x7fffffffLL) return H3_ERR_UNSUPPORTED;
    if (ndst < 1 || ndst > H3_EXCHANGE_MAX_RANKS) return H3_ERR_BAD_SHAPE;
    const int64_t T = x->shape[0];
    const h3_tensor *d0 = &q_dsts[0];
    if (d0->ndim != 3 || d0->shape[2] != 128) return H3_ERR_BAD_SHAPE;
    const int64_t hpd = d0->shape[1], H = hpd * ndst;
    if (hpd < 1 || w->shape[0] != 3 * H * 128) return H3_ERR_BAD_SHAPE;
    if ((H * 128) % gemm::BN != 0) return H3_ERR_UNSUPPORTED;   // two heads per tile: H even
    gemm::Params p{};
    const h3_tensor *sets[3] = {q_dsts, k_dsts, v_dsts};
    for (int part = 0; part < 3; ++part) {
        for (int i = 0; i < ndst; ++i) {
            const h3_tensor *d = &sets[part][i];
            H3_CHECK(check_bf16(d));
            if (d->ndim != 3 || d->shape[0] != T || d->shape[1] != hpd || d->shape[2] != 128) return H3_ERR_BAD_SHAPE;
            if (d->strides[0] != d0->strides[0] || d->strides[1] != d0->strides[1] || d->strides[2] != 1)
                return H3_ERR_BAD_LAYOUT;
            if (!aligned16(d->data)) return H3_ERR_BAD_LAYOUT;
            p.dst[part][i] = static_cast<__nv_bfloat16 *>(d->data);
        }
    }
    if (d0->strides[0] % 8 != 0 || d0->strides[1] % 8 != 0) return H3_ERR_BAD_LAYOUT;
    for (const h3_tensor *nw : {norm_q, norm_k}) {
        H3_CHECK(check_bf16(nw));
        if (nw->ndim != 1 || nw->shape[0] != 128) return H3_ERR_BAD_SHAPE;
        if (nw->strides[0] != 1 || !aligned16(nw->data)) return H3_ERR_BAD_LAYOUT;
    }
    for (const h3_tensor *cs : {cos, sin}) {
        H3_CHECK(check_bf16(cs));
        if (cs->ndim != 2 || cs->shape[0] != T) return H3_ERR_BAD_SHAPE;
        if (cs->shape[1] != gemm::QKV_HALF && cs->shape[1] != 64) return H3_ERR_UNSUPPORTED;
        if (cs->shape[1] != cos->shape[1]) return H3_ERR_BAD_SHAPE;
        if (cs->strides[1] != 1 || (T > 1 && cs->strides[0] % 8 != 0) || !aligned16(cs->data)) return H3_ERR_BAD_LAYOUT;
    }
    p.M = (int)T;
    p.N = (int)w->shape[0];
    p.K = (int)x->shape[1];
    p.hcols = (int)(H * 128);
    p.hpd = (int)hpd;
    p.drow = d0->strides[0];
    p.dhead = d0->strides[1];
    p.norm_q = static_cast<const __nv_bfloat16 *>(norm_q->data);
    p.norm_k = static_cast<const __nv_bfloat16 *>(norm_k->data);
    p.cos = static_cast<const __nv_bfloat16 *>(cos->data);
    p.sin = static_cast<const __nv_bfloat16 *>(sin->data);
    p.cs0 = cos->strides[0];
    p.ss0 = sin->strides[0];
    p.eps = eps;
    if (cos->shape[1] == 64) return launch_gemm<gemm::EPI_QKV64>(x, w, p, (cudaStream_t)stream);
    return launch_gemm<gemm::EPI_QKV>(x, w, p, (cudaStream_t)stream);
}

extern "C" int h3_pack_gate_up(const h3_tensor *dst, const h3_tensor *src, void *stream) {
    H3_CHECK(check_matrix(dst));
    H3_CHECK(check_matrix(src));
    H3_CHECK(check_same_shape(dst, src));
    if (src->shape[0] % 256 != 0 || src->shape[1] % 8 != 0) return H3_ERR_BAD_SHAPE;
    const int64_t F = src->shape[0] / 2, K = src->shape[1];
    if (F == 0 || K == 0) return H3_OK;
    const int64_t work = 2 * F * (K / 8);
    int blocks = (int)((work + 255) / 256);
    if (blocks > num_sms() * 16) blocks = num_sms() * 16;
    gemm::pack_gate_up_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
        static_cast<__nv_bfloat16 *>(dst->data), dst->strides[0], static_cast<const __nv_bfloat16 *>(src->data),
        src->strides[0], F, K);
    return launch_status();
}

extern "C" int h3_gemm_variant(int variant) {
    if (variant < 0 || variant > 2) return -1;
    return g_gemm_variant.exchange(variant);
}

extern "C" unsigned int h3_gemm_device_error_read_and_clear(void) {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, h3::g_h3_device_error, sizeof(v));
    cudaMemcpyToSymbol(h3::g_h3_device_error, &zero, sizeof(zero));
    return v;
}
