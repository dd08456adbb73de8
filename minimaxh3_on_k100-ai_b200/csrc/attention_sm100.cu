// Non-causal BF16 flash attention for sm_100a on tcgen05 / TMEM, fed by TMA.
//
// Computes what the reference's mha op computes for the H3 DiT
// (patches/InfiniCore.patch:1333-1426; NineToothed kernel tools/h3_attention.py:25-41):
//   logits = (Q K^T) * scale * log2(e)  (fp32),  online max,  P = exp2(logits - max),
//   O = sum P_bf16 V / sum P  (fp32 accumulation), keys masked by K's length.
//
// One CTA owns two 128-row Q tiles of one (batch, head) and streams the K/V tiles
// of 128 keys through a 5-slot TMA ring (no multicast).  Warp roles (384 threads):
//   warp 0        TMA producer (one elected lane)
//   warp 1        tcgen05.mma issuer (one lane) and TMEM owner
//   warps 4..7    softmax + correction + epilogue for Q tile 0
//   warps 8..11   softmax + correction + epilogue for Q tile 1
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512), fp32,
// one query row per TMEM lane.  The two tiles ping-pong: while one softmax
// warpgroup exponentiates its S, the tensor core computes the other tile's S or
// P V.  P is written by the softmax threads as packed BF16 pairs back into the
// first 64 columns of their own S region (tcgen05.st) and consumed from TMEM by
// a TS MMA (A operand in tensor memory); V is the MN-major B operand in shared
// memory.  Before S_t(j+1) overwrites that region the MMA warp waits for the
// commit of P_t(j) V_j, which is already in flight behind the other tile's PV,
// so the tensor pipe does not drain.  A configurable share of the exponentials
// (H3_ATTN_POLY_PAIRS of every 8 key pairs of a full tile) can be computed on the
// FMA pipe with a Cody-Waite split 2^x = 2^round(x) * 2^f, f in [-1/2, 1/2], and
// a degree-3 polynomial for 2^f fitted by Lawson's minimax iteration (max
// relative error 7.5e-5, far below the BF16 rounding P receives); on B200 the
// sweep 0/2/3/4/5 measured 1054/942/948/904/876 TFLOP/s at [1,40,18432,128],
// so the default keeps every exponential on the MUFU ex2 unit (the softmax is
// issue-bound, not MUFU-bound).  The running max is updated lazily (only when it grows by more than
// 2^8 in the exp2 domain), so O is rescaled rarely; the normalisation uses the
// same stale max in numerator and denominator, so the result is unchanged up to
// fp32 rounding.  The epilogue divides by the row sum, rounds to BF16 and writes
// through a swizzled shared tile with a TMA store (rows past Sq are clipped).
#include <math.h>
#include <stdint.h>

#include "h3_abi_util.h"
#include "h3_common.cuh"
#include "sm100_ptx.cuh"
#include "tma_host.h"

namespace h3 {
namespace attn {

constexpr int BM = 128;                       // query rows per tile
constexpr int BN = 128;                       // keys per K/V tile
constexpr int HD = 128;                       // head dim
constexpr int NQ = 2;                         // Q tiles per CTA
constexpr int STAGES = 5;                     // K/V ring slots
constexpr int TILE = BM * HD * 2;             // 32 KB: one 128x128 BF16 tile
constexpr int HALF = TILE / 2;                // 16 KB: 64 columns (one 128B swizzle span)
constexpr int THREADS = 384;
constexpr uint32_t TMEM_COLS = 512;
constexpr float RESCALE_THRESHOLD = 8.0f;     // log2 domain

#ifndef H3_ATTN_POLY_PAIRS
#define H3_ATTN_POLY_PAIRS 0   // measured fastest on B200: the MUFU is not the limit here
#endif
constexpr int POLY_PAIRS = H3_ATTN_POLY_PAIRS; // of every 8 key pairs, exponentiated on the FMA pipe

constexpr int OFF_Q = 0;
constexpr int OFF_KV = OFF_Q + NQ * TILE;
constexpr int OFF_BAR = OFF_KV + STAGES * TILE;
constexpr int NUM_BARS = 1 + 2 * STAGES + 3 * NQ;
constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 16 + 1024;  // + tmem slot, abort flag, alignment slack

struct Params {
    int Sq, Sk, H, B;
    int nkv;
    float scale_log2;
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x on the FMA pipe: x = n + f with n = round(x) (the 1.5*2^23 addition
// leaves n in the low mantissa bits), 2^f by a degree-3 polynomial on
// [-1/2, 1/2], then n is added to the exponent field.  x is clamped at -126 so
// the exponent never wraps (the result is then a tiny non-negative number).
__device__ __forceinline__ float exp2_poly(float x) {
    x = fmaxf(x, -126.0f);
    const float t = __fadd_rn(x, 12582912.0f);
    const float f = __fsub_rn(x, __fsub_rn(t, 12582912.0f));
    float p = fmaf(0.0551716685295105f, f, 0.2426111251115799f);
    p = fmaf(p, f, 0.6932609677314758f);
    p = fmaf(p, f, 0.9999280571937561f);
    return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// Blackwell packed fp32 pairs (fma.rn.f32x2 / add.rn.f32x2) and the 3-input
// max halve the issue slots of the softmax's per-element fp32 work.
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ uint64_t pk2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void up2(uint64_t v, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a 128B-swizzled 64-column half
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
    return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(THREADS, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to, Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem + OFF_Q;
    uint8_t *sKV = smem + OFF_KV;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *q_full = bars;
    uint64_t *kv_full = bars + 1;
    uint64_t *kv_empty = kv_full + STAGES;
    uint64_t *s_full = kv_empty + STAGES;
    uint64_t *p_ready = s_full + NQ;
    uint64_t *o_done = p_ready + NQ;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NUM_BARS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int h = blockIdx.y, b = blockIdx.z;
    const int q0 = blockIdx.x * (NQ * BM);

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int t = 0; t < NQ; ++t) {
            mbar_init(&s_full[t], 1);
            mbar_init(&p_ready[t], 128);
            mbar_init(&o_done[t], 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&tq);
            tma_prefetch_desc(&tk);
            tma_prefetch_desc(&tv);
            mbar_expect_tx(q_full, NQ * TILE);
            for (int t = 0; t < NQ; ++t)
                for (int hf = 0; hf < 2; ++hf)
                    tma_load_4d(sQ + t * TILE + hf * HALF, &tq, q_full, hf * 64, q0 + t * BM, h, b);
            for (int j = 0; j < p.nkv; ++j) {
                bool ok = true;
                for (int kv = 0; kv < 2 && ok; ++kv) {
                    const int i = 2 * j + kv, slot = i % STAGES, use = i / STAGES;
                    ok = mbar_wait(&kv_empty[slot], (use & 1) ^ 1, abort_flag);
                    if (!ok) break;
                    mbar_expect_tx(&kv_full[slot], TILE);
                    const CUtensorMap *m = kv ? &tv : &tk;
                    for (int hf = 0; hf < 2; ++hf)
                        tma_load_4d(sKV + slot * TILE + hf * HALF, m, &kv_full[slot], hf * 64, j * BN, h, b);
                }
                if (!ok) break;
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t ID_S = idesc_bf16_f32(BM, BN, false);  // Q (K-major) x K (K-major)
            constexpr uint32_t ID_PV = idesc_bf16_f32(BM, HD, true);  // P (K-major) x V (MN-major)
            bool ok = mbar_wait(q_full, 0, abort_flag);
            tc_fence_after();
            const uint32_t q_base = smem_u32(sQ), kv_base = smem_u32(sKV);
            // S_t(j) = Q_t K_j^T into TMEM columns [t*BN, t*BN+BN)
            auto issue_s = [&](int t, uint32_t kaddr) {
                const uint32_t qaddr = q_base + t * TILE;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk) {
                    const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
                    umma_ss(tmem + t * BN, smem_desc_sw128(qaddr + off, 16, 1024),
                            smem_desc_sw128(kaddr + off, 16, 1024), ID_S, kk > 0);
                }
                umma_commit(&s_full[t]);
            };
            // prologue: S_0(0), S_1(0)
            if (ok) ok = mbar_wait(&kv_full[0], 0, abort_flag);
            if (ok) {
                tc_fence_after();
                for (int t = 0; t < NQ; ++t) issue_s(t, kv_base);
                umma_commit(&kv_empty[0]);
            }
            // steady state, ping-pong order: PV_0(j), S_0(j+1), PV_1(j), S_1(j+1).  S_t(j+1)
            // overwrites P_t(j) (aliased in TMEM), so it waits for the commit of PV_t(j);
            // meanwhile the tensor pipe is busy with PV_t(j) itself, and softmax t can start
            // on tile j+1 while the other warpgroup still works on tile j.
            for (int j = 0; j < p.nkv && ok; ++j) {
                const int iv = 2 * j + 1, sv = iv % STAGES;
                const int ik = 2 * j + 2, sk = ik % STAGES;
                const bool more = j + 1 < p.nkv;
                ok = mbar_wait(&kv_full[sv], (iv / STAGES) & 1, abort_flag);
                if (!ok) break;
                const uint32_t vaddr = kv_base + sv * TILE;
                const uint32_t kaddr = kv_base + sk * TILE;
                for (int t = 0; t < NQ && ok; ++t) {
                    ok = mbar_wait(&p_ready[t], j & 1, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < BN / 16; ++kk)  // P: 16 keys = 8 packed columns per step
                        umma_ts(tmem + 2 * BN + t * HD, tmem + t * BN + kk * 8,
                                smem_desc_sw128(vaddr + kk * 2048, HALF, 1024), ID_PV, (j > 0 || kk > 0) ? 1u : 0u);
                    umma_commit(&o_done[t]);
                    if (more) {
                        if (t == 0) ok = mbar_wait(&kv_full[sk], (ik / STAGES) & 1, abort_flag);
                        if (ok) ok = mbar_wait(&o_done[t], j & 1, abort_flag);
                        if (!ok) break;
                        tc_fence_after();
                        issue_s(t, kaddr);
                    }
                }
                if (!ok) break;
                umma_commit(&kv_empty[sv]);
                if (more) umma_commit(&kv_empty[sk]);
            }
            if (!ok) drain_in_flight();
        }
    } else if (warp >= 4) {
        // ------------------------------------------------------------ softmax / epilogue
        const int t = (warp - 4) >> 2;
        const int row = (warp & 3) * 32 + lane;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t s_addr = tmem + t * BN + lane_off;
        const uint32_t o_addr = tmem + 2 * BN + t * HD + lane_off;
        const float c = p.scale_log2;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < p.nkv; ++j) {
            // s_full(j) implies P_t(j-1) V_{j-1} has landed: S_t(j) was issued after its commit
            ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, abort_flag));
            if (!ok) break;
            tc_fence_after();
            uint32_t s[128];
            tmem_ld32(s_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
            tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
            tmem_ld32(s_addr + 64, *reinterpret_cast<uint32_t(*)[32]>(&s[64]));
            tmem_ld32(s_addr + 96, *reinterpret_cast<uint32_t(*)[32]>(&s[96]));
            tmem_ld_wait();
            const int valid = p.Sk - j * BN;
            const bool full = valid >= BN;
            if (!full) {
#pragma unroll
                for (int i = 0; i < 128; ++i)
                    if (i >= valid) s[i] = __float_as_uint(-INFINITY);
            }
            float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
            for (int i = 0; i < 128; i += 8) {
                mx0 = max3f(mx0, __uint_as_float(s[i]), __uint_as_float(s[i + 1]));
                mx1 = max3f(mx1, __uint_as_float(s[i + 2]), __uint_as_float(s[i + 3]));
                mx2 = max3f(mx2, __uint_as_float(s[i + 4]), __uint_as_float(s[i + 5]));
                mx3 = max3f(mx3, __uint_as_float(s[i + 6]), __uint_as_float(s[i + 7]));
            }
            const float mnew = fmaxf(max3f(mx0, mx1, mx2), mx3) * c;
            float alpha = 1.f;
            bool rescale = false;
            if (j == 0) {
                m = mnew;
            } else if (mnew > m + RESCALE_THRESHOLD) {
                alpha = ex2(m - mnew);
                m = mnew;
                rescale = true;
            }
            // tcgen05.ld/st are warp-collective: rescale the whole warp's rows if any needs it
            if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
                for (int cc = 0; cc < 4; ++cc) {
                    uint32_t o[32];
                    tmem_ld32(o_addr + cc * 32, o);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                    tmem_st32(o_addr + cc * 32, o);
                }
            }
            const float neg_m = -m;
            const uint64_t c2 = pk2(c, c), nm2 = pk2(neg_m, neg_m);
            uint64_t rs0 = pk2(0.f, 0.f), rs1 = pk2(0.f, 0.f);
            // P overwrites columns [0, 64) of this tile's S region (S is already in registers)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                uint32_t w[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    float x0, x1;   // s * c - m for a key pair, one packed FMA
                    up2(ffma2(pk2(__uint_as_float(s[64 * hf + 2 * i]), __uint_as_float(s[64 * hf + 2 * i + 1])),
                              c2, nm2), x0, x1);
                    float p0, p1;
                    if (full && (i & 7) < POLY_PAIRS) {
                        p0 = exp2_poly(x0);
                        p1 = exp2_poly(x1);
                    } else {
                        p0 = ex2(x0);
                        p1 = ex2(x1);
                    }
                    if (i & 1) rs1 = fadd2(rs1, pk2(p0, p1));
                    else rs0 = fadd2(rs0, pk2(p0, p1));
                    w[i] = pack_bf16x2(p0, p1);
                }
                tmem_st32(s_addr + 32 * hf, w);
            }
            float r0, r1, r2, r3;
            up2(rs0, r0, r1);
            up2(rs1, r2, r3);
            l = l * alpha + ((r0 + r1) + (r2 + r3));
            tmem_st_wait();
            tc_fence_before();
            mbar_arrive(&p_ready[t]);
        }
        if (ok && p.nkv > 0) ok = mbar_wait(&o_done[t], (p.nkv - 1) & 1, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
            tc_fence_after();
            const float inv = 1.0f / l;
            const uint32_t out_tile = smem_u32(sQ + t * TILE);  // Q tile is free once the last PV landed
#pragma unroll 1
            for (int cc = 0; cc < 4; ++cc) {
                uint32_t o[32];
                tmem_ld32(o_addr + cc * 32, o);
                tmem_ld_wait();
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int chunk = (cc & 1) * 4 + q;
                    st_shared_v4(out_tile + (cc >> 1) * HALF + swz(row, chunk),
                                 pack_bf16x2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                                 pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                                 pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                                 pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
                }
            }
            fence_proxy_async_smem();
            named_bar_sync(1 + t, 128);
            if (row == 0 && q0 + t * BM < p.Sq) {
                tma_store_4d(&to, sQ + t * TILE, 0, q0 + t * BM, h, b);
                tma_store_4d(&to, sQ + t * TILE + HALF, 64, q0 + t * BM, h, b);
                tma_store_commit();
                tma_store_wait_all();
            }
        } else {
            drain_in_flight();
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace attn
}  // namespace h3

using namespace h3;

namespace {

// [B, S, H, 128] BF16 view -> 4-D tensor map (D, S, H, B), box (64, 128, 1, 1)
int attn_tmap(CUtensorMap *map, const h3_tensor *t) {
    const cuuint64_t dims[4] = {(cuuint64_t)t->shape[3], (cuuint64_t)t->shape[1], (cuuint64_t)t->shape[2],
                                (cuuint64_t)t->shape[0]};
    // a size-1 batch dim may carry any stride; give TMA a legal one
    const int64_t sb = t->shape[0] == 1 ? t->strides[1] * t->shape[1] : t->strides[0];
    const int64_t sh = t->shape[2] == 1 ? 128 : t->strides[2];
    const cuuint64_t strides[3] = {(cuuint64_t)t->strides[1] * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
    const cuuint32_t box[4] = {64, attn::BM, 1, 1};
    return make_tmap_bf16(map, t->data, 4, dims, strides, box);
}

int check_attn_operand(const h3_tensor *t) {
    H3_CHECK(check_bf16(t));
    if (t->ndim != 4 || t->shape[3] != 128) return H3_ERR_BAD_SHAPE;
    if (t->strides[3] != 1 || !aligned16(t->data)) return H3_ERR_BAD_LAYOUT;
    for (int i = 0; i < 3; ++i)
        if (t->shape[i] > 1 && (t->strides[i] % 8 != 0 || t->strides[i] <= 0)) return H3_ERR_BAD_LAYOUT;
    if (t->shape[1] > (int64_t)0x7fffffff || t->shape[2] > 65535 || t->shape[0] > 65535) return H3_ERR_UNSUPPORTED;
    return H3_OK;
}

}  // namespace

extern "C" int h3_mha(const h3_tensor *out, const h3_tensor *q, const h3_tensor *k, const h3_tensor *v, float scale,
                      void *stream) {
    H3_CHECK(check_attn_operand(out));
    H3_CHECK(check_attn_operand(q));
    H3_CHECK(check_attn_operand(k));
    H3_CHECK(check_attn_operand(v));
    H3_CHECK(check_same_shape(out, q));
    H3_CHECK(check_same_shape(k, v));
    if (q->shape[0] != k->shape[0] || q->shape[2] != k->shape[2]) return H3_ERR_BAD_SHAPE;
    const int B = (int)q->shape[0], Sq = (int)q->shape[1], H = (int)q->shape[2], Sk = (int)k->shape[1];
    if (B == 0 || Sq == 0 || H == 0) return H3_OK;
    if (Sk == 0) return H3_ERR_BAD_SHAPE;
    CUtensorMap tq, tk, tv, to;
    H3_CHECK(attn_tmap(&tq, q));
    H3_CHECK(attn_tmap(&tk, k));
    H3_CHECK(attn_tmap(&tv, v));
    H3_CHECK(attn_tmap(&to, out));
    attn::Params p;
    p.Sq = Sq;
    p.Sk = Sk;
    p.H = H;
    p.B = B;
    p.nkv = (Sk + attn::BN - 1) / attn::BN;
    p.scale_log2 = scale * 1.4426950408889634f;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !attr_set[dev]) {
        if (cudaFuncSetAttribute(attn::fa_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 attn::SMEM_BYTES) != cudaSuccess)
            return H3_ERR_LAUNCH;
        attr_set[dev] = true;
    }
    const dim3 grid((unsigned)((Sq + attn::NQ * attn::BM - 1) / (attn::NQ * attn::BM)), (unsigned)H, (unsigned)B);
    attn::fa_fwd_kernel<<<grid, attn::THREADS, attn::SMEM_BYTES, (cudaStream_t)stream>>>(tq, tk, tv, to, p);
    return launch_status();
}

// device error word of this translation unit (bounded waits in the attention kernel)
extern "C" unsigned int h3_attention_device_error_read_and_clear(void) {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, h3::g_h3_device_error, sizeof(v));
    cudaMemcpyToSymbol(h3::g_h3_device_error, &zero, sizeof(zero));
    return v;
}
