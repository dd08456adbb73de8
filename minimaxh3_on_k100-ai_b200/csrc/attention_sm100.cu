// Non-causal BF16 flash attention for sm_100a on tcgen05 / TMEM, fed by TMA.
//
// Computes what the reference's mha op computes for the H3 DiT
// (patches/InfiniCore.patch:1333-1426; NineToothed kernel tools/h3_attention.py:25-41):
//   logits = (Q K^T) * scale * log2(e)  (fp32),  online max,  P = exp2(logits - max),
//   O = sum P_bf16 V / sum P  (fp32 accumulation), keys masked by K's length.
//
// One CTA owns two 128-row Q tiles of one (batch, head) and streams K/V tiles of
// 128 keys by TMA (no multicast).  A CTA fills an SM, so when the grid's last
// wave would hold at most half as many pairs as there are SMs, those pairs run as
// two one-tile CTAs each (measured alone, a one-tile CTA takes about 0.7 of a pair's
// time); the per-tile arithmetic does not change, so results are bitwise the same.  Warp
// roles (384 threads):
//   warp 0        TMA producer for Q and K (one lane)
//   warp 1        tcgen05.mma issuer for S = Q K^T (one lane) and TMEM owner
//   warp 2        tcgen05.mma issuer for O += P V (one lane)
//   warp 3        TMA producer for V (one lane)
//   warps 4..7    softmax + correction + epilogue for Q tile 0
//   warps 8..11   softmax + correction + epilogue for Q tile 1
// TMEM (512 columns, fp32, one query row per lane): S_0 [0,128) S_1 [128,256)
// O_0 [256,384) O_1 [384,512).  The softmax warps write P_t(j) in BF16 to a
// 128B-swizzled shared tile per Q tile (the layout TMA gives Q), and P V is a
// shared x shared MMA with V as the MN-major B operand.  Shared memory: Q 64 KB,
// P 64 KB, a two-slot K ring 64 KB, one V buffer 32 KB.  K_j is read early in
// step j (by S_t(j)) and V_j late (by P_t(j) V_j); a 32 KB tile takes about 2000
// cycles to arrive, so K keeps one tile in flight and V reloads within the step.
//
// With P outside tensor memory nothing ties S_t(j+1) to P_t(j) V_j: the softmax
// warps release S_t as soon as their tcgen05.ld of it has completed, and the
// tensor core computes S_t(j+1) while they exponentiate tile j.  The waits left
// on a tile's path are the softmax itself and, before P_t(j+1) overwrites the P
// tile (and before a rescale of O_t), the commit of P_t(j) V_j, which by then
// has normally landed.  The two products have separate issuing threads (each
// thread's commits track only its own MMAs), so one thread's barrier waits
// overlap the other's issue; the tensor pipe's instruction queue is shallow.
// Measured on B200 at [1,40,18432,128] this layout runs at ~1220 TFLOP/s against
// ~1100 for P aliased into S in TMEM, and 936 for P in TMEM with a single in-order
// issuer (P_t(j) V_j then S_t(j+1)) and 1 in 4 exponentials on the FMA pipe -- there
// the softmax of tile t waits for two products after its own, so the two Q tiles
// cannot keep the tensor pipe fed; 64-key tiles with double-buffered S (N=64
// MMAs run at half rate), a shared P tile, alternating the two softmax groups'
// exponentials, and moving exponentials to the FMA pipe were all slower.  So was
// a CTA-pair form (clusters of 2, tcgen05 cta_group::2 M=256 products, each CTA
// holding half of every K and V tile, which halves the B-operand bytes the tensor
// core reads from shared memory): 824 TFLOP/s against 1199-1235, with 2 or 3 ring
// slots for K and V alike -- every key tile's S and P V products then wait on
// both CTAs' softmax warps through barriers on the other SM.
//
// The running max is updated lazily (only when it grows by more than 2^8 in the
// exp2 domain), so O is rescaled rarely.  Numerator and denominator use the same
// stale max, so the softmax itself is unchanged; but each P = exp2(x - m_stale)
// is rounded to BF16 at a scale that differs from the true-max one by a factor
// that is not a power of two, so a P term's BF16 rounding can differ from the
// reference kernel's by one BF16 ulp.  The result matches the reference within
// BF16 tolerance (the tests' fp32 bounds), not bit for bit.
//
// H3_ATTN_POLY_PAIRS of every 8 key pairs of a full tile can be exponentiated on
// the FMA pipe instead of the MUFU.  The epilogue divides by the row sum, rounds
// to BF16 and writes through a swizzled shared tile with a TMA store (rows past
// Sq are clipped), or -- for the Ulysses return leg (h3_mha_scatter) -- with
// 16-byte row stores straight into the return buffer of the rank that owns each
// row's token (a peer's memory over NVLink), so no separate copy or permute
// follows the attention.
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
#ifndef H3_ATTN_KSLOTS
#define H3_ATTN_KSLOTS 2
#endif
#ifndef H3_ATTN_VSLOTS
#define H3_ATTN_VSLOTS 1
#endif
constexpr int KSLOTS = H3_ATTN_KSLOTS;        // K ring slots
constexpr int VSLOTS = H3_ATTN_VSLOTS;        // V ring slots
#ifndef H3_ATTN_SPLIT_TAIL
#define H3_ATTN_SPLIT_TAIL 1   // run a short last wave of Q-tile pairs as one-tile CTAs
#endif
#ifndef H3_ATTN_L2_AHEAD
#define H3_ATTN_L2_AHEAD 4
#endif
constexpr int L2_AHEAD = H3_ATTN_L2_AHEAD;    // key tiles between an L2 prefetch and the load
constexpr int TILE = 128 * 128 * 2;           // 32 KB: one 128x128 BF16 tile (Q, P, K or V)
constexpr int HALF = TILE / 2;                // 16 KB: its 64-column (128B swizzle span) half
constexpr int THREADS = 384;
constexpr uint32_t TMEM_COLS = 512;
constexpr int O_COL = NQ * BN;                // first O column
constexpr float RESCALE_THRESHOLD = 8.0f;     // log2 domain

#ifndef H3_ATTN_POLY_PAIRS
#define H3_ATTN_POLY_PAIRS 0   // measured fastest on B200 (the softmax warps are latency-bound)
#endif
constexpr int POLY_PAIRS = H3_ATTN_POLY_PAIRS; // of every 8 key pairs, exponentiated on the FMA pipe
#ifndef H3_ATTN_SUM_GROUPS
#define H3_ATTN_SUM_GROUPS 2
#endif
// The row sum of a key tile is taken in SUM_GROUPS groups of consecutive key pairs,
// each with two packed fp32x2 accumulators (even / odd pairs), and each group keeps
// its own running sum across key tiles; short addition chains leave the scheduler
// room to overlap the exponentials (measured: one group of 64 pairs ran ~1200-1235
// TFLOP/s at [1,40,18432,128], two groups of 32 ~1315)
constexpr int SUM_GROUPS = H3_ATTN_SUM_GROUPS;
constexpr int GROUP_PAIRS = BN / 2 / SUM_GROUPS;
#ifndef H3_ATTN_MAX_BF16
#define H3_ATTN_MAX_BF16 0
#endif
// Measured equal within the pool's run-to-run spread at [1,40,18432,128] (1267-1311
// TFLOP/s for all four combinations in one call), so the defaults are kept:
#ifndef H3_ATTN_MAX_ACC
#define H3_ATTN_MAX_ACC 4      // independent max chains over a row of S (4 or 8)
#endif
#ifndef H3_ATTN_EARLY_P
#define H3_ATTN_EARLY_P 0      // store each row-sum group's P chunks as soon as they are ready
#endif
// Register split (setmaxnreg): the load / MMA warpgroup gives registers to the two
// softmax warpgroups.  0 = off.  CTRL_REGS * 128 + 2 * SOFTMAX_REGS * 128 may not
// exceed the registers the CTA is launched with (its per-thread count x 384); the
// host checks that before the first launch, since a setmaxnreg.inc that the pool
// cannot satisfy waits forever.
#ifndef H3_ATTN_SOFTMAX_REGS
#define H3_ATTN_SOFTMAX_REGS 0
#endif
#ifndef H3_ATTN_CTRL_REGS
#define H3_ATTN_CTRL_REGS 40
#endif
constexpr int SOFTMAX_REGS = H3_ATTN_SOFTMAX_REGS;
constexpr int CTRL_REGS = H3_ATTN_CTRL_REGS;
static_assert(SOFTMAX_REGS == 0 || (SOFTMAX_REGS % 8 == 0 && CTRL_REGS % 8 == 0 && CTRL_REGS >= 24 &&
                                    SOFTMAX_REGS <= 256 && CTRL_REGS * 128 + 2 * SOFTMAX_REGS * 128 <= 65536),
              "register split out of range");

constexpr int OFF_Q = 0;
constexpr int OFF_P = OFF_Q + NQ * TILE;
constexpr int OFF_K = OFF_P + NQ * TILE;
constexpr int OFF_V = OFF_K + KSLOTS * TILE;
constexpr int OFF_BAR = OFF_V + VSLOTS * TILE;
constexpr int VSLOTS_1 = VSLOTS > 2 ? VSLOTS : 2;  // V barriers: a one-tile CTA's slot 1 is Q tile 1's space
constexpr int NUM_BARS = 1 + 2 * KSLOTS + 2 * VSLOTS_1 + 4 * NQ;
constexpr int SMEM_BYTES = OFF_BAR + NUM_BARS * 8 + 16 + 1024;  // + tmem slot, abort flag, alignment slack
static_assert(SMEM_BYTES <= 232448, "shared memory over the sm_100 per-block limit");

struct Params {
    int Sq, Sk, H, B;
    int nkv;
    float scale_log2;
    int tiles;       // 128-row Q tiles per (batch, head)
    int pairs;       // Q tile pairs per (batch, head): ceil(tiles / 2)
    int split_from;  // CTAs [0, split_from) own a pair; pair split_from + i runs as CTAs split_from + 2i (+1)
    // Scatter epilogue (ndst > 0, batch 1): output row g of head h goes to
    // dst[g / rows_per_dst] + (g % rows_per_dst) * d_row + h * d_head -- the Ulysses
    // return leg, each destination a rank's return buffer (local or a peer's).
    int ndst;
    int rows_per_dst;
    int64_t d_row, d_head;
    __nv_bfloat16 *dst[H3_EXCHANGE_MAX_RANKS];
};

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
__device__ __forceinline__ void st_global_v4(void *ptr, const uint4 &v) {
    asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(ptr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}


__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
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

// 2^x for a pair of values on the FMA pipe (packed fp32x2): x = n + f with
// n = round(x) (the 1.5*2^23 addition leaves n in the low mantissa bits), 2^f by
// a degree-3 polynomial on [-1/2, 1/2] (Lawson minimax fit, max relative error
// 7.5e-5), then n is added to the exponent field.  x is clamped at -126 so the
// exponent never wraps (the result is then a tiny non-negative number).
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float &p0, float &p1) {
    const uint64_t x = pk2(fmaxf(x0, -126.0f), fmaxf(x1, -126.0f));
    const uint64_t t = fadd2(x, pk2(12582912.0f, 12582912.0f));
    const uint64_t r = fadd2(t, pk2(-12582912.0f, -12582912.0f));  // round(x), exact
    const uint64_t f = ffma2(r, pk2(-1.0f, -1.0f), x);               // x - round(x), exact
    uint64_t q = ffma2(pk2(0.0551716685295105f, 0.0551716685295105f), f,
                       pk2(0.2426111251115799f, 0.2426111251115799f));
    q = ffma2(q, f, pk2(0.6932609677314758f, 0.6932609677314758f));
    q = ffma2(q, f, pk2(0.9999280571937561f, 0.9999280571937561f));
    float q0, q1, t0, t1;
    up2(q, q0, q1);
    up2(t, t0, t1);
    p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
    p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}

// the smallest BF16 value >= x (x finite or -inf)
__device__ __forceinline__ float bf16_round_up(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0xFFFFu) != 0u && !(u >> 31)) u += 0x10000u;   // positive with dropped bits: up
    return __uint_as_float(u & 0xFFFF0000u);                 // negative: truncation rounds up
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

// The work of one CTA on NQT (1 or 2) Q tiles starting at row q0 of (batch b, head h).
template <int NQT>
__device__ __forceinline__ void fa_cta(const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv,
                                       const CUtensorMap &to, const Params &p, const int h, const int b,
                                       const int q0) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem + OFF_Q;
    uint8_t *sP = smem + OFF_P;
    uint8_t *sK = smem + OFF_K;
    uint8_t *sV = smem + OFF_V;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *q_full = bars;
    uint64_t *k_full = bars + 1;
    uint64_t *k_empty = k_full + KSLOTS;
    uint64_t *v_full = k_empty + KSLOTS;
    uint64_t *v_empty = v_full + VSLOTS_1;
    uint64_t *s_full = v_empty + VSLOTS_1;  // [t]: S_t(j) in TMEM
    uint64_t *s_free = s_full + NQ;         // [t]: softmax t has read S_t(j)
    uint64_t *p_ready = s_free + NQ;        // [t]: P_t(j) in shared memory, O_t rescaled
    uint64_t *o_done = p_ready + NQ;        // [t]: P_t(j) V_j has landed in O_t
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + NUM_BARS);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    constexpr int nq = NQT;
    const int nkv = p.nkv;
    // A pair's softmax hides a V tile's load behind the other tile's work; a lone
    // tile's does not, so a one-tile CTA double-buffers V, its second slot in the
    // unused Q tile 1.  V_j goes to slot vslot(j), its use count there is vuse(j).
    constexpr bool v2 = NQT == 1 && VSLOTS == 1;
    auto vslot = [&](int j) { return v2 ? (j & 1) : j % VSLOTS; };
    auto vuse = [&](int j) { return v2 ? (j >> 1) : j / VSLOTS; };

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < KSLOTS; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
        }
        for (int i = 0; i < VSLOTS_1; ++i) {
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int t = 0; t < NQ; ++t) {
            mbar_init(&s_full[t], 1);
            mbar_init(&s_free[t], 128);
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
    if (SOFTMAX_REGS > 0) {   // warpgroup-uniform: warps 0-3, 4-7, 8-11
        if (warp < 4) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(CTRL_REGS));
        else asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(SOFTMAX_REGS));
    }

    if (warp < 4) {
        if ((warp == 0 || warp == 3) && lane == 0) {
            // -------------------------------------------------------- TMA producers
            const bool kq = warp == 0;   // warp 0: Q and K; warp 3: V
            if (kq) {
                tma_prefetch_desc(&tq);
                tma_prefetch_desc(&tk);
                mbar_expect_tx(q_full, nq * TILE);
                for (int t = 0; t < nq; ++t)
                    for (int hf = 0; hf < 2; ++hf)
                        tma_load_4d(sQ + t * TILE + hf * HALF, &tq, q_full, hf * 64, q0 + t * BM, h, b);
            } else {
                tma_prefetch_desc(&tv);
            }
            // use u of a slot waits for the release of use u - 1
            auto load_tile = [&](const CUtensorMap *m, uint8_t *dst, uint64_t *full, uint64_t *empty, int use,
                                 int row0) -> bool {
                if (!mbar_wait(empty, (use & 1) ^ 1, abort_flag)) return false;
                mbar_expect_tx(full, TILE);
                for (int hf = 0; hf < 2; ++hf) tma_load_4d(dst + hf * HALF, m, full, hf * 64, row0, h, b);
                return true;
            };
            // K/V tiles are requested L2_AHEAD key tiles before their load, so the load
            // itself hits in L2 rather than waiting for HBM (or the other die)
            auto prefetch = [&](int j) {
                for (int hf = 0; hf < 2; ++hf) tma_prefetch_l2_4d(kq ? &tk : &tv, hf * 64, j * BN, h, b);
            };
            for (int j = 1; j < L2_AHEAD && j < nkv; ++j) prefetch(j);
            bool ok = true;
            for (int j = 0; j < nkv && ok; ++j) {
                if (j + L2_AHEAD < nkv) prefetch(j + L2_AHEAD);
                if (kq) {
                    const int ks = j % KSLOTS;
                    ok = load_tile(&tk, sK + ks * TILE, &k_full[ks], &k_empty[ks], j / KSLOTS, j * BN);
                } else {
                    const int vs = vslot(j);
                    uint8_t *dst = v2 ? (vs ? sQ + TILE : sV) : sV + vs * TILE;
                    ok = load_tile(&tv, dst, &v_full[vs], &v_empty[vs], vuse(j), j * BN);
                }
            }
        } else if ((warp == 1 || warp == 2) && lane == 0) {
            // -------------------------------------------------------- MMA issuers
            constexpr uint32_t ID_S = idesc_bf16_f32(BM, BN, false);  // Q (K-major) x K (K-major)
            constexpr uint32_t ID_PV = idesc_bf16_f32(BM, HD, true);  // P (K-major) x V (MN-major)
            const uint32_t q_base = smem_u32(sQ), p_base = smem_u32(sP), k_base = smem_u32(sK),
                           v_base = smem_u32(sV);
            // D[t] = A_t (128 x 128, K-major, 128B swizzle) x B (128 x 128)
            auto issue = [&](uint32_t d, uint32_t a, uint32_t bsrc, bool pv, bool acc) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t ka = (kk >> 2) * HALF + (kk & 3) * 32;
                    const uint64_t bdesc = pv ? smem_desc_sw128(bsrc + kk * 2048, HALF, 1024)
                                              : smem_desc_sw128(bsrc + ka, 16, 1024);
                    umma_ss(d, smem_desc_sw128(a + ka, 16, 1024), bdesc, pv ? ID_PV : ID_S,
                            (acc || kk > 0) ? 1u : 0u);
                }
            };
            bool ok = true;
            if (warp == 1) {
                // S_t(j) = Q_t K_j^T, issued as soon as softmax t has read S_t(j-1)
                ok = mbar_wait(q_full, 0, abort_flag);
                for (int j = 0; j < nkv && ok; ++j) {
                    const int ks = j % KSLOTS;
                    ok = mbar_wait(&k_full[ks], (j / KSLOTS) & 1, abort_flag);
                    for (int t = 0; t < nq && ok; ++t) {
                        if (j > 0) ok = mbar_wait(&s_free[t], (j - 1) & 1, abort_flag);
                        if (!ok) break;
                        tc_fence_after();
                        issue(tmem + t * BN, q_base + t * TILE, k_base + ks * TILE, false, false);
                        umma_commit(&s_full[t]);
                    }
                    if (!ok) break;
                    umma_commit(&k_empty[ks]);
                }
            } else {
                // O_t += P_t(j) V_j once softmax t has written P_t(j)
                for (int j = 0; j < nkv && ok; ++j) {
                    const int vs = vslot(j);
                    const uint32_t vb = v2 ? (vs ? q_base + TILE : v_base) : v_base + vs * TILE;
                    ok = mbar_wait(&v_full[vs], vuse(j) & 1, abort_flag);
                    for (int t = 0; t < nq && ok; ++t) {
                        ok = mbar_wait(&p_ready[t], j & 1, abort_flag);
                        if (!ok) break;
                        tc_fence_after();
                        issue(tmem + O_COL + t * HD, p_base + t * TILE, vb, true, j > 0);
                        umma_commit(&o_done[t]);
                    }
                    if (!ok) break;
                    umma_commit(&v_empty[vs]);
                }
            }
            if (!ok) drain_in_flight();
        }
    } else if (((warp - 4) >> 2) < nq) {
        // ------------------------------------------------------------ softmax / epilogue
        const int t = (warp - 4) >> 2;
        const int row = (warp & 3) * 32 + lane;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t s_addr = tmem + t * BN + lane_off;
        const uint32_t o_addr = tmem + O_COL + t * HD + lane_off;
        const uint32_t p_tile = smem_u32(sP + t * TILE);
        const float c = p.scale_log2;
        float m = -INFINITY;
        float l[SUM_GROUPS];
#pragma unroll
        for (int g = 0; g < SUM_GROUPS; ++g) l[g] = 0.f;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, abort_flag));
            if (!ok) break;
            tc_fence_after();
            uint32_t s[BN];
            tmem_ld32(s_addr + 0, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
            tmem_ld32(s_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
            tmem_ld32(s_addr + 64, *reinterpret_cast<uint32_t(*)[32]>(&s[64]));
            tmem_ld32(s_addr + 96, *reinterpret_cast<uint32_t(*)[32]>(&s[96]));
            tmem_ld_wait();
            // S_t(j) is in registers: the tensor core may overwrite it with S_t(j+1)
            tc_fence_before();
            mbar_arrive(&s_free[t]);
            const int valid = p.Sk - j * BN;
            const bool full = valid >= BN;
            if (!full) {
#pragma unroll
                for (int i = 0; i < BN; ++i)
                    if (i >= valid) s[i] = __float_as_uint(-INFINITY);
            }
            // the row max (exact in any order): H3_ATTN_MAX_ACC independent chains
            constexpr int MA = H3_ATTN_MAX_ACC;
            float mx[MA];
#pragma unroll
            for (int k = 0; k < MA; ++k) mx[k] = -INFINITY;
#pragma unroll
            for (int i = 0; i < BN; i += 2 * MA)
#pragma unroll
                for (int k = 0; k < MA; ++k)
                    mx[k] = max3f(mx[k], __uint_as_float(s[i + 2 * k]), __uint_as_float(s[i + 2 * k + 1]));
#pragma unroll
            for (int w2 = MA / 2; w2 > 0; w2 /= 2)
#pragma unroll
                for (int k = 0; k < w2; ++k) mx[k] = fmaxf(mx[k], mx[k + w2]);
#if H3_ATTN_MAX_BF16
            const float mnew = bf16_round_up(mx[0]) * c;
#else
            const float mnew = mx[0] * c;
#endif
            float alpha = 1.f;
            bool rescale = false;
            if (j == 0) {
                m = mnew;
            } else if (mnew > m + RESCALE_THRESHOLD) {
                alpha = ex2(m - mnew);
                m = mnew;
                rescale = true;
            }
            const float neg_m = -m;
            const uint64_t c2 = pk2(c, c), nm2 = pk2(neg_m, neg_m);
            uint32_t w[BN / 2];
            // P_t(j-1) V_{j-1} must have read the P tile (and landed in O_t) before P_t(j)
            // overwrites it or O_t is rescaled
            auto release_p_tile = [&]() -> bool {
                if (j > 0 && !__all_sync(0xffffffffu, mbar_wait(&o_done[t], (j - 1) & 1, abort_flag))) return false;
                // tcgen05.ld/st are warp-collective: rescale the whole warp's rows if any needs it
                if (__any_sync(0xffffffffu, rescale)) {
                    tc_fence_after();
#pragma unroll 1
                    for (int cc = 0; cc < 4; ++cc) {
                        uint32_t o[32];
                        tmem_ld32(o_addr + cc * 32, o);
                        tmem_ld_wait();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(o_addr + cc * 32, o);
                    }
                    tmem_st_wait();
                }
                return true;
            };
            // P_t(j): this thread's row, keys [64 hf + 8 q, +8) in 16-byte chunk q of half hf
            auto store_p = [&](int hf) {
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    st_shared_v4(p_tile + hf * HALF + swz(row, q), w[32 * hf + 4 * q], w[32 * hf + 4 * q + 1],
                                 w[32 * hf + 4 * q + 2], w[32 * hf + 4 * q + 3]);
            };
#pragma unroll
            for (int g = 0; g < SUM_GROUPS; ++g) {
                uint64_t rs0 = pk2(0.f, 0.f), rs1 = pk2(0.f, 0.f);
#pragma unroll
                for (int ii = 0; ii < GROUP_PAIRS; ++ii) {
                    const int i = g * GROUP_PAIRS + ii;
                    float x0, x1;   // s * c - m for a key pair, one packed FMA
                    up2(ffma2(pk2(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])), c2, nm2), x0, x1);
                    float p0, p1;
                    if (full && (i & 7) < POLY_PAIRS) {
                        exp2_poly2(x0, x1, p0, p1);
                    } else {
                        p0 = ex2(x0);
                        p1 = ex2(x1);
                    }
                    if (ii & 1) rs1 = fadd2(rs1, pk2(p0, p1));
                    else rs0 = fadd2(rs0, pk2(p0, p1));
                    w[i] = pack_bf16x2(p0, p1);
                }
                float r0, r1, r2, r3;
                up2(rs0, r0, r1);
                up2(rs1, r2, r3);
                l[g] = l[g] * alpha + ((r0 + r1) + (r2 + r3));
#if H3_ATTN_EARLY_P
                static_assert(SUM_GROUPS == 2, "early P stores go by 64-key halves");
                if (g == 0 && !(ok = release_p_tile())) break;
                store_p(g);
#endif
            }
            if (!ok) break;
#if !H3_ATTN_EARLY_P
            ok = release_p_tile();
            if (!ok) break;
            store_p(0);
            store_p(1);
#endif
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&p_ready[t]);
        }
        if (ok) ok = mbar_wait(&o_done[t], (nkv - 1) & 1, abort_flag);
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
            tc_fence_after();
            float lsum = l[0];   // the groups' running sums, in group order
#pragma unroll
            for (int g = 1; g < SUM_GROUPS; ++g) lsum += l[g];
            const float inv = 1.0f / lsum;
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
            if (p.ndst > 0) {
                // row stores to each row's owner: 16 threads per 256-byte row, 8 rows
                // per pass of the warpgroup (two whole rows per warp instruction)
                named_bar_sync(1 + t, 128);
                const int c = row & 15;
                const uint32_t tile = out_tile + (uint32_t)(c >> 3) * HALF;
#pragma unroll 4
                for (int k = 0; k < BM / 8; ++k) {
                    const int rr = (row >> 4) + 8 * k;
                    const int g = q0 + t * BM + rr;
                    if (g >= p.Sq) break;   // rows grow with k
                    const int dq = g / p.rows_per_dst;
                    const int tl = g - dq * p.rows_per_dst;
                    const uint4 v = ld_shared_v4(tile + swz(rr, c & 7));
                    st_global_v4(p.dst[dq] + (int64_t)tl * p.d_row + (int64_t)h * p.d_head + 8 * c, v);
                }
            } else {
                fence_proxy_async_smem();
                named_bar_sync(1 + t, 128);
                if (row == 0 && q0 + t * BM < p.Sq) {
                    tma_store_4d(&to, sQ + t * TILE, 0, q0 + t * BM, h, b);
                    tma_store_4d(&to, sQ + t * TILE + HALF, 64, q0 + t * BM, h, b);
                    tma_store_commit();
                    tma_store_wait_all();
                }
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

// CTA -> (batch, head, first Q row, Q tiles): CTAs [0, split_from) own a pair of Q
// tiles, the grid's last pairs run as two one-tile CTAs each.  Each kind runs its
// own compile-time specialisation of the same tile code (the pair path carries no
// run-time tile count), and a tile's arithmetic is the same in both.
__global__ void __launch_bounds__(THREADS, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to, Params p) {
    const int cta = (int)blockIdx.x;
    const bool single = cta >= p.split_from;
    int pair = cta, tile0 = 0;
    if (single) {
        pair = p.split_from + ((cta - p.split_from) >> 1);
        tile0 = (cta - p.split_from) & 1;
    }
    const int hb = pair / p.pairs;
    const int h = hb % p.H, b = hb / p.H;
    tile0 += (pair - hb * p.pairs) * NQ;
    const int left = p.tiles - tile0;   // Q tiles of this head from tile0 on
    if (left <= 0) return;              // second half of a split pair past Sq (uniform over the CTA)
    if (!single && left >= NQ) fa_cta<NQ>(tq, tk, tv, to, p, h, b, tile0 * BM);
    else fa_cta<1>(tq, tk, tv, to, p, h, b, tile0 * BM);
}

}  // namespace attn
}  // namespace h3

using namespace h3;

namespace {

// [B, S, H, 128] BF16 view -> 4-D tensor map (D, S, H, B), box (64, rows, 1, 1)
int attn_tmap(CUtensorMap *map, const h3_tensor *t, unsigned rows) {
    const cuuint64_t dims[4] = {(cuuint64_t)t->shape[3], (cuuint64_t)t->shape[1], (cuuint64_t)t->shape[2],
                                (cuuint64_t)t->shape[0]};
    // a size-1 batch dim may carry any stride; give TMA a legal one
    const int64_t sb = t->shape[0] == 1 ? t->strides[1] * t->shape[1] : t->strides[0];
    const int64_t sh = t->shape[2] == 1 ? 128 : t->strides[2];
    const cuuint64_t strides[3] = {(cuuint64_t)t->strides[1] * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
    const cuuint32_t box[4] = {64, rows, 1, 1};
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

namespace {

// Shared launcher: `out` is the output view, or null with p.ndst > 0 (scatter).
int launch_mha(const h3_tensor *out, const h3_tensor *q, const h3_tensor *k, const h3_tensor *v, float scale,
               attn::Params &p, cudaStream_t stream) {
    H3_CHECK(check_attn_operand(q));
    H3_CHECK(check_attn_operand(k));
    H3_CHECK(check_attn_operand(v));
    if (out) {
        H3_CHECK(check_attn_operand(out));
        H3_CHECK(check_same_shape(out, q));
    }
    H3_CHECK(check_same_shape(k, v));
    if (q->shape[0] != k->shape[0] || q->shape[2] != k->shape[2]) return H3_ERR_BAD_SHAPE;
    const int B = (int)q->shape[0], Sq = (int)q->shape[1], H = (int)q->shape[2], Sk = (int)k->shape[1];
    if (B == 0 || Sq == 0 || H == 0) return H3_OK;
    if (Sk == 0) return H3_ERR_BAD_SHAPE;
    CUtensorMap tq, tk, tv, to;
    H3_CHECK(attn_tmap(&tq, q, attn::BM));
    H3_CHECK(attn_tmap(&tk, k, attn::BN));
    H3_CHECK(attn_tmap(&tv, v, attn::BN));
    if (out) H3_CHECK(attn_tmap(&to, out, attn::BM));
    else to = tq;   // unused by the scatter epilogue
    p.Sq = Sq;
    p.Sk = Sk;
    p.H = H;
    p.B = B;
    p.nkv = (Sk + attn::BN - 1) / attn::BN;
    p.scale_log2 = scale * 1.4426950408889634f;
    static std::atomic<bool> attr_set[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return H3_ERR_UNSUPPORTED;
    if (!attr_set[dev].load()) {
        if (attn::SOFTMAX_REGS > 0) {
            // the register split must fit in what the CTA is launched with
            cudaFuncAttributes fa{};
            if (cudaFuncGetAttributes(&fa, attn::fa_fwd_kernel) != cudaSuccess) return H3_ERR_LAUNCH;
            if ((int64_t)fa.numRegs * attn::THREADS < attn::CTRL_REGS * 128 + 2 * attn::SOFTMAX_REGS * 128)
                return H3_ERR_UNSUPPORTED;
        }
        if (cudaFuncSetAttribute(attn::fa_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 attn::SMEM_BYTES) != cudaSuccess)
            return H3_ERR_LAUNCH;
        attr_set[dev].store(true);
    }
    const int sms = num_sms();
    p.tiles = (Sq + attn::BM - 1) / attn::BM;
    p.pairs = (p.tiles + attn::NQ - 1) / attn::NQ;
    const int64_t npairs = (int64_t)p.pairs * H * B;
    // one CTA per SM: a last wave of r <= SMs/2 pairs finishes sooner as 2r one-tile CTAs
    // (one per SM; measured alone, a one-tile CTA takes about 0.7 of a pair's time)
    const int64_t r = npairs % sms;
    const int64_t split = (H3_ATTN_SPLIT_TAIL && r > 0 && 2 * r <= sms) ? r : 0;
    const int64_t ctas = npairs + split;
    if (ctas > (int64_t)0x7fffffff) return H3_ERR_UNSUPPORTED;
    p.split_from = (int)(npairs - split);
    attn::fa_fwd_kernel<<<(unsigned)ctas, attn::THREADS, attn::SMEM_BYTES, stream>>>(tq, tk, tv, to, p);
    return launch_status();
}

}  // namespace

extern "C" int h3_mha(const h3_tensor *out, const h3_tensor *q, const h3_tensor *k, const h3_tensor *v, float scale,
                      void *stream) {
    if (!out) return H3_ERR_NULL;
    attn::Params p{};
    return launch_mha(out, q, k, v, scale, p, (cudaStream_t)stream);
}

extern "C" int h3_mha_scatter(const h3_tensor *dsts, int32_t ndst, const h3_tensor *q, const h3_tensor *k,
                              const h3_tensor *v, float scale, void *stream) {
    if (!dsts) return H3_ERR_NULL;
    if (ndst < 1 || ndst > H3_EXCHANGE_MAX_RANKS) return H3_ERR_BAD_SHAPE;
    H3_CHECK(check_attn_operand(q));
    if (q->shape[0] != 1) return H3_ERR_UNSUPPORTED;   // one sequence (the Ulysses layout)
    const h3_tensor *d0 = &dsts[0];
    attn::Params p{};
    for (int i = 0; i < ndst; ++i) {
        const h3_tensor *d = &dsts[i];
        H3_CHECK(check_bf16(d));
        if (d->ndim != 3 || d->shape[0] != d0->shape[0] || d->shape[1] != q->shape[2] || d->shape[2] != 128)
            return H3_ERR_BAD_SHAPE;
        if (d->strides[0] != d0->strides[0] || d->strides[1] != d0->strides[1] || d->strides[2] != 1 ||
            !aligned16(d->data) || d->strides[0] % 8 != 0 || d->strides[1] % 8 != 0)
            return H3_ERR_BAD_LAYOUT;
        p.dst[i] = static_cast<__nv_bfloat16 *>(d->data);
    }
    if (d0->shape[0] * ndst < q->shape[1] || d0->shape[0] > 0x7fffffffLL) return H3_ERR_BAD_SHAPE;
    if (d0->shape[0] == 0) return q->shape[1] == 0 ? H3_OK : H3_ERR_BAD_SHAPE;
    p.ndst = ndst;
    p.rows_per_dst = (int)d0->shape[0];
    p.d_row = d0->strides[0];
    p.d_head = d0->strides[1];
    return launch_mha(nullptr, q, k, v, scale, p, (cudaStream_t)stream);
}

// device error word of this translation unit (bounded waits in the attention kernel)
extern "C" unsigned int h3_attention_device_error_read_and_clear(void) {
    unsigned int v = 0, zero = 0;
    cudaMemcpyFromSymbol(&v, h3::g_h3_device_error, sizeof(v));
    cudaMemcpyToSymbol(h3::g_h3_device_error, &zero, sizeof(zero));
    return v;
}
