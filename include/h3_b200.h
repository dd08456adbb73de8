/*
 * h3_b200.h -- C-ABI of the B200 (sm_100a) MiniMax-H3 DiT-block hot path.
 *
 * Every entry point takes plain descriptors (pointer + shape + element strides),
 * launches on the caller's CUDA stream and returns an h3_status.  Callers own
 * every buffer; no entry point allocates device memory.  Validation mirrors the
 * reference op wrappers (shape/dtype checks that throw std::invalid_argument
 * there return H3_ERR_BAD_SHAPE / H3_ERR_BAD_DTYPE here), except that widths
 * are parameters instead of the reference's hard-coded 128/5376.
 *
 * Reference interfaces replaced (file:line inside the reference tree):
 *   h3_rms_norm                    InfiniCore.patch:160 (h3_numerics.hpp), checks :891-900
 *   h3_swiglu                      InfiniCore.patch:161, checks :909-917
 *   h3_rms_modulate                InfiniCore.patch:162, checks :928-939
 *   h3_rope                        InfiniCore.patch:164, checks :948-958
 *   h3_gated_residual              InfiniCore.patch:165, checks :963-979
 *   h3_gated_residual_rms_modulate InfiniCore.patch:179-181, checks :992-1004
 *   h3_qk_norm_rope                InfiniCore.patch:169-170 (h3_qk_norm_rope_), checks :1015-1024
 *   h3_rope_cache                  InfiniCore.patch:173, checks :1033-1041
 *   h3_mha                         InfiniCore.patch:1333-1426 (mha_ninetoothed.cc plan/run)
 *   h3_timestep_embedding          InfiniCore.patch:223-252 (infiniopTimestepEmbedding C API)
 *   h3_linear*                     InfiniCore.patch:1231-1292 (linear.cc) + the fused
 *                                  epilogues of InfiniLM.patch:1172-1179, 1377-1394
 *   h3_adaln_projection            InfiniLM.patch:1260-1279 (AdaLN projection linear + bias)
 *   h3_linear_f32                  linear_forward on the F32 modules (proj_in, audio_proj_in,
 *                                  proj_out, audio_proj_out, time embedder),
 *                                  InfiniLM.patch:1501-1517, 1662-1664, 1812-1814
 *   h3_gather_rows                 gather_rows -> op::embedding, InfiniLM.patch:587-590
 *   h3_index_copy_rows             op::index_copy of the packed sequence, InfiniLM.patch:1685-1690
 *   h3_silu                        op::silu + cast_to, InfiniLM.patch:1267-1268, 1511, 1535
 *   h3_ipc_* , h3_exchange_*       the Ulysses all-to-alls all_to_all_[on_stream_]
 *                                  (InfiniCore.patch:526-577) as used by gather_sequence /
 *                                  scatter_sequence (InfiniLM.patch:895-910, 1127-1137): peer
 *                                  receive buffers + epoch flags instead of a collective
 */
#ifndef H3_B200_H
#define H3_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define H3_ABI_VERSION 1
#define H3_MAX_DIMS 4
#define H3_EXCHANGE_MAX_RANKS 8
#define H3_EXCHANGE_SLOTS 4
#define H3_MAX_SEGMENTS 4   /* modulation segments one *_segmented launch can take */
#define H3_IPC_HANDLE_BYTES 64

typedef enum h3_dtype {
    H3_BF16 = 0,
    H3_F32 = 1,
    H3_F64 = 2,
    H3_I64 = 3
} h3_dtype;

typedef enum h3_status {
    H3_OK = 0,
    H3_ERR_NULL = 1,          /* a required descriptor or data pointer is null   */
    H3_ERR_BAD_SHAPE = 2,     /* shapes do not match the op's contract           */
    H3_ERR_BAD_DTYPE = 3,     /* unsupported element type                        */
    H3_ERR_BAD_LAYOUT = 4,    /* strides/alignment the op cannot address         */
    H3_ERR_UNSUPPORTED = 5,   /* valid request outside what this build supports  */
    H3_ERR_LAUNCH = 6,        /* the CUDA launch reported an error               */
    H3_ERR_DRIVER = 7,        /* a driver entry point could not be resolved      */
    H3_ERR_TIMEOUT = 8,       /* a bounded device-side wait gave up              */
    H3_ERR_INDEX = 9,         /* a row index was outside the indexed tensor      */
    H3_ERR_TOO_LARGE = 10     /* request exceeds the library's static scratch    */
} h3_status;

/* A strided view.  strides are in ELEMENTS (not bytes); stride 0 broadcasts.
 * Dimensions past ndim are ignored. */
typedef struct h3_tensor {
    void *data;
    int64_t shape[H3_MAX_DIMS];
    int64_t strides[H3_MAX_DIMS];
    int32_t ndim;
    int32_t dtype; /* h3_dtype */
} h3_tensor;

int h3_abi_version(void);
const char *h3_status_string(int status);

/* Synchronises the current device and reports (then clears) whether any bounded
 * device-side wait gave up since the last call (H3_ERR_TIMEOUT), else whether a
 * row gather/scatter met an index outside its table (H3_ERR_INDEX; that row was
 * left untouched), H3_ERR_LAUNCH if the device reports an error, else H3_OK.
 * No reference counterpart (the reference's waits are unbounded). */
int h3_device_error(void);

/* Failure-detection self test: launches one CTA that waits, with a limit of
 * limit_ns (at most 1 s), on a barrier nothing arrives at.  The wait gives up,
 * the kernel ends normally, and the next h3_device_error() returns
 * H3_ERR_TIMEOUT.  No fault, trap or hang is involved.  No reference counterpart. */
int h3_selftest_wait_timeout(uint64_t limit_ns, void *stream);

/* Tile form of the projections (every h3_linear* entry point): 0 = chosen per
 * launch (CTA-pair 256-row tiles unless they pad M by more than 1/64 over
 * 128-row tiles), 1 = single-CTA 128-row tiles, 2 = CTA-pair tiles.  Both forms
 * give bitwise the same results.  Returns the previous setting, or -1 for a
 * value outside 0..2 (setting unchanged).  A tuning and test hook; no reference
 * counterpart. */
int h3_gemm_variant(int variant);

/* ---------------- fused pointwise ops (BF16, reference rounding) ---------------- */

/* y = staged-BF16 RMSNorm(x) * weight over the last axis.  x, y [S,C] or [B,S,C]; weight [C]. */
int h3_rms_norm(const h3_tensor *y, const h3_tensor *x, const h3_tensor *weight, float eps,
                void *stream);

/* y = bf16(up * bf16(gate / (1 + exp(-gate)))).  up, gate, y same shape, 2-D or 3-D. */
int h3_swiglu(const h3_tensor *y, const h3_tensor *up, const h3_tensor *gate, void *stream);

/* y = bf16(bf16(rms_norm(x, weight) * bf16(1 + scale)) + shift).  scale/shift have
 * x's shape (stride 0 broadcasts a modulation row over tokens). */
int h3_rms_modulate(const h3_tensor *y, const h3_tensor *x, const h3_tensor *weight,
                    const h3_tensor *scale, const h3_tensor *shift, float eps, void *stream);

/* LayerNorm (mean-subtracted, no affine, fp32 statistics, one BF16 rounding)
 * followed by the same modulate.  Builder extension, no reference counterpart. */
int h3_ln_modulate(const h3_tensor *y, const h3_tensor *x, const h3_tensor *scale,
                   const h3_tensor *shift, float eps, void *stream);

/* out = bf16(x + bf16(gate * y)); gate may broadcast (stride 0). */
int h3_gated_residual(const h3_tensor *out, const h3_tensor *x, const h3_tensor *gate,
                      const h3_tensor *y, void *stream);

/* residual = bf16(x + bf16(gate * y)); out = h3_rms_modulate(residual, ...). */
int h3_gated_residual_rms_modulate(const h3_tensor *residual, const h3_tensor *out,
                                   const h3_tensor *x, const h3_tensor *gate, const h3_tensor *y,
                                   const h3_tensor *weight, const h3_tensor *scale,
                                   const h3_tensor *shift, float eps, void *stream);

/* NeoX RoPE of x [S,H,128] with token-ordered angles cos/sin [S,half] (half = 48 in
 * the reference layout, 64 for the full-D 44/42/42 layout): pairs (i, i+half) for
 * i < half rotate, channels [2*half, 128) pass through. */
int h3_rope(const h3_tensor *y, const h3_tensor *x, const h3_tensor *cos, const h3_tensor *sin,
            void *stream);

/* Per-head staged RMSNorm (weight [128]) then RoPE of x [T,P,Hs,128] (any strides)
 * written to out [T,P,Hs,128] (any strides -- e.g. the permuted view of an
 * all-to-all send buffer [P,T,Hs,128]).  cos/sin [T,half]. */
int h3_qk_norm_rope(const h3_tensor *out, const h3_tensor *x, const h3_tensor *weight,
                    const h3_tensor *cos, const h3_tensor *sin, float eps, void *stream);

/* RoPE table: out [T,96] BF16 = cat(cos, sin) of angle[t, 16a+k] =
 * f32(position[t,a]) * (1 / power[k]); position [T,3] F64, power [16] F32. */
int h3_rope_cache(const h3_tensor *out, const h3_tensor *position, const h3_tensor *power,
                  void *stream);

/* Sectioned generalisation: sections (f0,f1,f2) frequencies per axis, power
 * [f0+f1+f2] F32 (axis-major), out [T, 2*(f0+f1+f2)].  (16,16,16) with the 16
 * powers repeated reproduces h3_rope_cache. */
int h3_rope_cache_sectioned(const h3_tensor *out, const h3_tensor *position,
                            const h3_tensor *power, int32_t f0, int32_t f1, int32_t f2,
                            void *stream);

/* out [N,dim] F32: cos(t*f_k) for k < dim/2 then sin(t*f_k), f_k = exp(-ln(max_period)*k/(dim/2)).
 * t [N] F32. */
int h3_timestep_embedding(const h3_tensor *out, const h3_tensor *t, float max_period, void *stream);

/* ---------------- attention ---------------- */

/* Non-causal softmax(q k^T * scale) v.  q, out [B,Sq,H,128]; k, v [B,Sk,H,128]
 * (Sk may be shorter than Sq: sequence-parallel padding).  Strides arbitrary
 * with innermost stride 1 and 16-byte aligned rows.  fp32 softmax/accumulate. */
int h3_mha(const h3_tensor *out, const h3_tensor *q, const h3_tensor *k, const h3_tensor *v,
           float scale, void *stream);

/* h3_mha for one sequence (q [1,Sq,Hl,128]) whose output rows are stored straight
 * to their owners: row g of head h goes to dsts[g / R] row g % R, head slot h, where
 * dsts is an array of ndst descriptors [R, Hl, 128] (same strides, 16-byte aligned
 * rows; typically this rank's head slice of every rank's return buffer, mapped from
 * the peers) and ndst * R >= Sq.  The Ulysses heads -> tokens all-to-all of
 * attend_exchanged_groups / scatter_sequence (InfiniLM.patch:1006-1014, 1127-1137)
 * done by the attention kernel's own epilogue.  Arithmetic identical to h3_mha. */
int h3_mha_scatter(const h3_tensor *dsts, int32_t ndst, const h3_tensor *q, const h3_tensor *k,
                   const h3_tensor *v, float scale, void *stream);

/* ---------------- projections (BF16 in/out, fp32 accumulate) ---------------- */

/* y [M,N] = x [M,K] * w[N,K]^T.  Rows of x, w, y contiguous (inner stride 1),
 * row strides multiples of 8 elements, K a multiple of 64. */
int h3_linear(const h3_tensor *y, const h3_tensor *x, const h3_tensor *w, void *stream);

/* y [M,F] = swiglu(up, gate) with [up|gate] = x * w_packed^T, where w_packed is
 * h3_pack_gate_up() of the [up; gate] weight [2F,K].  F a multiple of 128. */
int h3_linear_swiglu(const h3_tensor *y, const h3_tensor *x, const h3_tensor *w_packed,
                     void *stream);

/* out [M,N] = bf16(residual + bf16(gate * bf16(x * w^T))); gate [M,N] (stride 0 ok). */
int h3_linear_gated_residual(const h3_tensor *out, const h3_tensor *x, const h3_tensor *w,
                             const h3_tensor *residual, const h3_tensor *gate, void *stream);

/* h3_linear_gated_residual, plus the row sums of squares of out in per-tile pieces:
 * sq [M, ceil(N/256)] F32, sq[i][n] = fp32 sum over columns [256n, 256n+256) of
 * bf16(out[i][c]^2), added in column order.  The out-projection + residual half of
 * the block's post-attention step (to_out.0 then h3_gated_residual_rms_modulate,
 * InfiniLM.patch:866, 1377-1390; op checks InfiniCore.patch:992-1004). */
int h3_linear_gated_residual_sq(const h3_tensor *out, const h3_tensor *sq, const h3_tensor *x,
                                const h3_tensor *w, const h3_tensor *residual, const h3_tensor *gate,
                                void *stream);

/* h3_rms_modulate with the row's sum of squares read from sq [rows, ceil(C/256)] F32
 * (as h3_linear_gated_residual_sq writes it) instead of recomputed: total = lane l of
 * a warp sums sq[l], sq[l+32], ... in order, then an xor-16/8/4/2/1 tree; then the
 * staged mean / eps / rsqrt / normalise / weight / modulate roundings of
 * h3_rms_modulate.  Element-wise (no row in registers).  Rows 16-byte aligned with
 * inner stride 1 (H3_ERR_BAD_LAYOUT otherwise).  The norm half of
 * h3_gated_residual_rms_modulate (InfiniCore.patch:179-181, 992-1004). */
int h3_rms_modulate_sq(const h3_tensor *y, const h3_tensor *x, const h3_tensor *sq, const h3_tensor *weight,
                       const h3_tensor *scale, const h3_tensor *shift, float eps, void *stream);

/* Per-segment forms, one launch for all of a rank's modulation segments (the block's
 * segmented application of the AdaLN rows, forward_segmented InfiniLM.patch:1353-1397,
 * MiniMaxH3ModulationSegment :2041-2045): rows are split into nseg <= H3_MAX_SEGMENTS
 * consecutive segments of seg_rows[s] rows (summing to M); segment s uses the
 * contiguous [N] row gates[s] (resp. scales[s], shifts[s]).  Arithmetic per row is that
 * of the single-segment entry points, so the result equals one launch per segment bit
 * for bit.  sq may be NULL: then h3_linear_gated_residual_segmented writes no partial
 * sums and h3_rms_modulate_segmented reduces the row itself (as h3_rms_modulate). */
int h3_linear_gated_residual_segmented(const h3_tensor *out, const h3_tensor *sq, const h3_tensor *x,
                                       const h3_tensor *w, const h3_tensor *residual, const h3_tensor *gates,
                                       const int64_t *seg_rows, int32_t nseg, void *stream);
int h3_rms_modulate_segmented(const h3_tensor *y, const h3_tensor *x, const h3_tensor *sq,
                              const h3_tensor *weight, const h3_tensor *scales, const h3_tensor *shifts,
                              const int64_t *seg_rows, int32_t nseg, float eps, void *stream);

/* The out-projection fused with h3_gated_residual_rms_modulate (InfiniLM.patch:866 then
 * :1377-1390): residual_out = bf16(residual + bf16(gate * bf16(x w^T))) and
 * out = RMSNorm + AdaLN of residual_out, with the sums of squares passed through
 * `workspace` [M, ceil(N/256)] F32 (caller-owned scratch: the two launches of
 * h3_linear_gated_residual_sq and h3_rms_modulate_sq). */
int h3_linear_gated_residual_rms_modulate(const h3_tensor *residual_out, const h3_tensor *out,
                                          const h3_tensor *x, const h3_tensor *w, const h3_tensor *residual,
                                          const h3_tensor *gate, const h3_tensor *weight,
                                          const h3_tensor *scale, const h3_tensor *shift, float eps,
                                          const h3_tensor *workspace, void *stream);

/* Capacity, in floats, of the scratch array behind the _noalloc entry point below
 * (4 MiB of device memory on every GPU that loads the library, held until exit). */
#define H3_NOALLOC_SQ_FLOATS (1 << 20)

/* h3_linear_gated_residual_rms_modulate without the workspace argument, for callers
 * that cannot allocate device memory where they call it: a host framework that owns
 * every device allocation through its own planned pool, or a plugin boundary whose
 * host side has no device allocator.  The per-tile sums of squares go to a fixed
 * array in the library's device image instead (H3_NOALLOC_SQ_FLOATS floats), so a
 * call needs M * ceil(N / 256) <= H3_NOALLOC_SQ_FLOATS (M = rows of residual_out,
 * N = rows of w: up to 52428 tokens at width 5120); larger requests return
 * H3_ERR_TOO_LARGE and launch nothing.  Allocates nothing and frees nothing.  The
 * first call on a device looks up the array's device address with that device
 * current; make that first call before any stream capture.  Every call shares the
 * one array (each call writes every entry it reads, so leftovers of an earlier call
 * do not matter), hence calls that can overlap on the GPU -- concurrent streams, or
 * several host threads on one device -- race; serialise them.  No counterpart in the
 * reference (its op wrappers allocate their outputs and need no scratch). */
int h3_linear_gated_residual_rms_modulate_noalloc(const h3_tensor *residual_out, const h3_tensor *out,
                                                  const h3_tensor *x, const h3_tensor *w,
                                                  const h3_tensor *residual, const h3_tensor *gate,
                                                  const h3_tensor *weight, const h3_tensor *scale,
                                                  const h3_tensor *shift, float eps, void *stream);

/* QKV projection with the q/k RMSNorm + RoPE of h3_qk_norm_rope applied in the GEMM
 * epilogue, each head row stored straight to its destination: x [T,K], w [3*H*128, K]
 * (rows [q | k | v], head-major), q_dsts / k_dsts / v_dsts arrays of ndst descriptors
 * [T, hpd, 128] (same strides; H = ndst * hpd, H even), head h to destination
 * h / hpd, slot h % hpd.  Destinations may be peers' receive buffers (the Ulysses
 * send).  cos/sin [T, half], half = 48 (reference layout) or 64 (full-D 44/42/42 layout).
 * Equal bit for bit to h3_linear followed by h3_qk_norm_rope. */
int h3_linear_qkv_norm_rope(const h3_tensor *x, const h3_tensor *w, const h3_tensor *q_dsts,
                            const h3_tensor *k_dsts, const h3_tensor *v_dsts, int32_t ndst,
                            const h3_tensor *norm_q, const h3_tensor *norm_k, const h3_tensor *cos,
                            const h3_tensor *sin, float eps, void *stream);

/* Reorder the [up; gate] rows of a gate_up weight [2F,K] into 128-row blocks
 * [up_0 | gate_0 | up_1 | gate_1 ...] consumed by h3_linear_swiglu. */
int h3_pack_gate_up(const h3_tensor *dst, const h3_tensor *src, void *stream);

/* AdaLN projection of the blocks' conditioning (MiniMaxH3AdaLNProjection::forward,
 * InfiniLM.patch:1260-1279, its linear + bias): y [M,N] = bf16(bf16(x w^T) + bias)
 * for M <= 4 rows of x [M,K] against w [N,K], all BF16; bias [N] may be NULL.  A
 * weight-streaming kernel with fp32 accumulation (fixed order: each lane's 16-byte
 * chunks in order, then a xor tree over the warp), so a column slice of w gives
 * bitwise the same columns.  K a multiple of 8, rows 16-byte aligned. */
int h3_adaln_projection(const h3_tensor *y, const h3_tensor *x, const h3_tensor *w, const h3_tensor *bias,
                        void *stream);

/* ---------------- model wrapper ops (outside the block loop) ---------------- */

/* y [M,N] = x [M,K] * w[N,K]^T (+ bias[N]); x BF16 or F32 (BF16 is widened
 * exactly, as cast_to F32 does), w and bias F32, fp32 accumulation in k order;
 * y F32, or BF16 rounded once from the fp32 result (cast_to after the F32
 * linear).  bias may be NULL.  Rows contiguous (inner stride 1). */
int h3_linear_f32(const h3_tensor *y, const h3_tensor *x, const h3_tensor *w, const h3_tensor *bias,
                  void *stream);

/* out [n,C] = table[indices[r], :]; table [T,C]; BF16 or F32; indices [n] I64.
 * An index outside [0,T) leaves its row untouched; h3_device_error() then
 * returns H3_ERR_INDEX. */
int h3_gather_rows(const h3_tensor *out, const h3_tensor *table, const h3_tensor *indices, void *stream);

/* out[indices[r], :] = src[r, :]; out [T,C], src [n,C]; BF16 or F32; indices
 * [n] I64, distinct (as for index_copy, repeated indices race).  Out-of-range
 * indices as for h3_gather_rows. */
int h3_index_copy_rows(const h3_tensor *out, const h3_tensor *indices, const h3_tensor *src, void *stream);

/* y = x / (1 + exp(-x)) computed in fp32 from x F32; y F32 or BF16 (rounded
 * once).  Contiguous. */
int h3_silu(const h3_tensor *y, const h3_tensor *x, void *stream);

/* ---------------- peer-memory exchange (sequence parallelism) ---------------- */

/* The q/k RMSNorm + RoPE of h3_qk_norm_rope for every destination block in one
 * launch: x [T, n, Hs, 128] (the head blocks of the QKV output), outs[p] (an
 * array of n descriptors, each [T, Hs, 128], same strides; typically slot r of
 * rank p's receive buffer, mapped from a peer) receives block p.  n <= 8. */
int h3_qk_norm_rope_multi(const h3_tensor *outs, int32_t n, const h3_tensor *x, const h3_tensor *weight,
                          const h3_tensor *cos, const h3_tensor *sin, float eps, void *stream);

/* dsts[b] [R, C] = src[b] for the n blocks of src [n, R, C] (strided, inner stride 1),
 * BF16 or F32, one launch; n <= 8.  The v and attention-output legs of the exchange. */
int h3_copy_blocks(const h3_tensor *dsts, int32_t n, const h3_tensor *src, void *stream);

/* The all-reduce step of the tensor-parallel block for the n ranks' rows this rank
 * owns: every dsts[i] [R, C] BF16 (rank i's sum buffer rows, mapped here)
 * receives bf16(sum over p = 0..n-1 of srcs[p]) (rank p's partial rows), summed
 * in fp32 in rank order.  Rows 16-byte aligned, C a multiple of 8.  Replaces the
 * reference's allreduce_on_stream_ after the row-parallel projections
 * (InfiniLM.patch:1432-1436, 1455-1459). */
int h3_peer_reduce_rows(const h3_tensor *dsts, const h3_tensor *srcs, int32_t n, void *stream);

/* Persistent buffers a peer process can map: cudaMalloc of `bytes` (zeroed) and
 * its CUDA IPC handle (H3_IPC_HANDLE_BYTES bytes written to `handle`).  Allocated
 * once at set-up, freed with h3_ipc_free; no other entry point allocates. */
int h3_ipc_alloc(uint64_t bytes, void **ptr, void *handle);
/* Map a peer's buffer from its handle (peer access enabled lazily); unmap with h3_ipc_close. */
int h3_ipc_open(const void *handle, void **ptr);
int h3_ipc_close(void *ptr);
int h3_ipc_free(void *ptr);

/* After the kernels that stored this rank's blocks into the peers' receive buffers
 * (earlier on `stream`): increment this rank's epoch[slot] and write the new value
 * into flags[slot][rank] of every peer.  peer_flags[p] is rank p's flag array
 * (uint64 [H3_EXCHANGE_SLOTS][H3_EXCHANGE_MAX_RANKS]) as mapped in this process
 * (own entry: the local array). */
int h3_exchange_signal(void *const *peer_flags, uint64_t *epoch, int32_t slot, int32_t rank, int32_t world,
                       void *stream);

/* Wait (on the device, bounded by timeout_ns) until every peer's flags[slot][q]
 * has reached this rank's epoch[slot]; later work on `stream` then sees the
 * peers' data.  A wait that gives up ends the kernel normally and
 * h3_device_error() returns H3_ERR_TIMEOUT. */
int h3_exchange_wait(const void *flags, const uint64_t *epoch, int32_t slot, int32_t rank, int32_t world,
                     uint64_t timeout_ns, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* H3_B200_H */
