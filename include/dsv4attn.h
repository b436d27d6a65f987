/*
 * dsv4attn.h - C ABI of the B200 (sm_100a) DeepSeek-V4-Flash decode
 * sparse-attention path.
 *
 * Every entry point takes raw device pointers, element counts / strides and
 * a CUDA stream, launches asynchronously on that stream and returns a
 * status code (DSA_OK = 0, negative on error).  No entry point allocates
 * device memory, synchronises the device or copies to or from the host:
 * all buffers are owned by the caller, so every call can be captured in a
 * CUDA graph.  Argument errors are detected on the host before any launch;
 * dsa_last_error() returns a message for the calling thread.
 *
 * Each function names the reference interface it replaces
 * (zoecarver/tt-deepseek-v4, file:line).  Tensor layouts are row-major;
 * "bf16" is IEEE bfloat16, "e4m3" is OCP FP8 E4M3 (float8_e4m3fn).
 */
#ifndef DSV4ATTN_H
#define DSV4ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct CUstream_st;
typedef struct CUstream_st* dsa_stream_t; /* == cudaStream_t */

enum {
  DSA_OK = 0,
  DSA_ERR_ARG = -1,         /* bad shape / stride / alignment / null pointer */
  DSA_ERR_CUDA = -2,        /* a CUDA launch or runtime call failed          */
  DSA_ERR_UNSUPPORTED = -3, /* shape outside what the kernels are built for */
  DSA_ERR_TIMEOUT = -4,     /* a bounded device-side wait expired            */
  DSA_ERR_WORKSPACE = -5    /* caller-provided workspace too small           */
};

/* Library version (major*10000 + minor*100 + patch) and the last error
 * message recorded on the calling host thread ("" if none). */
int dsa_version(void);
const char* dsa_last_error(void);

/* Spin budget of every bounded device-side wait in this library (mbarrier
 * waits of the attention and indexer kernels, grid barriers of the wide
 * top-k, peer flags of dsa_p2p_wait), in SM clock cycles; cycles <= 0
 * restores the default of 2e9 (about one second).  A wait that runs out
 * sets bit 2 of the call's status word (where it has one) and the kernel
 * ends instead of hanging, so the context stays usable.  Read at each launch
 * (host-side, process-wide); kernels already captured in a CUDA graph keep
 * the value of their capture.  No counterpart in the reference (its device
 * waits are inside ttnn). */
int dsa_set_wait_limit(long long cycles);
long long dsa_get_wait_limit(void);

/* ------------------------------------------------ projections around the path */

/* Y[b, g*N + n] = bf16(sum_k X[b, g*K + k] W[g*N + n, k]) for b < B, n < N,
 * g < G: the decode-step projections as one weight-streaming tcgen05 kernel.
 * X [B, ld_x] bf16 (row stride ld_x >= G*K, a multiple of 8, 16-byte
 * aligned), K a multiple of 64; w_packed = W [G*N, K] in the tile layout of
 * dsa_linear_pack (16-byte aligned).
 * Y [B, ld_y]: bf16, or with out_f32 the fp32 value of the bf16 result.
 * rope_dim > 0: interleaved rotary (pairs 2i, 2i+1) on the last rope_dim
 * columns of every head_dim block of columns [rope_col0, N) of each group of
 * Y (rope_col0 = 0: all of it; > 0: two projections of one input stored as
 * one weight, the second rotated), applied to the bf16 product with cos/sin
 * [n_pos, rope_dim/2] fp32 at position pos[b] and rounded again; positions
 * outside [0, n_pos) are clamped and set status bit 1.
 * Replaces the reference's DeviceColLinear / DeviceRowLinear matmuls at the
 * path's edges: the fused compressor wkv || wgate (inference.py:4954-4966),
 * the indexer's wq_b + rotary Lk-D-idx-q kernel and weights_proj
 * (5177-5185, 5226-5258), wq_a / wq_b / wkv (5934-5960), the head-grouped
 * wo_a (G groups) and wo_b (6096-6126). */
int dsa_linear(const void* x, int64_t ld_x, const void* w_packed, void* y, int64_t ld_y, int B, int N, int K,
               int G, int out_f32, const float* cos, const float* sin, int n_pos, const int32_t* pos,
               int head_dim, int rope_dim, int rope_col0, int32_t* status, dsa_stream_t stream);

/* Bytes of the tile layout of a W [G*N, K] (0 for invalid sizes): G x
 * ceil(N/128) x K/64 tiles of 16 KB. */
size_t dsa_linear_packed_bytes(int N, int K, int G);

/* Stores W [G*N, K] bf16 row-major (16-byte aligned) once, at weight-load
 * time, as the tiles dsa_linear streams: per (group, 128-row tile, 64-wide
 * k-block) 16 KB holding the 128 rows (zero past N) x 64 k in the 128-byte
 * swizzled K-major order of the tensor cores' shared-memory operand, tiles in
 * (group, row tile, k-block) order.  The reference's equivalent is the
 * conversion of its weights to the device's tiled layout when the
 * DeviceColLinear modules are built (inference.py:4954-4966, 5934-5953). */
int dsa_linear_pack(const void* w, int N, int K, int G, void* packed, size_t packed_bytes, dsa_stream_t stream);

/* ---------------------------------------------------------------- attn.kv */

/* Block-wise max-abs FP8-E4M3 round trip of an [M, N] bf16 matrix along N.
 * Per block of `block` columns: amax = max|x|; s = max(amax, eps) * r where
 * r = 1/fp8_max rounded to fp32 (the chain multiplies by the constant, it
 * does not divide); q = e4m3_rn_satfinite(clamp(x / s, +-fp8_max)) with an
 * IEEE division; out = bf16(float(q) * s).
 * scales [M, N/block] fp32 (may be NULL); codes [M, N] e4m3 (may be NULL).
 * Replaces the tt-lang factory
 *   _compile_act_quant_block_kernel(M_pad, N, BLOCK, fp8_max, eps)(x, scaler, out)
 *   inference.py:3383-3499, with the semantics of the ttnn chain
 *   _device_act_quant_block inference.py:4578-4607 plus the e4m3 cast. */
int dsa_act_quant_block(const void* x, void* out, float* scales, uint8_t* codes,
                        int64_t M, int64_t N, int64_t ld_x, int64_t ld_out,
                        int block, float fp8_max, float eps, dsa_stream_t stream);

/* attn.kv + attn.kv_update for B sequences: act_quant_block on the first
 * D - rope_dim dims of kv [B, D] bf16 (rope dims pass through) and write
 * the row into the window ring kv_cache[b, pos[b] % win, :].
 * kv_cache: bf16, batch stride cache_bstride elements, row stride D.
 * pos: [B] int32 device array.  scales [B, (D-rope_dim)/block] (may be NULL).
 * Replaces Lk-D1's act_quant stage + paged_update_cache:
 *   inference.py:5997-6006 (_lk_d1_kernel), 6072-6079 (attn.kv_update). */
int dsa_kv_window_write(const void* kv, void* kv_cache, float* scales,
                        const int32_t* pos, int B, int D, int rope_dim,
                        int64_t cache_bstride, int win, int block,
                        dsa_stream_t stream);

/* The whole Lk-D1 zone plus attn.kv_update in one launch, for B sequences:
 * kv [B, D] bf16 (the wkv output, row stride ld_kv) -> RMSNorm(gamma, eps)
 * rounded to bf16 -> interleaved rotary of the last rope_dim dims with row
 * pos[b] of cos/sin [n_pos, rope_dim/2] fp32 -> act_quant_block (block 64,
 * e4m3, fp8_max 448, eps 1e-4) on the first D - rope_dim dims -> ring write
 * kv_cache[b, pos[b] % win]; also stored to kv_out [B, D] when non-NULL.
 * D and rope_dim multiples of 64, D <= 2048.  A position outside the table
 * is clamped and flags *status (may be NULL).
 * Replaces _lk_d1_kernel(kv, cos_full, sin_full, start_pos, kv_out)
 *   inference.py:5997-6006 (kv_norm + rotary + act_quant) followed by the
 *   paged_update_cache of attn.kv_update, inference.py:6072-6079. */
int dsa_kv_norm_rope_window_write(const void* kv, int64_t ld_kv, const float* gamma,
                                  float eps, const float* cos_tab, const float* sin_tab,
                                  int n_pos, const int32_t* pos, void* kv_cache,
                                  int64_t cache_bstride, int win, void* kv_out,
                                  int64_t ld_out, float* scales, int B, int D,
                                  int rope_dim, int32_t* status, dsa_stream_t stream);

/* Per-head RMSNorm and/or interleaved rotary of x [B, H*Dh] bf16 (row
 * stride ld_x) into out (may alias x).  do_norm: y = w * x * rsqrt(mean(x^2)
 * + eps) with w = gamma[Dh] fp32, or the scalar `weight` when gamma is NULL,
 * rounded to bf16 (the reference RMSNorm returns the input dtype).  Then,
 * when rope_dim > 0, the last rope_dim dims of each head are rotated with
 * row pos[b] of cos/sin (inverse != 0: by the conjugate).
 * Replaces the q path rms_norm(q, q_rsqrt_ones) + _lk_c_q_rotary_kernel
 *   inference.py:5982-5993, the q_norm rms_norm inference.py:6032-6034, the
 *   indexer q rotary of _lk_d_idx_q_kernel inference.py:5242, and the
 *   inverse rotary _lk_o_rotary_kernel inference.py:6100-6102. */
int dsa_head_norm_rope(const void* x, int64_t ld_x, void* out, int64_t ld_out,
                       int B, int H, int Dh, int rope_dim, const float* gamma,
                       float weight, int do_norm, float eps, const float* cos_tab,
                       const float* sin_tab, int n_pos, const int32_t* pos,
                       int inverse, int32_t* status, dsa_stream_t stream);

/* out[i] = (valid[i] < 0 ? -1 : idx[i]) for i < n: folds the additive
 * {0, -inf} bf16 mask of the reference's (indices, mask) pair back into -1
 * sentinels, which is what dsa_sparse_attn reads.
 * Inverse of DeviceSparseAttn._idxs_int_tile_to_idxs_and_mask
 *   inference.py:4444-4457. */
int dsa_fold_index_mask(const int32_t* idx, const void* valid, int64_t n,
                        int32_t* out, dsa_stream_t stream);

/* ---------------------------------------------------------- attn.compress */

/* One compressor decode step for B sequences (one kernel):
 *   state write: score_row += ape[pos % r]; kv/score rows stored at slot
 *     (overlap ? r + pos % r : pos % r)               inference.py:4954-4991
 *   if (pos + 1) % r == 0 (per sequence, read from device `pos`):
 *     softmax over slots of the overlap view, weighted sum, RMSNorm(gamma,
 *     eps), interleaved rotary of the last rope_dim dims with row
 *     pos + 1 - r of cos/sin, optional orthonormal Hadamard (rotate != 0),
 *     bf16 row written to kv_cache[b, slot_offset + pos / r], and (overlap)
 *     slot shift rows [0,r) <- rows [r,2r)             inference.py:4997-5097
 *       (cssn 3205-3364, fanout slot shift 3101-3186)
 * kv_row/score_row: [B, coff*d] bf16 (row stride ld_row), coff = 1 + overlap.
 * ape [r, coff*d] fp32.  kv_state/score_state: [B, coff*r, coff*d] fp32.
 * gamma [d] fp32.  cos/sin [n_pos, rope_dim/2] fp32.  kv_cache bf16 rows
 * of d, batch stride cache_bstride.  emitted (may be NULL): [B] int32 set
 * to 1 where a row was emitted this step, 0 where not, -1 where the emit
 * row or angle row fell outside kv_cache / the table (nothing written).
 * write_state = 0 skips the state write (kv_row/score_row/ape unused):
 * that is _emit_body alone.
 * Replaces DeviceCompressor.forward_device (inference.py:4938) with its
 * _emit_body (4997). */
int dsa_compressor_step(const void* kv_row, const void* score_row, int64_t ld_row,
                        const float* ape, float* kv_state, float* score_state,
                        const float* gamma, const float* cos_tab, const float* sin_tab,
                        int n_pos, void* kv_cache, int64_t cache_bstride,
                        int64_t cache_rows, int slot_offset, const int32_t* pos,
                        int32_t* emitted, int B, int d, int rope_dim, int ratio,
                        int overlap, int rotate, int write_state, float eps,
                        dsa_stream_t stream);

/* One compressor's arguments, as for dsa_compressor_step (the state is
 * always written; no emitted flags). */
typedef struct dsa_compressor_args {
  const void* kv_row;
  const void* score_row;
  int64_t ld_row;
  const float* ape;
  float* kv_state;
  float* score_state;
  const float* gamma;
  void* kv_cache;
  int64_t cache_bstride;
  int64_t cache_rows;
  int slot_offset;
  int d, rope_dim, ratio, overlap, rotate;
} dsa_compressor_args;

/* A decode layer's small per-sequence stages in one launch, B sequences:
 *   dsa_compressor_step(*icmp) then dsa_indexer_score_newest on its cache
 *     (icmp->kv_cache [B, >= T, 128], q iq [B, 64, 128] bf16, w iw [B, 64]
 *     fp32, score [B, ld_score] fp32, t_active);
 *   dsa_kv_window_write(kv [B, D] bf16 into cmp->kv_cache's ring rows,
 *     kv_scales may be NULL, win), dsa_window_indices(idx[:, 0:win]) and
 *     dsa_compressor_step(*cmp) on the same cache;
 * cos/sin [n_pos, rope_dim/2], pos [B] and eps shared (inference.py:
 * 4938-5097, 5997-6006, 6020-6026, 5260-5275).  Same results as those five
 * calls.  DSA_BESIDE_PREVIOUS: the caller guarantees that every input was
 * complete when the previous kernel on the stream began and that the
 * previous kernel neither writes what this call reads nor reads or writes
 * what it writes (in a decode step: the indexer score, which covers rows
 * [0, t_active - 1) while this call writes row t_active - 1 of the indexer
 * cache and of score).  The kernel then runs beside that kernel, letting the
 * next kernel launch early, and waits for it only before completing, so a
 * successor that waits for this call also sees the previous kernel's
 * writes.  No counterpart as one call in the reference (five device
 * chains). */
enum { DSA_BESIDE_PREVIOUS = 1 };
int dsa_layer_prologue(const dsa_compressor_args* icmp, const dsa_compressor_args* cmp,
                       const float* cos_tab, const float* sin_tab, int n_pos, float eps,
                       const int32_t* pos, const int32_t* t_active, const void* iq, const float* iw,
                       float* score, int64_t ld_score, int T, const void* kv, float* kv_scales, int D,
                       int rope_dim, int win, int32_t* idx, int64_t ld_idx, int B, unsigned flags,
                       dsa_stream_t stream);

/* ------------------------------------------------------------- attn.topk */

/* Window ring indices for B sequences: idx[b, i] for i < win is the
 * reference's per-position row of _build_window_topk_table (inference.py:
 * 479-506, picked at 6020-6026): [0..p, -1...] while p < win, else
 * [(p%win)+1 .. win-1, 0 .. p%win].  idx row stride ld_idx. */
int dsa_window_indices(const int32_t* pos, int32_t* idx, int64_t ld_idx, int B,
                       int win, dsa_stream_t stream);

/* Indexer score s[b, t] = sum_h w[b, h] * relu(q[b, h, :] . k[b, t, :]),
 * fp32 accumulation, for t < T.  q [B, H, Di] bf16; k bf16 rows of Di with
 * batch stride k_bstride elements; w [B, H] fp32 (already scaled by
 * Di^-1/2 * H^-1/2 when the caller follows the reference's fold);
 * score [B, T] fp32 with row stride ld_score.  k_bstride 0: one key cache
 * shared by all B rows (the queries of a prefill chunk).  t_valid (may be NULL):
 * device [B] int32; keys t >= t_valid[b] are neither read nor scored (their
 * score entries are left untouched).  Requires H == 64, Di == 128.
 * Replaces DeviceIndexer.forward_device_score's score stage
 * (inference.py:5260-5275: matmul, relu*w, head sum). */
int dsa_indexer_score(const void* q, const void* k, const float* w, float* score,
                      const int32_t* t_valid, int B, int H, int Di, int T,
                      int64_t k_bstride, int64_t ld_score, dsa_stream_t stream);

/* dsa_indexer_score with flags (same result; replaces the same reference
 * stage, inference.py:5260-5275).  DSA_KEYS_READY: the caller guarantees
 * that k and t_valid were complete before the kernel that precedes this
 * call on the stream started (in a decode step: keys written by earlier
 * steps, t_valid staged before the first layer, so no kernel between
 * writes them).  The kernel may then request its first key tiles before
 * waiting for that preceding kernel (programmatic dependent launch),
 * overlapping their latency with its tail; q and w are read after the
 * wait.  Only the per-sequence key path (k_bstride != 0) uses the flag. */
enum { DSA_KEYS_READY = 1 };
int dsa_indexer_score_ex(const void* q, const void* k, const float* w, float* score,
                         const int32_t* t_valid, int B, int H, int Di, int T,
                         int64_t k_bstride, int64_t ld_score, int flags, dsa_stream_t stream);

/* dsa_indexer_score_ex with the per-sequence keys' work split dynamically:
 * each of the persistent kernel's CTAs scores four fifths of an even share
 * of the (sequence, 128-key tile) items and then claims further ones from
 * counters
 * (uint32 [2], 8-byte aligned device memory, zero before the first call;
 * every call leaves them zero), so CTAs that start late - on SMs the
 * previous kernel still held - take fewer and all finish together.  The
 * same scores, bit for bit.  Calls that can overlap on the GPU (other
 * streams) need their own counters; after a wait timed out, re-zero them.
 * Needs k_bstride != 0 and B <= 4096.  Replaces the same reference stage
 * (inference.py:5260-5275). */
int dsa_indexer_score_dyn(const void* q, const void* k, const float* w, float* score,
                          const int32_t* t_valid, int B, int H, int Di, int T,
                          int64_t k_bstride, int64_t ld_score, int flags, uint32_t* counters,
                          dsa_stream_t stream);

/* The score of each sequence's newest live compressed row: for each b with
 * t = min(t_active[b], T) - 1 >= 0, score[b * ld_score + t] = sum_h w[b, h]
 * relu(q[b, h, :] . k[b * k_bstride + t * 128 + :]) (the score stage of
 * inference.py:5260-5275 for that one row; H = 64, Di = 128; q, k and the
 * row stride 8-byte aligned).  A decode step scores the rows before the
 * newest (dsa_indexer_score_ex with t_valid = t_active - 1) while the
 * indexer compressor may write the newest row, and calls this after the
 * compressor on the compressor's stream; the plain top-k then reads every
 * live score.  Bit-identical to the recompute of dsa_indexer_topk_newest. */
int dsa_indexer_score_newest(const void* q, const void* k, int64_t k_bstride, const float* w,
                             const int32_t* t_active, float* score, int64_t ld_score, int B, int T,
                             dsa_stream_t stream);

/* Top-k of the masked indexer score, the reference's bucketed pad+mask
 * path (inference.py:5823-5851): masked = s - 1e4 * (t >= t_active[b]);
 * select the k largest of masked[b, 0:T]; out = t + win where
 * masked >= -1000, else -1.  Ties at the k-th value are broken towards the
 * lower index.  k <= T, k <= 4096.  Output order: descending score when
 * sort_desc != 0 (the reference's sorted=True), else ascending position.
 * out_idx [B, k] int32 (row stride ld_out); out_score (may be NULL) [B, k]
 * fp32 masked scores in the same order.  mask_mode 0 is the reference's
 * additive mask; mask_mode 1 treats positions t >= t_active[b] as -inf
 * without reading them (identical output unless a score exceeds 9000, and
 * lets the score buffer beyond t_active stay unwritten, see t_valid of
 * dsa_indexer_score).  Rows with T > 16384 are selected
 * in two levels and need caller workspace: use dsa_indexer_topk_ws with
 * dsa_indexer_topk_workspace_size(B, T, k) bytes (dsa_indexer_topk returns
 * DSA_ERR_WORKSPACE for them). */
int dsa_indexer_topk(const float* score, int64_t ld_score, const int32_t* t_active,
                     int32_t* out_idx, float* out_score, int64_t ld_out,
                     int B, int T, int k, int win, int sort_desc, int mask_mode,
                     dsa_stream_t stream);
size_t dsa_indexer_topk_workspace_size(int B, int T, int k);
int dsa_indexer_topk_ws(const float* score, int64_t ld_score, const int32_t* t_active,
                        int32_t* out_idx, float* out_score, int64_t ld_out,
                        int B, int T, int k, int win, int sort_desc, int mask_mode,
                        void* workspace, size_t workspace_bytes, dsa_stream_t stream);

/* dsa_indexer_topk_ws with the score of each row's newest live entry,
 * t = min(t_active[b], T) - 1, recomputed from the indexer inputs rather than
 * read from `score`: sum_h w[b,h] relu(q[b,h,:] . k_cache[b,t,:]) (the same
 * formula as dsa_indexer_score, heads summed in order).  The decode step
 * then scores rows [0, t_active - 1) while the indexer compressor writes
 * row t_active - 1 (inference.py:5260-5275 followed by 5823-5851; the
 * reference runs the compressor first).  q [B, 64, 128] bf16 contiguous,
 * k_cache rows of 128 bf16 with batch stride k_bstride elements (>= T * 128,
 * a multiple of 8), w [B, 64] fp32; q and k_cache 16-byte aligned.
 * Workspace as for dsa_indexer_topk_ws (NULL / 0 when T <= 16384). */
int dsa_indexer_topk_newest(const float* score, int64_t ld_score, const int32_t* t_active,
                            int32_t* out_idx, float* out_score, int64_t ld_out,
                            int B, int T, int k, int win, int sort_desc, int mask_mode,
                            const void* q, const void* k_cache, int64_t k_bstride, const float* w,
                            void* workspace, size_t workspace_bytes, dsa_stream_t stream);

/* Top-k of a few long rows spread over many CTAs: one cooperative launch
 * of cpr CTAs per row (cpr * B <= the SM count) running an MSD radix select
 * with grid-wide barriers, for rows too long / too few for one CTA each
 * (the sequence split's single context).  Same masking, validity, tie and
 * win rules as dsa_indexer_topk; output in ascending position order.
 * seg_len > 0: each row is T / seg_len segments of seg_len elements placed
 * seg_stride elements apart (score and ids alike; the per-rank lists of an
 * all-gather), else contiguous.
 * ids (may be NULL): [B, T] int32 - the output then carries ids[t] + win
 * and slots with ids[t] < 0 count as -inf (the candidate merge of the split;
 * ties break towards the lower slot, so pass candidates in position order).
 * workspace: dsa_topk_wide_workspace_size(B, T) bytes, 16-byte aligned,
 * zeroed before its first use (the kernel leaves its histograms zeroed, so
 * one workspace serves calls of any B and T it is large enough for; re-zero
 * after a timeout).  status (may be NULL): bit 2 set when a grid barrier
 * timed out.
 * Returns DSA_ERR_UNSUPPORTED when the rows need more CTAs than SMs.
 * Replaces the ttnn.topk of _indexer_topk_body (inference.py:5841-5842) for
 * single long rows. */
size_t dsa_topk_wide_workspace_size(int B, int T);
int dsa_topk_wide(const float* score, int64_t ld_score, const int32_t* ids, int64_t ld_ids,
                  const int32_t* t_active, int32_t* out_idx, float* out_score, int64_t ld_out,
                  int B, int T, int k, int win, int mask_mode, int seg_len, int64_t seg_stride,
                  void* workspace, size_t workspace_bytes, int32_t* status, dsa_stream_t stream);

/* Device-side position advance for graph-replayed decode: pos[b] += step;
 * t_active[b] = (pos[b] + 1) / ratio (T_active of inference.py:6028; may
 * be NULL).  Replaces the per-step host staging of pre_stage_decode
 * (inference.py:5853-5885) when the step loop stays on the device. */
int dsa_advance_positions(int32_t* pos, int32_t* t_active, int B, int ratio, int step,
                          dsa_stream_t stream);

/* Global top-k over candidate lists (sequence split): cand_score/cand_idx
 * [B, n_cand] (fp32 masked score, int32 global compressed position, -1 =
 * empty slot); selects the k best (ties: lower position), n_cand <= 16384,
 * and writes out_idx = position + win (or -1 when the score is below -1000
 * or the slot is empty) and out_score, [B, k], in descending-score order.
 * This is the merge step of the per-shard top-k of the sequence split the
 * reference plans in briefs/future_max_utilization.md:177-204; on one GPU
 * it equals ttnn.topk over the full row (inference.py:5841-5842). */
int dsa_topk_merge(const float* cand_score, const int32_t* cand_idx, int n_cand,
                   int32_t* out_idx, float* out_score, int64_t ld_out, int B, int k,
                   int win, dsa_stream_t stream);

/* Sequence split helpers (one context's compressed entries cut into
 * contiguous shards [lo, hi), one per GPU; the split the reference plans in
 * briefs/future_max_utilization.md:177-204).
 * dsa_shard_active: t_local[b] = clamp(t_active[b] - lo, 0, n_local), the
 * shard's share of T_active (inference.py:6028).
 * dsa_shard_local_indices: from the merged global selection sel [B, k]
 * (compressed positions, -1 = none) build this shard's attention index
 * list out [B, W + k]: window slots win_idx[b, j] + win_base (win_idx NULL:
 * this shard does not attend the window, all -1), then sel - lo +
 * local_base for positions in [lo, hi), else -1.  The local list is what
 * dsa_sparse_attn_partial reads over the shard's [B, rows, D] cache. */
int dsa_shard_active(const int32_t* t_active, int32_t* t_local, int B, int lo, int n_local,
                     dsa_stream_t stream);
int dsa_shard_local_indices(const int32_t* sel, int64_t ld_sel, int k, const int32_t* win_idx,
                            int64_t ld_win, int W, int lo, int hi, int local_base, int win_base,
                            int32_t* out, int64_t ld_out, int B, dsa_stream_t stream);

/* Peer-memory exchange (the sequence split's all-gathers over NVLink).
 * dsa_p2p_export: CUDA IPC handle (dsa_p2p_handle_size() bytes) of the
 *   allocation holding ptr, and ptr's byte offset in it; dsa_p2p_import
 *   maps a peer's handle (add the offset), dsa_p2p_close unmaps it.
 *   dsa_p2p_alloc / dsa_p2p_free: a zeroed cudaMalloc buffer (set-up only;
 *   the hot calls below allocate nothing).
 * dsa_p2p_publish: copy `bytes` (multiple of 16) from src to the G device
 *   addresses dst_ptrs[g] (device array; peers' receive slots, one may be
 *   local), then release-store *epoch into the G flags flag_ptrs[g] once all
 *   of that destination's stores are visible system-wide.  done: G local
 *   zero-initialised counters (left zeroed).
 * dsa_p2p_wait: wait (acquire, bounded by the wait limit below; a timeout
 *   sets status bit 2 and the kernel returns) until flags[i] >= *epoch for
 *   all i < G.
 * dsa_counter_bump: *counter += 1 on the device (the per-step epoch).
 * Replaces the ttnn.all_gather / all_reduce collectives the reference's
 * multi-device path issues (inference.py:5274-5275) for the split of
 * briefs/future_max_utilization.md:177-204. */
int dsa_p2p_alloc(size_t bytes, void** ptr);
int dsa_p2p_free(void* ptr);
size_t dsa_p2p_handle_size(void);
int dsa_p2p_export(void* ptr, void* handle, uint64_t* offset);
int dsa_p2p_import(const void* handle, void** ptr);
int dsa_p2p_close(void* ptr);
int dsa_p2p_publish(const void* src, size_t bytes, const unsigned long long* dst_ptrs,
                    const unsigned long long* flag_ptrs, const uint32_t* epoch, int G,
                    uint32_t* done, dsa_stream_t stream);
int dsa_p2p_wait(const uint32_t* flags, int G, const uint32_t* epoch, int32_t* status,
                 dsa_stream_t stream);
int dsa_counter_bump(uint32_t* counter, dsa_stream_t stream);

/* Prefill chunk of S tokens at positions base .. base+S-1 (one sequence):
 * t_active[s] = min(T, (base + s + 1) / ratio) - the compressed entries the
 * token at that position may see (entry j is complete once 4j+3 <= p) - and
 * the first W columns of idx [S, ld_idx]: the causal window, rows of a raw
 * buffer holding the n_hist tokens before the chunk and then the chunk
 * (row s + i + n_hist - (W-1) for position p - W + 1 + i; -1 before row 0).
 * The multi-token form of the window table and T_active
 * (inference.py:479-506, 6028); the indexer scores of such a chunk come
 * from dsa_indexer_score with B = S and k_bstride = 0 (one shared key
 * cache), its per-token selection from dsa_indexer_topk with t_active. */
int dsa_prefill_positions(int S, int base, int ratio, int T, int W, int n_hist,
                          int32_t* t_active, int32_t* idx, int64_t ld_idx, dsa_stream_t stream);

/* ------------------------------------------------------------ attn.sparse */

/* Bytes of workspace dsa_sparse_attn needs for this shape (0 when it runs
 * without splitting the key range). */
size_t dsa_sparse_attn_workspace_size(int B, int S, int H, int D, int K);

/* Sparse sink attention (DeviceSparseAttn.forward_device, inference.py:
 * 4459-4501, with the index->mask conversion 4444-4457 folded in):
 *   for query row m = b*S + s:  g = kv[b, max(idx[m, j], 0)];
 *   z = (q[m] . g^T) * scale, -inf where idx[m, j] < 0;
 *   m_h = max(max_j z, sink[h]);
 *   p = e^{z - m_h} / (sum_j e^{z - m_h} + e^{sink[h] - m_h});  o = p . g.
 * q [B*S, H, D] bf16; kv bf16 rows of D with batch stride kv_bstride and
 * kv_rows rows per batch (indices >= kv_rows are an error the kernel
 * clamps and reports through `status`); idx [B*S, K] int32 (row stride
 * ld_idx); sink [H] fp32; out [B*S, H, D] bf16.  lse (may be NULL):
 * [B*S, H] fp32 natural-log partition sum including the sink.
 * workspace: >= dsa_sparse_attn_workspace_size() bytes (may be NULL when
 * that is 0).  status (may be NULL): device int32, set non-zero if any
 * index was >= kv_rows.  Requires H == 64, D == 512. */
int dsa_sparse_attn(const void* q, const void* kv, int64_t kv_bstride, int64_t kv_rows,
                    const int32_t* idx, int64_t ld_idx, const float* sink, void* out,
                    float* lse, int B, int S, int H, int D, int K, float scale,
                    void* workspace, size_t workspace_bytes, int32_t* status,
                    dsa_stream_t stream);

/* dsa_sparse_attn with a scheduling hint.  lead_cols (a multiple of 64,
 * < K; 0 = none): the first lead_cols index columns of every row (in this
 * path the window ring slots, written before the top-k).  With
 * DSA_LEAD_READY the caller guarantees that the kernel this launch may
 * overlap (the previous kernel on the stream, under programmatic dependent
 * launch) writes neither q, nor those index columns, nor the kv rows they
 * name, and that every other writer of them completed before this launch;
 * each key split then takes one 64-entry lead tile first and requests it,
 * with q, before waiting for that kernel, and the rest of the row in even
 * runs.  Same results
 * as dsa_sparse_attn (up to fp32 summation order across splits); the
 * workspace size is the same.  Has no counterpart in the reference (its
 * device path is one ttnn op chain per call). */
enum { DSA_LEAD_READY = 1 };
int dsa_sparse_attn_ex(const void* q, const void* kv, int64_t kv_bstride, int64_t kv_rows,
                       const int32_t* idx, int64_t ld_idx, const float* sink, void* out,
                       float* lse, int B, int S, int H, int D, int K, float scale,
                       void* workspace, size_t workspace_bytes, int lead_cols, unsigned flags,
                       int32_t* status, dsa_stream_t stream);

/* Allocation-free variant of dsa_sparse_attn, for callers that cannot
 * allocate device memory where they call the attention (a runtime that owns
 * a fixed device arena, a plugin running inside another framework's memory
 * manager).  Same arguments and result as dsa_sparse_attn, without the
 * workspace: the split-K partials go to an 8 MiB scratch array that the
 * library reserves in device memory on every GPU that loads it and keeps
 * until the process exits.  Shapes whose partials need more than 8 MiB
 * (dsa_sparse_attn_workspace_size() > 8 MiB) are rejected with
 * DSA_ERR_WORKSPACE.  The partials take nsplit * B * S * 64 * (2 * 4 + 512 * 2)
 * bytes (fp32 m and l, the bf16 o / l), so about 127 (query row, key split)
 * pairs fit: a few decode rows or one long context do, config 2's
 * 64-sequence decode (2 splits per row, 8.45 MB) does not and must use
 * dsa_sparse_attn with a workspace.  The
 * first call on a device looks up the array's device address and caches it
 * for the life of the process; make that first call before any stream
 * capture, and do not use this entry point across a device reset
 * (cudaDeviceReset) or a destroyed and recreated primary context, which
 * would leave the cached address stale.  All calls share the one array, so
 * calls that overlap on the GPU (other streams, other host threads) race on
 * it.  This entry point has no counterpart in the reference. */
int dsa_sparse_attn_noalloc(const void* q, const void* kv, int64_t kv_bstride, int64_t kv_rows,
                            const int32_t* idx, int64_t ld_idx, const float* sink, void* out,
                            float* lse, int B, int S, int H, int D, int K, float scale,
                            int32_t* status, dsa_stream_t stream);

/* Un-normalised partial attention for a sequence split: like
 * dsa_sparse_attn but without the sink and without normalisation; writes
 * part_ml [B*S, H, 2] = (m, l) and part_o [B*S, H, D] fp32 with
 * o = sum_j e^{z_j - m} g_j, l = sum_j e^{z_j - m} (m = -inf, l = 0, o = 0
 * when every index is masked).  Partials of disjoint index sets combine
 * with dsa_lse_combine.  (Per-shard step of the split planned in
 * briefs/future_max_utilization.md:185-199.) */
int dsa_sparse_attn_partial(const void* q, const void* kv, int64_t kv_bstride,
                            int64_t kv_rows, const int32_t* idx, int64_t ld_idx,
                            float* part_ml, float* part_o, int B, int S, int H, int D,
                            int K, float scale, void* workspace, size_t workspace_bytes,
                            int32_t* status, dsa_stream_t stream);

/* Log-sum-exp merge of P partials with the sink counted once:
 * part_ml [P, M, H, 2], part_o [P, M, H, D] fp32 (P-major, M = B*S rows);
 * M_h = max(max_p m_p, sink_h); L = sum_p l_p e^{m_p - M_h} + e^{sink_h - M_h};
 * out = sum_p o_p e^{m_p - M_h} / L as bf16 [M, H, D].  Built for D = 512;
 * part_o and out 16-byte aligned. */
int dsa_lse_combine(const float* part_ml, const float* part_o, const float* sink,
                    void* out, int P, int M, int H, int D, dsa_stream_t stream);
/* dsa_lse_combine with the P partials ml_pstride / o_pstride floats apart
 * (o_pstride a multiple of 4): partials packed one rank after another in
 * one all-gathered buffer. */
int dsa_lse_combine_strided(const float* part_ml, int64_t ml_pstride, const float* part_o,
                            int64_t o_pstride, const float* sink, void* out, int P, int M,
                            int H, int D, dsa_stream_t stream);

/* --------------------------------------------------------------- tracing */

/* Phase tracing (the device-side counterpart of the reference's _phase
 * wall-clock timers, inference.py:174-266): while a device buffer of at
 * least 8 * 256 int64 is set, sparse-attention launches record clock64()
 * stamps of their first CTA per 32-row tile: slot 0 producer issued, 1 tile
 * landed, 2 MMA warp got the tile, 3 S issued, 4 PV issued, 5 softmax got S,
 * 6 P written; slot 7 holds kernel start / end.  NULL turns it off. */
int dsa_set_trace(void* dev_buffer, size_t bytes);

#ifdef __cplusplus
}
#endif

#endif /* DSV4ATTN_H */
