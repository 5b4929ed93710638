/*
 * vesper_b200.h -- the C ABI of libvesper_b200.so, the B200 (sm_100a) kernels of the
 * mstampfli/vesper-preview column hot path.
 *
 * Conventions (every entry point):
 *   - plain device pointers and sizes; `stream` is a cudaStream_t passed as void* (NULL = the
 *     legacy default stream); work is enqueued on it and the call returns without synchronizing,
 *     so every entry point can be captured in a CUDA graph;
 *   - no allocation: outputs and workspaces are the caller's (size queries are provided);
 *   - the return value is VB_OK or an error code; vb_last_error() gives the message of the last
 *     failure on the calling host thread;
 *   - tensors are dense and row-major in the layouts named below; `dtype` codes are VB_F32,
 *     VB_BF16 and VB_F16;
 *   - deterministic: no floating-point atomics; reductions run in a fixed order.
 *
 * Each declaration cites the reference interface (file:line inside mstampfli/vesper-preview) whose
 * work it performs.
 */
#ifndef VESPER_B200_H
#define VESPER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define VB_API __attribute__((visibility("default")))
#else
#define VB_API
#endif

enum { VB_OK = 0, VB_ERR_INVALID = 1, VB_ERR_CUDA = 2, VB_ERR_TIMEOUT = 3 };
enum { VB_F32 = 0, VB_BF16 = 1, VB_F16 = 2 };

/* The message of the last failed call on this host thread ("" if none). */
VB_API const char *vb_last_error(void);
/* ABI version of this library. */
VB_API int vb_abi_version(void);
/* Kernels this library has launched in this process (every entry point counts its own). */
VB_API unsigned long long vb_launch_count(void);

/* ---- RMSNorm --------------------------------------------------------------------------------
 * y = x / sqrt(mean(x^2) + eps) * weight per row, computed scale-safely (each row divided by
 * max(max|x|, floor) first), statistics in float32, y in x's dtype; inv[r] = 1/sqrt(mean(x^2)+eps).
 * Replaces vesper/kernels/norm_triton.py:85-93 (rms_forward), reached from
 * vesper/kernels/norm.py:24-52 (fused_rms_norm) and vesper/column.py:178-180 (RMSNorm.forward).
 * x, y: [rows, width] of `dtype`; weight: [width] float32; inv: [rows] float32. */
VB_API int vb_rms_norm_fwd(const void *x, const float *weight, void *y, float *inv, int64_t rows,
                    int width, float floor_, float eps, int dtype, void *stream);

/* The forward with the output in another element type: a float32 x normalised in float32 and y
 * rounded once to bf16 or f16 (y_dtype), as the norm's float32 output cast to the autocast dtype
 * rounds it; equal dtypes are vb_rms_norm_fwd. Replaces the norm followed by the cast that every
 * consumer of a float32 norm output makes under autocast (vesper/column.py:159-188 RMSNorm, its
 * output fed to F.linear). */
VB_API int vb_rms_norm_fwd_cast(const void *x, const float *weight, void *y, float *inv, int64_t rows,
                                int width, float floor_, float eps, int x_dtype, int y_dtype,
                                void *stream);

/* Bytes of workspace vb_rms_norm_bwd needs (the gain gradient's fixed-order partial sums). */
VB_API size_t vb_rms_norm_bwd_workspace(int64_t rows, int width);

/* dx = inv * (dy*g - xhat * mean(dy*g*xhat)), xhat = x*inv; dweight = sum over rows of dy*xhat
 * (float32, fixed-order). Replaces vesper/kernels/norm_triton.py:96-109 (rms_backward). */
VB_API int vb_rms_norm_bwd(const void *x, const float *weight, const void *dy, const float *inv,
                    void *dx, float *dweight, void *workspace, int64_t rows, int width,
                    int dtype, void *stream);

/* The backward of vb_rms_norm_fwd_cast: dy in y's dtype (bf16 or f16, read as float32 exactly),
 * x and dx float32; equal dtypes are vb_rms_norm_bwd. Replaces the cast's backward followed by
 * vesper/kernels/norm_triton.py:96-109 (rms_backward). */
VB_API int vb_rms_norm_bwd_cast(const void *x, const float *weight, const void *dy, const float *inv,
                                void *dx, float *dweight, void *workspace, int64_t rows, int width,
                                int x_dtype, int dy_dtype, void *stream);

/* A residual add fused with the RMSNorm that reads its sum, over a float32 residual stream:
 * sum = x + r (x, sum float32; r float32, bf16 or f16, added as float32 in one IEEE addition),
 * y = RMSNorm(sum) in y_dtype (rounded once, as vb_rms_norm_fwd_cast), inv as vb_rms_norm_fwd.
 * width a multiple of 4 up to 1024, every tensor 16-byte aligned. Replaces the column's
 * `x = x + r` followed by the next sublayer's norm (vesper/column.py:709-812 Column.step,
 * :159-188 RMSNorm). */
VB_API int vb_add_rms_norm_fwd(const float *x, const void *r, const float *weight, float *sum, void *y,
                               float *inv, int64_t rows, int width, float floor_, float eps, int r_dtype,
                               int y_dtype, void *stream);

/* Its backward: d = RMSNorm'(sum) dy + dsum (dsum: the sum's gradient from its other readers,
 * float32, or NULL for none), dx = d (float32), dr = d rounded to r_dtype (skipped when NULL),
 * dweight as vb_rms_norm_bwd (workspace of vb_rms_norm_bwd_workspace bytes). dy in dy_dtype.
 * Replaces the norm's backward, the gradient sum autograd forms for the sum, and the add's
 * backward cast. */
VB_API int vb_add_rms_norm_bwd(const float *sum, const float *weight, const void *dy, const float *inv,
                               const float *dsum, float *dx, void *dr, float *dweight, void *workspace,
                               int64_t rows, int width, int dy_dtype, int r_dtype, void *stream);

/* The same backward as vb_rms_norm_bwd for callers that cannot allocate device memory (a plugin
 * host with a pre-planned memory budget, a loop that must not allocate, a capture or memory plan
 * an allocation would break): no workspace argument, and no cudaMalloc, cudaFree or allocating
 * library call inside. The gain gradient's partial sums live in a file-scope device array of
 * 2^20 floats (4 MiB, held by every GPU that loads the library until exit), which bounds
 * ceil(rows / 64) * width <= 2^20 (e.g. 65536 rows at width 1024); larger calls return
 * VB_ERR_INVALID with the limit in vb_last_error(). The array's address is looked up once per
 * device by the first call made with that device current, so make that first call before any
 * stream capture. All calls share the array: calls that overlap on the GPU (other streams, other
 * host threads) race and must be serialised by the caller. Nothing needs clearing between calls:
 * each call writes every partial sum it reads. Has no counterpart in the reference. */
VB_API int vb_rms_norm_bwd_noalloc(const void *x, const float *weight, const void *dy,
                                   const float *inv, void *dx, float *dweight, int64_t rows,
                                   int width, int dtype, void *stream);

/* The residual add that ends a column, over the float32 residual stream, with the loop's zeroing
 * of halted rows fused in: out[row] = keep[row] ? x + f : 0 (x, out float32 [rows, width]; f in
 * f_dtype, added as float32 in one IEEE addition; keep uint8 [rows] or NULL for every row); width
 * a multiple of 4, tensors 16-byte aligned. Replaces the column's `x + ffn(...)`
 * (vesper/column.py:709-812) followed by the loop's zeroing of halted rows. */
VB_API int vb_residual_add(const float *x, const void *f, const unsigned char *keep, float *out, long long rows,
                           int width, int f_dtype, void *stream);

/* Its backward: dx = keep ? g : 0 (float32, skipped when NULL) and df the same rounded to f_dtype
 * (skipped when NULL). */
VB_API int vb_residual_add_bwd(const float *g, const unsigned char *keep, float *dx, void *df, long long rows,
                               int width, int f_dtype, void *stream);

/* ---- causal key filter + key normalisation ---------------------------------------------------
 * u[b,t,j] = sum_r taps[r,j] * full[b, t+K-1-r, j] with full = cat(hist, z) along t, then
 * normalize_keys per head (scale-safe L2 norm, floor `floor_`), float32 arithmetic, keys in z's
 * dtype. z, keys: [B,T,W] (keys viewed [B,T,heads,W/heads]); hist: [B,K-1,W] float32;
 * taps: [K,W] float32. stats: [B,heads,T,2] float32 (8-byte aligned) or NULL: per token and head
 * r = 1 / max(||u||, floor) (the key is u r) and -1 where the clamp passes gradient (+1 where the
 * head vector stays below the floor), for vb_keys_bwd. Replaces vesper/kernels/keys_triton.py:148-156
 * (keys_forward) reached from vesper/kernels/keys.py:28-46 (fused_keys) and
 * vesper/column.py:255-289 (RecurrentSublayer.keys). */
VB_API int vb_keys_fwd(const void *z, const float *hist, const float *taps, void *keys, float *stats,
                int B, int T, int width, int heads, int taps_count, float floor_, int dtype, void *stream);

VB_API size_t vb_keys_bwd_workspace(int B, int T, int width, int heads, int taps_count);

/* Gradients of sum(keys * grad_keys): grad_z [B,T,W] in z's dtype, grad_taps [K,W] float32
 * (fixed-order), grad_hist [B,K-1,W] float32 (skipped when NULL; 16-byte aligned, as the
 * workspace). stats: vb_keys_fwd's output for
 * the same inputs, or NULL to recompute the statistics (slower). Replaces
 * vesper/kernels/keys_triton.py:159-177 (keys_backward) and vesper/kernels/keys.py:67-78
 * (_history_gradient). */
VB_API int vb_keys_bwd(const void *z, const float *hist, const float *taps, const void *grad_keys,
                const float *stats, void *grad_z, float *grad_taps, float *grad_hist, void *workspace,
                int B, int T, int width, int heads, int taps_count, float floor_, int dtype, void *stream);

/* ---- delta-rule scan, float32 (token-serial) --------------------------------------------------
 * H_t = H_{t-1} + beta_t k_t (v_t - H_{t-1}^T k_t)^T, o_t = H_t^T q_t, H read as [key, value].
 * q, k, v, o: [B,T,H,D] float32; beta: [B,T,H]; state0, state_n: [B,H,D,D]; resid: [B,T,H,D]
 * float32 (v_t - H_{t-1}^T k_t, saved for the backward; may be NULL). D <= 256.
 * Replaces vesper/kernels/delta_scan.py:156-187 (delta_scan_fused_fp32, which ran fla-core's
 * fused_recurrent_delta_rule) with the semantics of vesper/recurrence.py:143-217. */
VB_API int vb_delta_scan_f32_fwd(const float *q, const float *k, const float *v, const float *beta,
                          const float *state0, float *o, float *state_n, float *resid, int B,
                          int T, int H, int D, void *stream);

VB_API size_t vb_delta_scan_f32_bwd_workspace(int B, int T, int H, int D);

/* Gradients of sum(o*dout) + sum(state_n*dstate_n) (dstate_n may be NULL = zero) for all five
 * inputs; `resid` from the forward. */
VB_API int vb_delta_scan_f32_bwd(const float *q, const float *k, const float *v, const float *beta,
                          const float *state0, const float *resid, const float *dout,
                          const float *dstate_n, float *dq, float *dk, float *dv, float *dbeta,
                          float *dstate0, void *workspace, int B, int T, int H, int D,
                          void *stream);

/* The same scan taking the write-strength LOGITS: beta = sigmoid(beta_logits + shift) is formed
 * inside the kernels (shift: [B,T] float32, one value per token shared by the heads, or NULL = 0;
 * -inf gives an exact zero write), and the backward returns the logits' gradient
 * dlogits = (dbeta * (1 - beta)) * beta in `dlogits`. Replaces vesper/recurrence.py:34-88
 * (write_strength: sigmoid(logits), with the modulator's odds shift ln(1 + alpha m)) fused with
 * the scan, as called from vesper/column.py:236-253 (RecurrentSublayer.project). */
VB_API int vb_delta_scan_f32_fwd_logits(const float *q, const float *k, const float *v,
                                        const float *beta_logits, const float *shift,
                                        const float *state0, float *o, float *state_n, float *resid,
                                        int B, int T, int H, int D, void *stream);

VB_API int vb_delta_scan_f32_bwd_logits(const float *q, const float *k, const float *v,
                                        const float *beta_logits, const float *shift,
                                        const float *state0, const float *resid, const float *dout,
                                        const float *dstate_n, float *dq, float *dk, float *dv,
                                        float *dlogits, float *dstate0, void *workspace, int B,
                                        int T, int H, int D, void *stream);

/* One token per (batch, head) applied to the float32 state: the decode step
 * H' = H + beta k (v - H^T k)^T, o = H'^T q, for q, k, v [B,H,D] and beta [B,H] of `dtype`
 * (VB_F32 or VB_BF16; bf16 beta, or the sigmoid of bf16 logits with `from_logits`, rounded to
 * bf16 as the chunked kernels round it), shift [B] float32 or NULL, o [B,H,D] of `dtype`.
 * state0 and state_n [B,H,D,D] float32 may be the same buffer (an in-place step). D <= 256.
 * Replaces vesper/recurrence.py:143-163 (delta_scan_step, one token of delta_update + read) as
 * the batched decode of vesper/decode.py:29-46 (decode_step) reaches it. */
VB_API int vb_delta_scan_step(const void *q, const void *k, const void *v, const void *beta,
                              const float *shift, int from_logits, const float *state0,
                              float *state_n, void *o, int B, int H, int D, int dtype,
                              void *stream);

/* ---- delta-rule scan, bfloat16 (chunked WY form on tcgen05) -----------------------------------
 * The same recurrence as above with bf16 q, k, v, beta, o [B,T,H,D] / [B,T,H] and float32
 * state0, state_n [B,H,D,D]; 64-token chunks, D <= 128 and a multiple of 8, 16-byte aligned
 * tensors. `saved` (vb_delta_scan_bf16_saved_bytes) receives what the backward reuses: the
 * per-chunk (I + strictly_lower(diag(beta) K K^T))^-1 tiles and the per-chunk state checkpoints.
 * `status` is one device int32: a kernel that gave up waiting on the tensor core ORs in a bit
 * (the caller checks it after synchronising; it is never reset here).
 * Replaces vesper/kernels/delta_scan.py:132-153 (delta_scan_fused, which ran fla-core's
 * chunk_delta_rule) with the semantics of vesper/recurrence.py:166-217. */
VB_API size_t vb_delta_scan_bf16_saved_bytes(int B, int T, int H, int D);

VB_API int vb_delta_scan_bf16_fwd(const void *q, const void *k, const void *v, const void *beta,
                                  const float *state0, void *o, float *state_n, void *saved,
                                  int *status, int B, int T, int H, int D, void *stream);

VB_API size_t vb_delta_scan_bf16_bwd_workspace(int B, int T, int H, int D);

/* Gradients of sum(o*dout) + sum(state_n*dstate_n) (dstate_n may be NULL = zero): dq, dk, dv,
 * dbeta in bf16, dstate0 in float32; `saved` from the forward on the same inputs. */
VB_API int vb_delta_scan_bf16_bwd(const void *q, const void *k, const void *v, const void *beta,
                                  const void *saved, const void *dout, const float *dstate_n,
                                  void *dq, void *dk, void *dv, void *dbeta, float *dstate0,
                                  void *workspace, int *status, int B, int T, int H, int D,
                                  void *stream);

/* The bf16 scan taking the write-strength logits (bf16 [B,T,H]) and an optional per-token float32
 * shift [B,T]: beta = bf16(sigmoid(float(logit) + shift)) as torch.sigmoid rounds its bf16
 * output, and dlogits = bf16(dbeta) * (1 - beta) * beta with every intermediate rounded to bf16,
 * as torch's bf16 sigmoid_backward forms it (bit-identical to sigmoid then the scan). Replaces vesper/recurrence.py:34-88 (write_strength) fused with
 * vesper/kernels/delta_scan.py:132-153 (delta_scan_fused). */
VB_API int vb_delta_scan_bf16_fwd_logits(const void *q, const void *k, const void *v,
                                         const void *beta_logits, const float *shift,
                                         const float *state0, void *o, float *state_n, void *saved,
                                         int *status, int B, int T, int H, int D, void *stream);

VB_API int vb_delta_scan_bf16_bwd_logits(const void *q, const void *k, const void *v,
                                         const void *beta_logits, const float *shift,
                                         const void *saved, const void *dout,
                                         const float *dstate_n, void *dq, void *dk, void *dv,
                                         void *dlogits, float *dstate0, void *workspace,
                                         int *status, int B, int T, int H, int D, void *stream);

/* ---- windowed attention ------------------------------------------------------------------
 * Softmax attention of q [B,NQ,H,DK] over keys, values [B,L,HKV,DK] (bf16 or f16 by `dtype`,
 * DK a multiple of 16 in [16, 128], H a multiple of HKV, 16-byte aligned tensors): query row r
 * at key index p attends the keys j with p - window < j <= p, scale 1/sqrt(DK), query head h
 * reading key head h / (H / HKV). `qpos` NULL: p = L - NQ + r (the cache's L - NQ rows come
 * first, then the chunk; the reference's zero-query padding of the cache rows is not needed).
 * `qpos` [B,NQ] int32: the positions of compacted query rows, ascending along each batch row;
 * `counts` [B] int32 (or NULL = NQ) says how many rows of each batch are live, the rest get zero
 * output and no gradient. `lse` [B,H,NQ] float32 is saved for the backward (base-2 log-sum-exp
 * of the scaled scores). `status`: as for the scan.
 * Replaces vesper/kernels/window_attn.py:27-39 (window_attention, which ran fla-core's
 * parallel_attn) with the semantics of vesper/attention.py:340-407 (WindowedAttention.attend). */
VB_API int vb_window_attn_fwd(const void *q, const int *qpos, const int *counts, const void *keys,
                              const void *values, void *o, float *lse, int *status, int B, int NQ,
                              int L, int H, int HKV, int DK, int window, int dtype, void *stream);

VB_API size_t vb_window_attn_bwd_workspace(int B, int NQ, int H);

/* Gradients of sum(o*dout): dq [B,NQ,H,DK], dkeys, dvalues [B,L,HKV,DK] in the input type, from
 * the forward's o and lse; deterministic (no atomics). */
VB_API int vb_window_attn_bwd(const void *q, const int *qpos, const int *counts, const void *keys,
                              const void *values, const void *o, const float *lse,
                              const void *dout, void *dq, void *dkeys, void *dvalues,
                              void *workspace, int *status, int B, int NQ, int L, int H, int HKV,
                              int DK, int window, int dtype, void *stream);

/* ---- the loop's active-token bookkeeping --------------------------------------------------
 * Per batch row of `active` [B,N] (one byte per token, nonzero = active): idx[b][r] = the r-th
 * active token (ascending), -1 beyond the count; rank[b][t] = its compact row, -1 for a halted
 * token; counts[b] = the active count; qpos (optional, may be NULL) = idx + qpos_offset, the
 * attention's key index of each compact row. Device arrays, no host synchronisation.
 * Replaces the dense compute of halted tokens in vesper/loop.py:349-465 (Loop.forward), which
 * computes every position and discards the halted ones (vesper/loop.py:24-26). */
VB_API int vb_compact_index(const unsigned char *active, int *idx, int *rank, int *counts,
                            int *qpos, int B, int N, int qpos_offset, void *stream);

/* Row copies over up to 12 tensors in one launch; tensor i is a byte array of rows of
 * row_bytes[i]; a NULL source pointer (or array) reads as zero bytes.
 * select: out_i[t] = (mask[t] != 0) != invert ? a_i[t] : b_i[t] over `tokens` rows: the
 * copy-forward merges of vesper/column.py:140-143 (_carry) and vesper/loop.py:523-537 (_merge),
 * and the zeroing of inactive rows (vesper/loop.py:427-428), as one launch each. */
VB_API int vb_select_rows(const unsigned char *mask, int invert, int ntensors,
                          const void *const *a, const void *const *b, void *const *out,
                          const long long *row_bytes, long long tokens, void *stream);

/* gather: dst_i[b][r] = src_i[b][idx[b][r]] for r < counts[b] (counts NULL = all NC rows) and an
 * index inside [0, N); zero otherwise. src_i is [B,N,row], dst_i [B,NC,row]. */
VB_API int vb_gather_rows(const int *idx, const int *counts, int B, int N, int NC, int ntensors,
                          const void *const *src, void *const *dst, const long long *row_bytes,
                          void *stream);

/* expand: dst_i[b][t] = src_i[b][rank[b][t]] where 0 <= rank < NC, else fallback_i[b][t] (NULL =
 * zero). src_i is [B,NC,row], fallback_i and dst_i [B,N,row]. The inverse of gather. */
VB_API int vb_expand_rows(const int *rank, int B, int N, int NC, int ntensors,
                          const void *const *src, const void *const *fallback, void *const *dst,
                          const long long *row_bytes, void *stream);

/* gather for bucketed work: as vb_gather_rows with counts required, except that the rows from
 * counts[b] up to the end of its bucket (the smallest first * 2^k >= counts[b], clamped to NC) are
 * zeroed and the rows past it are left untouched, so the copy's cost follows the active rows. */
VB_API int vb_gather_rows_slabs(const int *idx, const int *counts, int B, int N, int NC, int first,
                                int ntensors, const void *const *src, void *const *dst,
                                const long long *row_bytes, void *stream);

/* flatten: the compaction of all B x N tokens as one row from the per-row one (vb_compact_index):
 * flat_idx[base_b + r] = b N + idx[b][r] for r < counts[b], flat_rank[b N + t] = base_b +
 * rank[b][t] (-1 halted), *flat_count = the active total; base_b = counts[0] + ... + counts[b-1].
 * With flat_pb and pb_flat (both or neither), the map between flat compact rows and per-row
 * compact rows (b, r) stored at b N + r: flat_pb[base_b + r] = b N + r, pb_flat[b N + r] =
 * base_b + r for r < counts[b], else -1. The loop's per-token work after compaction
 * (vesper/loop.py:24-26: "a kernel skips them"). */
VB_API int vb_flatten_compaction(const int *idx, const int *rank, const int *counts, int B, int N,
                                 int *flat_idx, int *flat_rank, int *flat_count, int *flat_pb,
                                 int *pb_flat, void *stream);

/* ---- buckets: work over a device-side row count inside one captured graph ----
 * The prefixes [0, end_k) of a buffer of `cap` rows, end_0 = first, end_k = 2 end_{k-1} (the last
 * clamped to cap), are the buckets; vb_slab_count gives their number n (at most 24). While
 * `stream` is being captured, vb_slab_switch captures a kernel that reads *count when the graph
 * runs, then adds a SWITCH conditional node with n bodies (returned in bodies[0..n)): the node
 * runs body k for the smallest k with end_k >= *count, and none for a count of zero.
 * vb_slab_begin starts capturing one body on `body_stream` (launches made there until
 * vb_slab_close form it). A replay then does the work of at most twice the active rows. The
 * loop's dense compute of halted tokens is what this removes (vesper/loop.py:24-26); the graph it
 * lives in is the captured train step (vesper/graphs.py:49-289). */
VB_API int vb_slab_count(int cap, int first);
VB_API int vb_slab_switch(const int *count, int cap, int first, void *stream, void **bodies);
VB_API int vb_slab_begin(void *body, void *body_stream);
VB_API int vb_slab_close(void *body_stream);

/* ---- fused elementwise ops of the column (bf16, f16 or f32 by `dtype`, 16-byte aligned) ----
 * relu_square: y = relu(z)^2 and dz from dy, n elements, bit-identical to the reference's
 * separate relu and product ops in the same dtype. Replaces vesper/kernels/act.py:21
 * (relu_square) with the semantics of vesper/ffn.py:44-56. */
VB_API int vb_relu_square_fwd(const void *z, void *y, long long n, int dtype, void *stream);
VB_API int vb_relu_square_bwd(const void *z, const void *dy, void *dz, long long n, int dtype,
                              void *stream);

/* rotary: x [tokens, heads, dk] rotated pairwise by pos[token] * inv_freq[j] (inv_freq [dk/2]
 * float64, pos int64), phases in float64 and each product and sum rounded to the dtype as the
 * reference's ops round; backward != 0 applies the transposed rotation to an output gradient.
 * Replaces the op sequence of vesper/attention.py:178-217 (rotary). */
VB_API int vb_rotary(const void *x, const long long *pos, const double *inv_freq, void *y,
                     long long tokens, int heads, int dk, int backward, int dtype, void *stream);

/* ---- one-token decoding attention over a ring window ---------------------------------------
 * q [B,H,DK] (one token per row), k_new, v_new [B,HKV,DK], the ring k, v [B,W,HKV,DK], pos
 * [B,W] int64, valid [B,W] bytes, the new tokens' positions pos [B] int64; o [B,H,DK]. Every
 * element tensor is of `dtype`. The token attends the valid slots with p - window < pos <= p and
 * itself (scale 1/sqrt(DK), head h reading key head h / (H / HKV), H / HKV <= 8, DK <= 128), then
 * is written IN PLACE into slot p % W (k, v, pos, valid). `workspace`
 * (vb_ring_attend_workspace bytes) holds the partial results of the window's 128-slot ranges.
 * Replaces vesper/attention.py:298-338 (attend_ring) with :109-139 (kv_ring_write), batched over
 * the rows of a decode step. */
VB_API size_t vb_ring_attend_workspace(int B, int W, int H, int HKV, int DK);

VB_API int vb_ring_attend(const void *q, const void *k_new, const void *v_new, void *ring_k,
                          void *ring_v, int64_t *ring_pos, uint8_t *ring_valid, const int64_t *pos,
                          void *o, void *workspace, int B, int W, int H, int HKV, int DK, int window,
                          int dtype, void *stream);

/* ---- the head's per-row next-token loss (linear_nll's row steps) ---------------------------
 * logits: [rows, V] of `dtype` with row stride `stride` (elements); targets: [rows] int64 in
 * [0, V). vb_nll_row_stats writes float32 top[r] = max_j x[r,j], log_total[r] =
 * log sum_j exp(x[r,j] - top[r]) and nll[r] = (top[r] - x[r,target]) + log_total[r].
 * vb_nll_row_grad overwrites the logits in place with
 * grad[r] * (exp((x - top[r]) - log_total[r]) - onehot(target)), computed in float32.
 * Replaces vesper/kernels/nll_triton.py:24-103 (row_stats, row_grad_), the row steps of
 * vesper/kernels/nll.py:48-169 (linear_nll). */
VB_API int vb_nll_row_stats(const void *logits, int64_t stride, const int64_t *targets, float *top,
                            float *log_total, float *nll, int64_t rows, int V, int dtype,
                            void *stream);

VB_API int vb_nll_row_grad(void *logits, int64_t stride, const int64_t *targets, const float *top,
                           const float *log_total, const float *grad, int64_t rows, int V,
                           int dtype, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* VESPER_B200_H */
