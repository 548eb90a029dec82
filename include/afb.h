/*
 * alphafly_b200 -- C ABI of the B200 (sm_100a) connectome recurrence.
 *
 * The path:  h <- h + alpha (clamp(W h + b + u, 0, h_max) - h), T steps, over a fixed signed CSR
 * wiring W[post, pre] with per-synapse gains (chessfly/brain.py), evaluated through the light
 * cone (only rows that can vary and still reach an output) in float32 or as a float16 deviation
 * from the resting trajectory.
 *
 * Conventions
 *  - Every pointer argument is DEVICE memory of the current CUDA device unless it says "host".
 *  - `stream` is a cudaStream_t (NULL = the legacy default stream); all work is queued on it and
 *    every call returns without waiting for the GPU, except where "synchronous" is stated.
 *  - Dense state and drive matrices are (rows, batch) row-major with a leading dimension `ld`
 *    (elements), the layout of chessfly/brain.py:67-68,211-213.
 *  - Return value: AFB_OK (0) or a negative AFB_E* code; afb_last_error() gives the message of the
 *    last failure on the calling thread.  Argument errors are detected on the host before any work
 *    is queued, so a failed call leaves outputs untouched.
 *  - Handles are not thread-safe: one thread (or external locking) per handle.  Calls on the same
 *    handle from different streams must be ordered by the caller.
 */
#ifndef AFB_H
#define AFB_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AFB_API __attribute__((visibility("default")))
#else
#define AFB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define AFB_OK 0
#define AFB_EINVAL (-1)  /* bad argument: shape, size, alignment, mode */
#define AFB_ECUDA (-2)   /* a CUDA runtime call failed */
#define AFB_ESTATE (-3)  /* call out of order, e.g. forward before afb_cone_set_weights */

/* State modes of the forward pass. */
#define AFB_MODE_F32 0   /* absolute state h in float32 (chessfly/brain.py:307-329) */
#define AFB_MODE_DEV16 1 /* float16 deviation d = h - c from the resting trajectory (brain.py:254-280) */

/* Message of the last failed call on this thread ("" if none). */
AFB_API const char *afb_last_error(void);

/* Library version and the device architecture it was compiled for (e.g. 100 for sm_100a). */
AFB_API int afb_version(void);
AFB_API int afb_compiled_arch(void);

/* ---- per-synapse weights ------------------------------------------------------------------
 * w[e] = sign[e] * w0[e] * exp(log_gain[e])      replaces ConnectomeRNN.edge_weights
 *                                                (chessfly/brain.py:201-202)               */
AFB_API int afb_edge_weights(int64_t e, const float *sign, const float *w0, const float *log_gain, float *w,
                     void *stream);

/* ---- light cone ----------------------------------------------------------------------------
 * Replaces LightCone.__init__ + _SubMatrix (chessfly/brain.py:102-173) and ConnectomeRNN's
 * CSR buffers (brain.py:187-195).  Built on the GPU from the edge list (pre, post) of E synapses
 * over n neurons, sorted by (post, pre).  in_idx / out_idx: the input and output neurons (int64;
 * duplicates in in_idx resolve to the last occurrence).  Synchronous (it sizes its own arrays).  */
typedef struct afb_cone afb_cone;

AFB_API int afb_cone_create(afb_cone **cone, int64_t n, int64_t e, const int64_t *pre, const int64_t *post,
                    const int64_t *in_idx, int64_t n_in, const int64_t *out_idx, int64_t n_out,
                    int steps, void *stream);
AFB_API void afb_cone_destroy(afb_cone *cone);

/* Sizes, written to HOST arrays: rows_len[t] = |R_t| and nnz[t] = edges of the step-t sub-matrix
 * for t = 0..steps (nnz[t] = -1 where the reference has no matrix, i.e. R_{t-1} is empty);
 * n_keep[t], n_fed[t] likewise; *n_hit = outputs inside R_T; *edge_visits = sum of nnz. */
AFB_API int afb_cone_sizes(const afb_cone *cone, int64_t *rows_len, int64_t *nnz, int64_t *n_keep,
                   int64_t *n_fed, int64_t *n_hit, int64_t *edge_visits);

/* Field ids for afb_cone_export (names of the reference's LightCone / _SubMatrix fields). */
#define AFB_F_ROWS 0       /* rows[t]              (|R_t|)        brain.py:151 */
#define AFB_F_CARRIED 1    /* carried[t] as 0 / 1  (|R_t|)        brain.py:161 */
#define AFB_F_KEEP_NEXT 2  /* keep_next[t]         (n_keep[t])    brain.py:162 */
#define AFB_F_KEEP_PREV 3  /* keep_prev[t]         (n_keep[t])    brain.py:163 */
#define AFB_F_PREV_ROW 4   /* prev_row[t]          (|R_t|)        brain.py:165 */
#define AFB_F_U_POS 5      /* u_pos[t]             (n_fed[t])     brain.py:167 */
#define AFB_F_U_SRC 6      /* u_src[t]             (n_fed[t])     brain.py:168 */
#define AFB_F_OP_EDGES 7   /* ops[t].edges         (nnz[t])       brain.py:112 */
#define AFB_F_OP_POST 8    /* ops[t].post          (nnz[t])       brain.py:113 */
#define AFB_F_OP_PRE 9     /* ops[t].pre           (nnz[t])       brain.py:113 */
#define AFB_F_OP_CROW 10   /* ops[t].crow          (|R_t| + 1)    brain.py:115 */
#define AFB_F_OP_T_ORDER 11/* ops[t].t_order       (nnz[t])       brain.py:116 */
#define AFB_F_OP_T_CROW 12 /* ops[t].t_crow        (|R_{t-1}| + 1) brain.py:117 */
#define AFB_F_OP_T_COL 13  /* ops[t].t_col         (nnz[t])       brain.py:117 */
#define AFB_F_OUT_POS 14   /* out_pos (t ignored)  (n_hit)        brain.py:172 */
#define AFB_F_OUT_SRC 15   /* out_src (t ignored)  (n_hit)        brain.py:172 */

/* Copy one field of step t, widened to int64, into dst (device). */
AFB_API int afb_cone_export(const afb_cone *cone, int field, int t, int64_t *dst, void *stream);

/* ---- weight-version precompute -------------------------------------------------------------
 * Replaces the cached part of forward_io (chessfly/brain.py:257-270, 296-306) and _constants
 * (brain.py:238-252): the resting trajectory c_0..c_T (c_0 = 0, c_t = lerp(c_{t-1},
 * clamp(W c_{t-1} + b, 0, h_max), alpha)), the per-row constants of every step for `mode`, and the
 * sub-matrix values w[edges] (float32 for AFB_MODE_F32, float16 for AFB_MODE_DEV16).  w: (E) edge
 * weights; bias, alpha_logit: (n).  Must be called again whenever w, bias or alpha_logit change. */
AFB_API int afb_cone_set_weights(afb_cone *cone, int mode, const float *w, const float *bias,
                         const float *alpha_logit, float h_max, void *stream);

/* Copy the resting trajectory c_t (n floats) into dst.  t = 0..steps. */
AFB_API int afb_cone_resting(const afb_cone *cone, int t, float *dst, void *stream);

/* ---- inference forward through the light cone -----------------------------------------------
 * Replaces ConnectomeRNN.forward_io's no-grad paths (chessfly/brain.py:282-329 float32,
 * brain.py:254-280 float16 deviation).  u_in: (n_in, batch) drive of the input neurons, float32 for
 * AFB_MODE_F32 or float16 for AFB_MODE_DEV16, leading dimension ld_u >= batch.  out: (n_out, batch)
 * float32, leading dimension ld_out >= batch.  workspace: scratch of afb_cone_forward_workspace()
 * bytes, 256-byte aligned; contents need no initialisation. */
AFB_API size_t afb_cone_forward_workspace(const afb_cone *cone, int mode, int64_t batch);
AFB_API int afb_cone_forward(const afb_cone *cone, int mode, const void *u_in, int64_t ld_u, int64_t batch,
                     float *out, int64_t ld_out, void *workspace, size_t workspace_bytes, void *stream);

/* As afb_cone_forward, and records events[t - 1] on `stream` just before the kernel of step t
 * (t = 1..steps), events[steps] after the last step and events[steps + 1] after the output kernel.
 * events: steps + 2 cudaEvent_t handles of the current device.  For per-step timing (the reference
 * times its steps from Python, scripts/profile_gpu.py:29-44). */
AFB_API int afb_cone_forward_timed(const afb_cone *cone, int mode, const void *u_in, int64_t ld_u, int64_t batch,
                           float *out, int64_t ld_out, void *workspace, size_t workspace_bytes,
                           void *const *events, void *stream);

/* As afb_cone_forward, but allocating nothing and taking no workspace: for callers that cannot
 * allocate device memory at evaluation time (their device memory belongs to another framework's pool,
 * or their serving loop cannot take cudaMalloc's implicit synchronisation).  No counterpart in the
 * reference, which always allocates through torch.  The state lives in a fixed 32 MiB device array
 * built into the library (held on every GPU that loads it until the process exits); a cone and batch
 * whose afb_cone_forward_workspace() exceeds 32 MiB are rejected with AFB_EINVAL.  The current device
 * and `stream`'s device must be the device the cone was created on (AFB_EINVAL otherwise).  The first call
 * on a device resolves that array's device address (cudaGetSymbolAddress) and should come before any
 * stream capture on that device; the address is cached for the life of the process, so the call must not
 * be used across a cudaDeviceReset of that device.  The array needs no clearing (every step overwrites
 * what the next reads).  All calls on a device share it: calls whose work overlaps on the GPU (other
 * streams, other cones) race and corrupt each other's results; order them. */
AFB_API int afb_cone_forward_noalloc(const afb_cone *cone, int mode, const void *u_in, int64_t ld_u, int64_t batch,
                                     float *out, int64_t ld_out, void *stream);

/* Device status word of the handle's step kernels, copied to *status (HOST): 0 = ok; a non-zero value
 * would mean that a step kernel's bounded wait gave up and that forward's output is not valid.  The
 * current step kernels load their rows straight into registers and have no such waits, so the word stays
 * 0; it is kept as part of the interface.  With reset != 0 the word is cleared.  Synchronous on `stream`. */
AFB_API int afb_cone_status(const afb_cone *cone, int *status, int reset, void *stream);

/* ---- training: forward with saved state, and backward -----------------------------------------
 * Replaces forward_io with autograd enabled (chessfly/brain.py:289-294, 315-329) and the backward of
 * _SparseRecurrent (brain.py:78-99) and _constants (brain.py:238-252).  float32 only; needs
 * afb_cone_set_weights(AFB_MODE_F32) with the current weights.
 * afb_cone_forward_train: as afb_cone_forward(AFB_MODE_F32), keeping every step's state and pre-clamp
 *   drive in `saved` (afb_cone_train_workspace bytes, 256-byte aligned) for afb_cone_backward.
 * afb_cone_backward: given dL/dout (n_out, batch), writes dL/du_in (n_in, batch), dL/dw (E), dL/db (n)
 *   and dL/dalpha (n, alpha = sigmoid(alpha_logit)); the chain rule to log_gain (dL/dw * w) and to
 *   alpha_logit (dL/dalpha * alpha (1 - alpha)) is the caller's.  workspace: afb_cone_backward_workspace
 *   bytes, 256-byte aligned, no initialisation needed.  Deterministic: no floating-point atomics except
 *   where two output positions name the same neuron. */
AFB_API size_t afb_cone_train_workspace(const afb_cone *cone, int64_t batch);
AFB_API int afb_cone_forward_train(const afb_cone *cone, const float *u_in, int64_t ld_u, int64_t batch, float *out,
                                   int64_t ld_out, void *saved, size_t saved_bytes, void *stream);
AFB_API size_t afb_cone_backward_workspace(const afb_cone *cone, int64_t batch);
AFB_API int afb_cone_backward(const afb_cone *cone, const float *g_out, int64_t ld_g, int64_t batch, const void *saved,
                              size_t saved_bytes, float *g_u_in, int64_t ld_gu, float *g_w, float *g_bias, float *g_alpha,
                              void *workspace, size_t workspace_bytes, void *stream);

/* ---- the literal recurrence over all neurons --------------------------------------------------
 * Replaces ConnectomeRNN.forward's no-grad branch (chessfly/brain.py:211-223): from h = 0,
 * `steps` times  h <- lerp(h, clamp(W h + b + u, 0, h_max), alpha)  over all n neurons, float32.
 * u: (n, batch) drive, ld_u >= batch; h: (n, batch) result, ld_h >= batch. */
typedef struct afb_graph afb_graph;

AFB_API int afb_graph_create(afb_graph **graph, int64_t n, int64_t e, const int64_t *pre, const int64_t *post,
                     void *stream);
AFB_API void afb_graph_destroy(afb_graph *graph);
AFB_API int afb_graph_status(const afb_graph *graph, int *status, int reset, void *stream);
AFB_API size_t afb_graph_forward_workspace(const afb_graph *graph, int64_t batch);
AFB_API int afb_graph_forward(const afb_graph *graph, const float *w, const float *bias, const float *alpha_logit,
                      float h_max, const float *u, int64_t ld_u, int64_t batch, int steps, float *h,
                      int64_t ld_h, void *workspace, size_t workspace_bytes, void *stream);

/* ---- the readout heads on the tensor cores (chessfly/model.py:103-105) -----------------------------
 * The reference normalises the output neurons with RunningNorm and applies the dense heads in float32:
 *     r = clamp((out^T - mean) / sqrt(var + eps), -clip, clip)
 *     logits = r Wp^T + bp + (r Wf^T + bf)[:, move_from] + (r Wt^T + bt)[:, move_to],  wdl = r Wv^T + bv.
 * The from/to terms are linear in r, so the caller folds them into the policy rows once per weight version
 * (W[m] = Wp[m] + Wf[move_from[m]] + Wt[move_to[m]], b[m] likewise) and stacks the value rows below:
 * W (n_rows x n_out) with n_rows = n_policy + n_value.
 *
 * afb_heads_split: hi = fp16(x), lo = fp16((x - hi) * 2^11) of a float32 matrix src (rows x cols, row
 *   stride ld_src) into hi, lo (rows x ld_dst float16, columns cols..ld_dst-1 zero).  Run once per weight
 *   version on W.  Asynchronous on `stream`.
 * afb_readout_workspace: bytes of scratch afb_readout_heads needs for `batch` positions.
 * afb_readout_heads: out (n_out, batch) float32 with row stride ld_r (the layout of the light-cone
 *   forward's output); mean, var (n_out) the normaliser's statistics; w_hi, w_lo from afb_heads_split
 *   (row stride ldw, a multiple of 8; 16-byte aligned); bias (n_rows) float32.  Writes
 *   logits[p * ld_logits + m] for m < n_policy (float32, or float16 with logits_f16 != 0) and
 *   values[p * ld_values + j] = D[n_policy + j, p] for j < n_rows - n_policy, p < batch.  The product runs
 *   on the tensor cores with both operands split into float16 hi and lo parts and two float32
 *   accumulators (D = W_hi r_hi + (W_hi r_lo + W_lo r_hi) / 2^11): float32 accuracy (~1e-6 relative).
 *   status: optional device int, OR-ed with a non-zero code if one of the kernel's bounded waits gave up
 *   (never expected).  Asynchronous on `stream`. */
AFB_API int afb_heads_split(int64_t rows, int64_t cols, const float *src, int64_t ld_src, void *hi, void *lo,
                            int64_t ld_dst, void *stream);
AFB_API size_t afb_readout_workspace(int64_t batch, int64_t n_out);
AFB_API int afb_readout_heads(int64_t n_out, int64_t batch, const float *out, int64_t ld_r, const float *mean,
                              const float *var, float eps, float clip, int64_t n_rows, int64_t n_policy, const void *w_hi,
                              const void *w_lo, int64_t ldw, const float *bias, void *logits, int64_t ld_logits,
                              int logits_f16, float *values, int64_t ld_values, void *workspace, size_t workspace_bytes,
                              int *status, void *stream);

/* ---- the float16 input map (chessfly/model.py:101-102) ----------------------------------------------
 * The reference computes the drive of the input neurons as  u_in = (x[:, :k] W^T + b) * input_gain,
 * transposed to (n_in, B) and cast to float16 for the deviation path.  This entry point computes
 *     u[i * ldu + p] = fp16( gain * (sum_{k < k_dim} w[i * ldw + k] x[p * ldx + k] + b[i]) )
 * for i < n_in, p < batch on the tensor cores (tcgen05.mma, float16 operands, float32 accumulation, one
 * rounding).  w (n_in rows) and x (batch rows) are float16, row-major with k_dim valid elements per row;
 * ldw and ldx must be multiples of 8 and w, x 16-byte aligned (TMA operands).  b: n_in float16.  u: float16,
 * ldu >= batch (any; multiples of 8 take the vector stores).  status: optional device int, OR-ed with a
 * non-zero code if one of the kernel's bounded waits gave up (never expected).  Asynchronous on `stream`. */
AFB_API int afb_input_map_f16(int64_t n_in, int64_t batch, int64_t k_dim, const void *w, int64_t ldw, const void *x,
                              int64_t ldx, const void *b, float gain, void *u, int64_t ldu, int *status, void *stream);

/* ---- float32 GEMMs of the training path (chessfly/model.py:95-105 trained by chessfly/train.py:126-138) --
 * The reference trains its encoder and heads as float32 nn.Linear layers (their forward and the two
 * gradient products of each).  afb_gemm_f32 computes
 *     r[i * ld_r + j] = alpha * sum_{l < k} X[i, l] Y[j, l] + beta * bias        (i < p, j < q)
 * with X[i, l] = x[i * ld_x + l] (x_trans = 0) or x[l * ld_x + i] (x_trans = 1), Y likewise, and bias = 0
 * (bias_dim 0), bias[i] (1) or bias[j] (2).  float32 in and out, float32 accuracy (~1e-6 relative to the
 * largest products): each operand is scaled by a power of two and split into float16 hi and lo parts, the
 * products run on the tensor cores (tcgen05.mma) with two float32 accumulators.  workspace: at least
 * afb_gemm_workspace(p, q, k) bytes; one call at a time per workspace.  status: optional device int, OR-ed
 * with a non-zero code if one of the kernel's bounded waits gave up (never expected).  Asynchronous on
 * `stream`. */
AFB_API size_t afb_gemm_workspace(int64_t p, int64_t q, int64_t k);
AFB_API int afb_gemm_f32(int64_t p, int64_t q, int64_t k, float alpha, const float *x, int64_t ld_x, int x_trans,
                         const float *y, int64_t ld_y, int y_trans, const float *bias, int bias_dim, float beta, float *r,
                         int64_t ld_r, void *workspace, size_t workspace_bytes, int *status, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* AFB_H */
