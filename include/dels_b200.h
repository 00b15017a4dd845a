/*
 * dels_b200.h — C ABI of the B200-native DeLS draft-scoring hot path.
 *
 * Plain pointers, sizes and a CUDA stream handle; no framework types.  Every entry
 * point only enqueues work on `stream` (a cudaStream_t passed as void*): none
 * allocates device memory or synchronises the host, so all of them can be captured
 * in a CUDA graph (call dels_init() for the device once, before any capture).
 *
 * Conventions
 *   - bf16 tensors are row-major with a leading dimension `ld_*` in elements; it must
 *     be a multiple of 8 and base pointers 16-byte aligned (tensor-memory-access tiles).
 *   - fp32 tensors used by the fp32 scorer need 16-byte aligned rows (ld % 4 == 0).
 *   - alpha / beta are fp32 device arrays of length n_pos; row `i` uses position
 *     p = row_pos[i] when row_pos != NULL, else p = i % n_pos (rows laid out [B, P]).
 *   - `prior` is the fp32 log-unigram prior (the bf16-rounded values of the reference
 *     run are exactly representable); NULL skips the beta term, as the reference does
 *     when it has no baseline or beta == 0 (code/kernel/dels.py:382, :454).
 *   - Argmax ties go to the lowest vocabulary index (torch.argmax, and the strict '>'
 *     of code/kernel/dels.py:134); a NaN score is treated as the largest value.
 *   - Packed keys (int64): ((ordered score) << 32) | (0xFFFFFFFF - global index).  The
 *     signed maximum of two keys is the argmax of the two candidates, so per-rank keys
 *     combine with an all-reduce(MAX) on int64 (vocab sharding).
 *   - Workspace `ws`: caller-owned device memory, zero-filled once before first use.
 *     Bytes [0,4) are a completion counter (left at zero after every call), bytes [4,8)
 *     an int32 device status word: a kernel that gives up on a bounded wait stores
 *     DELS_ERR_DEVICE_TIMEOUT there; the status persists until the caller clears it.
 *
 * Return values: DELS_OK or a negative DELS_ERR_* code; dels_last_error() gives a
 * message for the calling thread's most recent failure.
 */
#ifndef DELS_B200_H_
#define DELS_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DELS_API __attribute__((visibility("default")))
#else
#define DELS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DELS_OK 0
#define DELS_ERR_INVALID_ARG (-1)
#define DELS_ERR_ALIGNMENT (-2)
#define DELS_ERR_WORKSPACE (-3)
#define DELS_ERR_CUDA (-4)
#define DELS_ERR_UNSUPPORTED (-5)
#define DELS_ERR_DEVICE_TIMEOUT (-6)

#define DELS_ACT_IDENTITY 0 /* code/dels.py:14 "identity" */
#define DELS_ACT_SILU 1     /* code/dels.py:14 "silu"     */

/* keys[] already hold the empty key (set by dels_rank_project_bf16 / dels_keys_init). */
#define DELS_FLAG_KEYS_READY 1u

#define DELS_WS_HEADER_BYTES 256

DELS_API int dels_version(void);
DELS_API const char* dels_status_string(int status);
DELS_API const char* dels_last_error(void);

/* Load every kernel of the library on `device` and set its launch attributes.  Call
 * before the first CUDA-graph capture that contains a dels_* call. */
DELS_API int dels_init(int device);

/* Number of streaming multiprocessors the persistent kernels size their grids for. */
DELS_API int dels_sm_count(int device);

/* ---------------------------------------------------------------------------------
 * Rank projection.  Replaces code/kernel/dels.py:437-439
 *   rank_state = F.linear(h, W_rank); rank_state = F.silu(rank_state) (optional)
 * and produces the scorer operand alpha_p * rank_state.
 *   x        [rows, K] bf16 (ld_x)       w_rank [r, K] bf16 (ld_w), nn.Linear layout
 *   s_out    [rows, r] bf16 or NULL      s = bf16(act(bf16(x . w_rank^T)))
 *   s_scaled [rows, r] bf16              bf16(alpha_p * s)
 *   keys     [rows] int64 or NULL        set to the empty key (saves an init launch)
 * Tensor-core split-K GEMM + SIMT finalisation; ws >= dels_rank_workspace_bytes().
 * --------------------------------------------------------------------------------- */
DELS_API size_t dels_rank_workspace_bytes(int rows, int K, int r);
DELS_API int dels_rank_project_bf16(const void* x, int64_t ld_x, const void* w_rank, int64_t ld_w, int rows, int K, int r,
                           int activation, const float* alpha, int n_pos, const int32_t* row_pos, void* s_out,
                           void* s_scaled, int64_t* keys, void* ws, size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------------
 * Fused draft scorer, bf16 tensor cores.  Replaces
 * _fused_low_rank_argmax_kernel + _reduce_argmax_kernel (code/kernel/dels.py:15-138,
 * launched at :375-423) and the long-logit GEMM code/dflash.py:468, without ever
 * materialising logits:
 *   score[i, v] = h[i] . W[v] + s_scaled[i] . Vr[v] - beta_p * prior[v]
 *   keys[i]     = max over v of pack(score[i, v], v_begin + v)     (atomicMax)
 *   idx_out[i]  = argmax index (int64), score_out[i] = its score   (either may be NULL)
 *   h [rows, H] bf16, W [V, H] bf16 (the target LM head, or this rank's vocab slice
 *   starting at global index v_begin), s_scaled [rows, r] bf16, Vr [V, r] bf16
 *   (low_rank_lm_head.weight), prior [V] fp32 or NULL.
 * rows_dev (optional) holds the actual row count on the device (<= rows), so a ragged
 * batch needs no host round trip.  With idx_out == NULL the keys are left for a
 * cross-rank all-reduce(MAX) followed by dels_keys_decode().  H == 0 drops the W.h
 * term.  ws >= DELS_WS_HEADER_BYTES.
 * --------------------------------------------------------------------------------- */
DELS_API int dels_fused_argmax_bf16(const void* h, int64_t ld_h, const void* W, int64_t ld_w, const void* s_scaled,
                           int64_t ld_s, const void* Vr, int64_t ld_vr, const float* prior, const float* beta,
                           int n_pos, const int32_t* row_pos, int rows, const int32_t* rows_dev, int H, int r,
                           int V, int64_t v_begin, uint32_t flags, int64_t* keys, int64_t* idx_out,
                           float* score_out, void* ws, size_t ws_bytes, void* stream);

/* Base-logits variant: the exact DeLSGraphRunner step (code/kernel/dels.py:70-90),
 *   score[i, v] = base[i, v] + s_scaled[i] . Vr[v] - beta_p * prior[v]
 * with base [rows, V] bf16 (ld_base), e.g. static_base_logits[:, step, :]. */
DELS_API int dels_fused_argmax_base_bf16(const void* base, int64_t ld_base, const void* s_scaled, int64_t ld_s,
                                const void* Vr, int64_t ld_vr, const float* prior, const float* beta, int n_pos,
                                const int32_t* row_pos, int rows, const int32_t* rows_dev, int r, int V,
                                int64_t v_begin, uint32_t flags, int64_t* keys, int64_t* idx_out,
                                float* score_out, void* ws, size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------------
 * Whole draft-scoring step, bf16 (dense, ragged and vocab-sharded batches): rank projection
 * s = act(h . w_rank^T) then the fused scorer.  Replaces one step of
 * DeLSGraphRunner._forward_impl (code/kernel/dels.py:436-458) with the long logits of
 * code/dflash.py:468 folded in; the eager twin is code/dflash.py:516-534.
 * ws >= dels_score_workspace_bytes(rows, H, r).
 * --------------------------------------------------------------------------------- */
DELS_API size_t dels_score_workspace_bytes(int rows, int H, int r);
DELS_API int dels_draft_score_bf16(const void* h, int64_t ld_h, const void* W, int64_t ld_w, const void* w_rank,
                          int64_t ld_wr, const void* Vr, int64_t ld_vr, const float* prior, const float* alpha,
                          const float* beta, int n_pos, const int32_t* row_pos, int rows, const int32_t* rows_dev,
                          int H, int r, int V, int64_t v_begin, int activation, int64_t* keys, int64_t* idx_out,
                          float* score_out, void* ws, size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------------
 * fp32 draft scorer on CUDA cores (fp32 workloads; scores within 1e-5).  Same
 * formula as dels_draft_score_bf16 with every tensor fp32 and s kept in fp32:
 *   s[i] = alpha_p * (h[i] . w_rank^T),  score = h.W[v] + s.Vr[v] - beta_p prior[v].
 * H % 4 == 0, r % 4 == 0.  ws >= dels_score_f32_workspace_bytes(rows, H, r).
 * --------------------------------------------------------------------------------- */
DELS_API size_t dels_score_f32_workspace_bytes(int rows, int H, int r);
DELS_API int dels_draft_score_f32(const float* h, int64_t ld_h, const float* W, int64_t ld_w, const float* w_rank,
                         int64_t ld_wr, const float* Vr, int64_t ld_vr, const float* prior, const float* alpha,
                         const float* beta, int n_pos, const int32_t* row_pos, int rows, int H, int r, int V,
                         int64_t v_begin, int64_t* keys, int64_t* idx_out, float* score_out, void* ws,
                         size_t ws_bytes, void* stream);

/* Set keys[0..rows) to the empty key and zero the workspace counter. */
DELS_API int dels_keys_init(int64_t* keys, int rows, void* ws, void* stream);

/* Decode packed keys (e.g. after a cross-rank all-reduce(MAX)) into int64 token ids
 * and fp32 scores (either output may be NULL).  rows_dev as above. */
DELS_API int dels_keys_decode(const int64_t* keys, int rows, const int32_t* rows_dev, int64_t* idx_out, float* score_out,
                     void* stream);

/* Health check of the device-side bounded waits (no counterpart in the reference).
 * Launches one CTA in which one thread waits on an mbarrier that nothing completes,
 * giving up after limit_ms (0 < limit_ms <= 1000), and a second thread on another such
 * barrier that must leave as soon as the first raises the CTA's abort flag.  Afterwards
 * *status (device int, zero before the call) holds DELS_ERR_DEVICE_TIMEOUT and
 * waited_ns[0..1] (device uint64) how long each waited.  No fault, trap or hang: the
 * context stays usable. */
DELS_API int dels_selftest_bounded_wait(int* status, uint64_t* waited_ns, double limit_ms, void* stream);

/* ---------------------------------------------------------------------------------
 * Acceptance.  Replaces code/dflash.py:645-651
 *   accept = (verify_ids[:, 1:] == posterior[:, :-1]).cumprod(1).sum(1)
 * for a ragged continuous batch, without the host round trip of `.item()`:
 *   draft [n_seq, n_draft] int64 (ld_draft), target [n_seq, >= n_draft] int64
 *   accept[b]  = length of the prefix on which draft[b, j] == target[b, j]   (int32)
 *   offsets[0] = 0, offsets[b+1] = offsets[b] + accept[b] + commit_extra     (int32)
 * commit_extra = 1 counts the bonus target token the decode loop also commits
 * (code/dflash.py:652-660).
 * --------------------------------------------------------------------------------- */
DELS_API int dels_accept_offsets(const int64_t* draft, int64_t ld_draft, const int64_t* target, int64_t ld_target,
                        int n_seq, int n_draft, int commit_extra, int32_t* accept, int32_t* offsets, void* stream);

/* Pack the accepted rows of hidden [n_seq, P, H] bf16 (strides ld_seq, ld_row in
 * elements): packed[offsets[b] + j] = hidden[b, j] for j < accept[b], row_pos of that
 * packed row = j.  Use offsets from dels_accept_offsets(commit_extra = 0); the total
 * row count offsets[n_seq] can be passed to the scorer as rows_dev. */
DELS_API int dels_pack_rows_bf16(const void* hidden, int64_t ld_seq, int64_t ld_row, int n_seq, int P, int H,
                        const int32_t* accept, const int32_t* offsets, void* packed, int64_t ld_packed,
                        int32_t* row_pos, void* stream);

/* ---------------------------------------------------------------------------------
 * Input-projected RNN local head (a recurrence over the block positions; the reference only has the GRU
 * form, code/kernel/dels.py:359-373, whose input projection is likewise precomputed
 * at :265-268):
 *   s_t = tanh(W_in x_t + W_s s_{t-1} + b), s_0 = 0, for t = 0..T-1 of each sequence
 *   x [n_seq*T, H] bf16 (rows in [seq, t] order), w_in [r, H] bf16, w_s [r, r] bf16,
 *   bias [r] fp32 or NULL, alpha [T] fp32.
 *   s_scaled [n_seq*T, r] bf16 = bf16(alpha_t * s_t); s_out (optional) = bf16(s_t).
 * r even and <= 256.  ws >= dels_rnn_workspace_bytes(n_seq, T, H, r).
 * --------------------------------------------------------------------------------- */
DELS_API size_t dels_rnn_workspace_bytes(int n_seq, int T, int H, int r);
DELS_API int dels_rnn_rank_states_bf16(const void* x, int64_t ld_x, const void* w_in, int64_t ld_win, const void* w_s,
                              const float* bias, const float* alpha, int n_seq, int T, int H, int r,
                              void* s_scaled, void* s_out, int64_t* keys, void* ws, size_t ws_bytes,
                              void* stream);

/* ---------------------------------------------------------------------------------
 * Small-batch kernels of the greedy suffix rollout captured by DeLSGraphRunner /
 * MarkovDeLSGraphRunner (B rows, typically 1..64).
 *
 * GRU step — replaces DeLSGraphRunner._gru_cell + the input-table gather
 * (code/kernel/dels.py:359-373, :432, :461; Triton cell :140-211):
 *   gi = gi_table[tokens[b * tok_stride]]   ([V, 3G] bf16 = F.linear(embed, W_ih, b_ih))
 *   gh = bf16(W_hh . h_in[b] + b_hh)        (W_hh [3G, G] bf16, b_hh [3G] bf16 or NULL)
 *   r, z = sigmoid(gi + gh) (first two G-blocks), n = tanh(gi_n + r * gh_n)
 *   h_out[b] = bf16((1 - z) * n + z * h_in[b])      (h_in NULL = zero state)
 * G % 8 == 0.  Out-of-range token ids are clamped and flagged in the ws status word
 * (DELS_ERR_INVALID_ARG) when ws is given.  token_keys != 0: tokens[] holds the previous
 * step's packed (score, index) argmax keys, decoded here. */
DELS_API int dels_gru_step_bf16(const int64_t* tokens, int64_t tok_stride, int token_keys, const void* gi_table,
                                int64_t ld_table, const void* w_hh, const void* b_hh, const void* h_in, void* h_out,
                                int B, int G, int V, void* ws, void* stream);

/* The gates of the same GRU step when gh = bf16(W_hh . h_in + b_hh) [B, 3G] (row stride
 * ld_gh) was computed separately, e.g. by dels_linear_bf16 for larger batches, where the
 * tensor-core projection beats one warp per gate row (code/kernel/dels.py:368-373):
 *   r, z = sigmoid(gi + gh), n = tanh(gi_n + r * gh_n), h_out[b] = bf16((1 - z) n + z h_in[b]),
 * gi = gi_table[tokens[b * tok_stride]], h_in NULL = zero state.  Out-of-range ids are
 * clamped and flagged as in dels_gru_step_bf16.  token_keys != 0: tokens[] holds the
 * previous step's packed (score, index) argmax keys, decoded here. */
DELS_API int dels_gru_gates_bf16(const int64_t* tokens, int64_t tok_stride, int token_keys, const void* gi_table,
                                 int64_t ld_table, const void* gh, int64_t ld_gh, const void* h_in, void* h_out,
                                 int B, int G, int V, void* ws, void* stream);

/* The same GRU step for larger batches in two launches: gh = W_hh . h_in as a tensor-core
 * split-K GEMM into fp32 partials (the workspace), then one kernel that sums each unit's
 * three gate columns in split order, adds b_hh (NULL = none) and rounds to bf16 exactly as
 * dels_linear_bf16 writes gh, and evaluates the gates as dels_gru_gates_bf16 does:
 * h_out bit-identical to dels_linear_bf16 followed by dels_gru_gates_bf16.  h_in and w_hh
 * row-major with row stride G (16-byte rows, G % 8 == 0); h_in must not be NULL;
 * token_keys as in dels_gru_gates_bf16. */
DELS_API size_t dels_gru_step_tc_workspace_bytes(int B, int G);
DELS_API int dels_gru_step_tc_bf16(const int64_t* tokens, int64_t tok_stride, int token_keys, const void* gi_table,
                                   int64_t ld_table, const void* w_hh, const void* b_hh, const void* h_in, void* h_out,
                                   int B, int G, int V, void* ws, size_t ws_bytes, void* stream);

/* Rank projection for small batches (code/kernel/dels.py:437-443):
 *   s = bf16(act(bf16(x . w^T + bias))), s_scaled = bf16(alpha_p * s), keys[0..B) reset,
 * one warp per output feature.  K % 8 == 0.  ws (optional) supplies the counter that
 * the following scorer call expects at zero. */
DELS_API int dels_rank_gemv_bf16(const void* x, int64_t ld_x, const void* w, int64_t ld_w, const void* bias, int B,
                                 int K, int r, int activation, const float* alpha, int n_pos,
                                 const int32_t* row_pos, void* s_out, void* s_scaled, int64_t* keys, void* ws,
                                 void* stream);

/* The base-logit scorer of one rollout step (dels_fused_argmax_base_bf16, row positions
 * 0..rows-1, v_begin 0, no score output) with the NEXT step's GRU hidden projection in the
 * same launch: gh_out[b] = bf16(w_hh . h[b] + b_hh), w_hh [3G, G], h [rows, G] (the
 * state after this step's GRU update), gh_out [rows, 3G] (code/kernel/dels.py:366,
 * F.linear(h_state, W_hh, b_hh)).  It needs h but not this step's token, so two extra
 * warps per CTA compute it while the others score, and the next step's GRU gates
 * (dels_gru_gates_bf16 or dels_gru_rank_gemv_bf16) start from it.  At most 8 rows; G % 8 == 0. */
DELS_API int dels_fused_argmax_base_gru_bf16(const void* base, int64_t ld_base, const void* s_scaled, int64_t ld_s,
                                             const void* Vr, int64_t ld_vr, const float* prior, const float* beta,
                                             int n_pos, int rows, int r, int V, uint32_t flags, int64_t* keys,
                                             int64_t* idx_out, void* ws, size_t ws_bytes, const void* w_hh,
                                             const void* b_hh, const void* h, int G, void* gh_out, void* stream);

/* One small-batch rollout step's GRU gates fused into its rank projection
 * (code/kernel/dels.py:368-373 then :437-443):
 *   h_out[b] = GRU gates of (gi = gi_table[tokens[b * tok_stride]], gh[b], h_in[b]) as in
 *   dels_gru_gates_bf16, then s = bf16(act(bf16(w_rank . h_out[b] + bias))),
 *   s_scaled[b] = bf16(alpha[0] * s), keys[0..B) reset, as in dels_rank_gemv_bf16.
 * gh = bf16(W_hh h_in + b_hh) comes from an earlier call (dels_rank_gemv_bf16 with
 * w = W_hh, bias = b_hh, identity activation and alpha NULL), which can run beside the
 * previous step's scorer since it does not need that step's token.  Every CTA evaluates
 * the gates for all B rows itself; G, ld_table, ld_gh % 8 == 0, 16-byte aligned rows.
 * ws (optional) supplies the counter that the following scorer call expects at zero and
 * the status word for out-of-range token ids (clamped).  token_keys != 0: tokens[] holds
 * the previous step's packed argmax keys (a keys-only scorer call, idx_out NULL), decoded
 * here, so the rollout's scorer needs no in-kernel decode (its last-CTA count and fences)
 * and one dels_keys_decode per call yields all the tokens. */
DELS_API int dels_gru_rank_gemv_bf16(const int64_t* tokens, int64_t tok_stride, int token_keys, const void* gi_table,
                                     int64_t ld_table, const void* gh, int64_t ld_gh, const void* h_in, void* h_out,
                                     int B, int G, int V, const void* w_rank, int64_t ld_w, const void* bias, int r,
                                     int activation, const float* alpha, void* s_scaled, int64_t* keys, void* ws,
                                     void* stream);

/* The same fusion for the Domino correction runner: the GRU gates of the previous token
 * (code/kernel/domino.py:423-435) into the correction MLP's hidden layer of the next step
 * (:402, :92-97),
 * h_out as in dels_gru_rank_gemv_bf16, then s_scaled[b] = bf16(alpha[0] * SiLU(z[b] +
 * bf16(w_s . h_out[b]))) and keys[0..B) reset as in dels_correction_mid_bf16; token_keys
 * as above. */
DELS_API int dels_gru_correction_mid_bf16(const int64_t* tokens, int64_t tok_stride, int token_keys, const void* gi_table,
                                          int64_t ld_table, const void* gh, int64_t ld_gh, const void* h_in,
                                          void* h_out, int B, int G, int V, const void* w_s, int64_t ld_ws,
                                          const void* z, int64_t ld_z, int M, const float* alpha, void* s_scaled,
                                          int64_t* keys, void* ws, void* stream);

/* Markov rank state (code/kernel/markov_dels.py:288):
 *   s_scaled[b] = bf16(alpha_p * emb[tokens[b * tok_stride]]),  emb [V, r] bf16,
 * keys[0..B) reset.  Out-of-range ids are clamped and flagged as above.  token_keys != 0:
 * tokens[] holds the previous step's packed (score, index) argmax keys, decoded here (a
 * keys-only rollout, as in dels_gru_rank_gemv_bf16). */
DELS_API int dels_gather_scaled_rows_bf16(const int64_t* tokens, int64_t tok_stride, int token_keys, const void* emb,
                                          int64_t ld_emb, const float* alpha, int n_pos, int B, int r, int V,
                                          void* s_scaled, int64_t* keys, void* ws, void* stream);

/* ---------------------------------------------------------------------------------
 * Domino draft-correction rollout (code/kernel/domino.py:232-520).  Per step the
 * correction MLP's logits are alpha * (SiLU(z_t + W_s h) . fc2^T + b2) + base_t; the
 * step runs dels_correction_mid_bf16 (below), then dels_fused_argmax_base_bf16 with
 * Vr = fc2 [V, M], prior = b2 as fp32 and beta = -alpha (so -beta * prior = alpha * b2),
 * then dels_gru_step_bf16 on the chosen token.
 * --------------------------------------------------------------------------------- */

/* F.linear with an optional bias (code/kernel/domino.py:404-408 z = F.linear(hiddens,
 * W_z, b1); :325-327 and code/kernel/dels.py:265-268, the GRU input table;
 * code/dflash.py:468, the long logits lm_head(parallel_hiddens)):
 *   out[row] = bf16(x[row] . w^T + bias)     x [rows, K], w [N, K], bias [N] bf16 or NULL,
 * one rounding of the fp32 accumulator (bias included), like the bf16 GEMM's bias
 * epilogue.  tcgen05 split-K GEMM with deterministic fp32 partials in ws, then the
 * finalisation; when the output tiles alone fill the device (vocabulary-sized N) K is not
 * split and the GEMM writes the bf16 result itself (same values, one launch, ws = the
 * header only).  ws >= dels_linear_workspace_bytes(rows, K, N). */
DELS_API size_t dels_linear_workspace_bytes(int rows, int K, int N);
DELS_API int dels_linear_bf16(const void* x, int64_t ld_x, const void* w, int64_t ld_w, const void* bias, int rows,
                              int K, int N, void* out, int64_t ld_out, void* ws, size_t ws_bytes, void* stream);

/* The correction MLP's hidden layer for one step (code/kernel/domino.py:422 s_proj =
 * F.linear(h, W_s); :92-97 SiLU(z + s) in fp32; :113 the guidance alpha):
 *   s = bf16(W_s . h[b]),  mid = SiLU(z[b] + s) (fp32),  s_scaled[b] = bf16(alpha[0] * mid),
 * h [B, G], W_s [M, G], z [B, M] (row stride ld_z), keys[0..B) reset.  G % 8 == 0.
 * ws (optional) supplies the counter that the following scorer call expects at zero. */
DELS_API int dels_correction_mid_bf16(const void* h, int64_t ld_h, const void* w_s, int64_t ld_ws, const void* z,
                                      int64_t ld_z, int B, int G, int M, const float* alpha, void* s_scaled,
                                      int64_t* keys, void* ws, void* stream);

/* The same layer for larger batches, where one warp per output row does not scale: s =
 * W_s . h[b] by the tensor-core split-K projection GEMM, then the same epilogue
 * (s_scaled[b] = bf16(alpha[0] * SiLU(z[b] + bf16(s))), keys[0..B) reset).  G % 8 == 0;
 * ws >= dels_correction_mid_tc_workspace_bytes(B, G, M). */
DELS_API size_t dels_correction_mid_tc_workspace_bytes(int B, int G, int M);
DELS_API int dels_correction_mid_tc_bf16(const void* h, int64_t ld_h, const void* w_s, int64_t ld_ws, const void* z,
                                         int64_t ld_z, int B, int G, int M, const float* alpha, void* s_scaled,
                                         int64_t* keys, void* ws, size_t ws_bytes, void* stream);

/* ---------------------------------------------------------------------------------
 * Allocation-free variant of dels_draft_score_bf16 (no counterpart in the reference).
 * For callers that cannot hand the library device memory — an FFI host without a
 * device allocator, or a serving engine whose memory pool already owns the device —
 * the scratch lives in a fixed array of DELS_NOALLOC_SCRATCH_BYTES that is part of the
 * library's device module: it is reserved on every device on which that module is
 * loaded, whether or not this entry point is called, until the process exits.  Same
 * arguments and results as dels_draft_score_bf16 without ws / ws_bytes; shapes whose
 * dels_score_workspace_bytes(rows, H, r) exceeds the array are rejected with
 * DELS_ERR_WORKSPACE (the Qwen3-8B block batch, 512 x 4096 x 256, fits).  Each call
 * looks up the array's device address in the current context; the first call on a
 * device may load the module, so make it before any stream capture.  All calls share
 * the one array: calls that may overlap on the device race, so serialise them.  Never
 * calls cudaMalloc / cudaFree.
 * --------------------------------------------------------------------------------- */
#define DELS_NOALLOC_SCRATCH_BYTES (12u * 1024u * 1024u)
DELS_API int dels_draft_score_bf16_noalloc(const void* h, int64_t ld_h, const void* W, int64_t ld_w,
                                           const void* w_rank, int64_t ld_wr, const void* Vr, int64_t ld_vr,
                                           const float* prior, const float* alpha, const float* beta, int n_pos,
                                           const int32_t* row_pos, int rows, const int32_t* rows_dev, int H, int r,
                                           int V, int64_t v_begin, int activation, int64_t* keys, int64_t* idx_out,
                                           float* score_out, void* stream);

/* Device status word of the allocation-free entry point (no counterpart in the
 * reference): the counterpart of the workspace status word at bytes [4, 8) of a caller
 * workspace.  A kernel of dels_draft_score_bf16_noalloc that gives up on a bounded wait
 * stores DELS_ERR_DEVICE_TIMEOUT there, and the word stays set across calls until it
 * is cleared.  Enqueues on `stream` one single-thread kernel that writes the word to
 * *status_out (an int the GPU can write: device memory or mapped pinned host memory;
 * NULL to only clear) and, when `clear` != 0, resets it to 0.  Read *status_out after
 * the stream has reached this point. */
DELS_API int dels_noalloc_status(int* status_out, int clear, void* stream);

/* dels_selftest_bounded_wait with the allocation-free status word as its status: lets a
 * caller (and the test suite) check that a device timeout there is seen and cleared by
 * dels_noalloc_status.  No fault, trap or hang. */
DELS_API int dels_selftest_bounded_wait_noalloc(uint64_t* waited_ns, double limit_ms, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DELS_B200_H_ */
