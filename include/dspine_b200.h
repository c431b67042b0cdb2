/*
 * dspine_b200.h -- C ABI of the B200 draft-block verification library (libdspine_b200.so).
 *
 * Every entry point takes device pointers, sizes and a cudaStream_t, enqueues its work on that
 * stream and returns a dsv_status (0 = success).  Arguments are validated on the host before
 * anything is launched; nothing here synchronizes the stream unless stated.  Outputs are
 * caller-owned buffers; inputs are never modified.
 *
 * Each declaration names the reference interface it replaces (paths inside the reference
 * project, package sglang_dspine).
 */
#ifndef DSPINE_B200_H
#define DSPINE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* dsv_stream_t; /* == cudaStream_t */

typedef enum {
    DSV_OK = 0,
    DSV_BAD_SHAPE = 1,
    DSV_BAD_DTYPE = 2,
    DSV_BAD_POINTER = 3,
    DSV_BAD_ALIGNMENT = 4,
    DSV_LAUNCH_FAILED = 5,
    DSV_WORKSPACE_TOO_SMALL = 6,
    DSV_DEVICE_TIMEOUT = 7,
    DSV_UNSUPPORTED = 8
} dsv_status;

typedef enum { DSV_BF16 = 0, DSV_F32 = 1 } dsv_dtype;

/* Filter modes of the target distribution (runtime/worker.py:473-508 filter_target_probs):
 * JOINT  flashinfer backend, no min-p in the batch: rank < top_k and mass ranked ahead <= top_p,
 *        both on the unfiltered p;
 * SEQ    flashinfer backend with min-p in the batch (need_min_p_sampling): top-k, then top-p
 *        against the top-k's own mass, then p >= min_p * max p;
 * TORCH  pytorch backend (runtime/worker.py:52-67): the joint top-k / top-p set and
 *        p >= min_p * max p.
 * The min-p test is e >= min_p with e = exp2c((l - m) c); the floor is found by bisection over
 * the 32-bit ordered keys (so the kept set stays a prefix of the rank order). */
typedef enum { DSV_FILTER_JOINT = 0, DSV_FILTER_SEQ = 1, DSV_FILTER_TORCH = 2 } dsv_filter_mode;

/* Library version string and a readable name for a status code. */
const char* dsv_version(void);
const char* dsv_status_string(int status);
/* Kernels this process has enqueued through the library so far (all entry points, all
 * devices); a diagnostic for benchmarks.  No counterpart in the reference. */
uint64_t dsv_launch_count(void);

/* ---- workspace ----------------------------------------------------------------------------
 * Scratch for dsv_verify_logits: task counters, per-row decisions, the ready list of requests
 * and (last 8.5 MB) the slots through which the two halves of a split row meet.  Zero it once
 * after allocation (dsv_workspace_init); every launch that ends without an internal failure
 * (error bits 0, 5-7 below) leaves it zeroed again for the next launch with the same batch
 * size, except for a counter of the logit bytes read (dsv_workspace_bytes_read).  Its regions
 * are laid out by the batch size, so a workspace sized for the largest batch serves smaller
 * ones, but must be zeroed again when the batch size changes.  A workspace without the
 * split-row slots (the size for the batch minus that region) is accepted and then no row is
 * split. */
int dsv_verify_workspace_size(int32_t batch, size_t* bytes);
int dsv_workspace_init(void* workspace, size_t bytes, dsv_stream_t stream);
/* Copy the device error word of a workspace to *err and clear it (synchronizes `stream`).
 * bit 0: a shared-memory bulk copy did not complete within its time limit;
 * bit 1: a request addressed a row outside the logit tensors. */
int dsv_workspace_error(void* workspace, uint32_t* err, dsv_stream_t stream);
/* Logit bytes that verifications and bf16 target-probability calls through this workspace
 * have read from memory since it was last zeroed (synchronizes `stream`).  Verification takes
 * the rows in verify-position order across the batch and drops the rows after a step already
 * known to be rejected (the chain stops there) and, for bf16 logits, the rows of a request
 * whose outcome is already known, when it reaches them or while it reads them: those rows
 * cannot change any output.  No counterpart in the reference (a diagnostic). */
int dsv_workspace_bytes_read(const void* workspace, uint64_t* bytes, dsv_stream_t stream);
/* Host -> device copy of row ranges between two buffers of the same row layout (row_bytes
 * apart): range i is rows [first_row[i], first_row[i] + n_rows[i]); ranges that continue one
 * another are merged; one cudaMemcpyAsync per merged range on `stream` (pinned host memory
 * makes them asynchronous).  The staged copies of dspine_b200.verify.verify_logits_host,
 * which sends to the device only the logit rows the outcome can depend on.  No counterpart in
 * the reference (SGLang's logits are on the device). */
int dsv_copy_row_ranges(void* dst, const void* src, size_t row_bytes, int32_t n,
                        const int64_t* first_row, const int64_t* n_rows, dsv_stream_t stream);
/* bit 2 of the error word: a compaction read a KV slot position outside `slots_len`;
 * bits 3-4: a selection or a tie cut found no boundary (inconsistent input); bit 6: a chain
 * task waited past its time limit for its request; bit 7: the second half of a split row
 * waited past its time limit for the first.  Bits 0 and 5-7 are internal failures: the
 * outputs of that call are not valid, and the workspace's counters and split-row flags may be
 * left set (a late first half can raise its flag after the second gave up), so zero the
 * workspace again (dsv_workspace_init) before its next use. */

/* ---- accept-compact outputs (optional argument of dsv_verify_logits) ----------------------
 * Restates SGLang's commit of accepted tokens and KV slots (wrapped by the reference at
 * runtime/worker.py:745-777): request b keeps tokens output[b, :commit_b] and the KV slots of
 * its verify positions [0, commit_b); positions [commit_b, verify_len_b) are freed. */
typedef struct {
    const int32_t* slots;     /* KV slot of verify position s of request b: slots[slot_row[b]+s] */
    int64_t slots_len;        /* entries in `slots`; positions outside it read as -1 */
    const int64_t* slot_row;  /* [B] */
    int64_t* tokens;          /* [B*16] accepted tokens, request-major (first sum(commit) used) */
    int32_t* kept_slots;      /* [B*16] */
    int32_t* offsets;         /* [B+1] exclusive scan of commit */
    int32_t* freed_slots;     /* [B*16] */
    int32_t* freed_offsets;   /* [B+1] */
} dsv_compact_out;

/* ---- fused verification from logits -------------------------------------------------------
 * Replaces runtime/worker.py:440-508 build_dspine_target_probs (flashinfer backend, min-p off:
 * temperature softmax, joint top-k/top-p, greedy rows one-hot at the lowest-index argmax)
 * followed by the capped chain rejection of sampling/rejection.py:12-98
 * (_sample_capped_chain; the dense-q path of runtime/worker.py:511-581 dspine_accept_sampling).
 *
 * Target row of (request b, position s) is target_row[b] + s; its draft row (the distribution
 * draft s+1 was sampled from: the same temperature/top-k/top-p applied to draft logits) is
 * draft_row[b] + s.  draft_logits == NULL, or a greedy request (top_k <= 1 or temperature <= 0),
 * means q is one-hot at the drafted token.  Rows hold `vocab` logits of `dtype`, `row_stride`
 * elements apart.  Outputs as sample_capped_chain_from_probs (sampling/rejection.py:101-153):
 * accept i32[B], commit i32[B], bonus i64[B], output i64[B,16], new_seq i32[B].
 * Sums that feed decisions are exact (2^-40 fixed point), so results do not depend on launch
 * shape.  `compact` may be NULL. */
int dsv_verify_logits(int32_t batch, int32_t vocab, int32_t dtype, const int64_t* candidates,
                      const void* target_logits, const int64_t* target_row, int64_t target_rows,
                      const void* draft_logits, const int64_t* draft_row, int64_t draft_rows,
                      int64_t row_stride, const float* temperature, const int32_t* top_k,
                      const float* top_p, const int32_t* verify_lens, const float* uniforms,
                      const float* uniform_final, const int32_t* prefix_lens, int32_t* accept,
                      int32_t* commit, int64_t* bonus, int64_t* output, int32_t* new_seq,
                      const dsv_compact_out* compact, void* workspace, size_t workspace_bytes,
                      dsv_stream_t stream);

/* The same verification with min-p and a filter mode (dsv_filter_mode): min_p [B] (NULL, or
 * 0 for a request, means no min-p floor; ignored in the JOINT mode).  Replaces the other
 * branches of runtime/worker.py:473-508 filter_target_probs (min-p on: :485-491; the pytorch
 * backend: :52-67, :480-484).  dsv_verify_logits is this call with min_p NULL and JOINT. */
int dsv_verify_logits_ex(int32_t batch, int32_t vocab, int32_t dtype, const int64_t* candidates,
                         const void* target_logits, const int64_t* target_row,
                         int64_t target_rows, const void* draft_logits, const int64_t* draft_row,
                         int64_t draft_rows, int64_t row_stride, const float* temperature,
                         const int32_t* top_k, const float* top_p, const float* min_p,
                         int32_t filter_mode, const int32_t* verify_lens, const float* uniforms,
                         const float* uniform_final, const int32_t* prefix_lens, int32_t* accept,
                         int32_t* commit, int64_t* bonus, int64_t* output, int32_t* new_seq,
                         const dsv_compact_out* compact, void* workspace,
                         size_t workspace_bytes, dsv_stream_t stream);

/* ---- draft LM head fused with top-k and logsumexp --------------------------------------------
 * Replaces the materialised `torch.matmul(rows, W.T)` of runtime/worker.py:283-285 followed by
 * kernels/dspine.py:165-207 topk_ids (and, per vocabulary shard, the local candidates that
 * sampling/tp_head.py:76-82 TPHead.global_topk merges).  hidden_states [rows, hidden] and
 * weight [vocab, hidden] are bf16 (hidden a multiple of 64, row pitches multiples of 8
 * elements, 16-byte aligned bases); the [rows, vocab] logits are never written.
 * Per row: the k (<= 32) largest logits ranked by their bf16 value (the value torch.matmul
 * materialises), ties to the lower index, as ids (column + id_offset; pad_id where vocab < k)
 * and values (fp32 holding the bf16-rounded logit); lse (optional) = logsumexp of the fp32
 * logits.  sort_ids = 0 gives rank order, 1 ids ascending (topk_ids order).  The workspace
 * (dsv_lmhead_workspace_size) holds per-CTA partial lists and the error word of
 * dsv_workspace_error; zero it once (dsv_workspace_init). */
int dsv_lmhead_workspace_size(int32_t rows, int32_t vocab, int32_t k, size_t* bytes);
int dsv_lmhead_topk(int32_t rows, int32_t vocab, int32_t hidden, int32_t k,
                    const void* hidden_states, int64_t hidden_stride, const void* weight,
                    int64_t weight_stride, int64_t id_offset, int64_t pad_id, int32_t sort_ids,
                    int64_t* ids, float* values, float* lse, void* workspace,
                    size_t workspace_bytes, dsv_stream_t stream);

/* ---- vocab-parallel merge --------------------------------------------------------------------
 * Replaces sampling/tp_head.py:9-14 merge_topk over the all-gathered shard candidates: shard s
 * contributes, for row r, k candidates (rank order) at values[s * values_shard_stride + r * k],
 * ids[s * ids_shard_stride + r * k] and its logsumexp lse[s * lse_shard_stride + r].  Output per
 * row: the global top-k by (value desc, id asc) and the global logsumexp; identical on every
 * rank that merges the same gathered buffer. */
int dsv_tp_merge(int32_t rows, int32_t shards, int32_t k, const float* values,
                 int64_t values_shard_stride, const int64_t* ids, int64_t ids_shard_stride,
                 const float* lse, int64_t lse_shard_stride, int64_t pad_id, int32_t sort_ids,
                 int64_t* out_ids, float* out_values, float* out_lse, dsv_stream_t stream);

/* ---- target probabilities from logits --------------------------------------------------------
 * Replaces runtime/worker.py:440-508 build_dspine_target_probs / filter_target_probs (SoftmaxTemp
 * + joint top-k / top-p, greedy rows one-hot at the lowest-index argmax) as a standalone step:
 * logits [rows, vocab] bf16 (rows row_stride elements apart), request r = rows
 * [r * rows_per_request, (r+1) * rows_per_request) with temperature[r], top_k[r], top_p[r]
 * (rows_per_request <= 16, rows a multiple of it); probs [rows, vocab] fp32 with the exact
 * canonical kept set and p_i = exp2c((l_i - m) c) * (1 / S_kept).  The workspace is a
 * dsv_verify_logits workspace for min(rows / rows_per_request, 1024) requests. */
int dsv_target_probs(int64_t rows, int32_t vocab, int32_t rows_per_request, const void* logits,
                     int64_t row_stride, const float* temperature, const int32_t* top_k,
                     const float* top_p, float* probs, void* workspace, size_t workspace_bytes,
                     dsv_stream_t stream);

/* dsv_target_probs for bf16 or fp32 logits (dtype), with min-p and a filter mode (see
 * dsv_verify_logits_ex): min_p per request or NULL.  bf16 rows with vocab <= 262000 and
 * rows_per_request <= 16 take the streaming row kernel and need a dsv_verify_logits workspace
 * for min(requests, 1024) requests; other rows (fp32, larger vocabularies, any
 * rows_per_request) take one 8-CTA cluster per row and use only the first 64 bytes of a zeroed
 * workspace (vocab up to about 220000 for fp32). */
int dsv_target_probs_ex(int64_t rows, int32_t vocab, int32_t dtype, int32_t rows_per_request,
                        const void* logits, int64_t row_stride, const float* temperature,
                        const int32_t* top_k, const float* top_p, const float* min_p,
                        int32_t filter_mode, float* probs, void* workspace,
                        size_t workspace_bytes, dsv_stream_t stream);

/* ---- capped chain rejection from dense probabilities ---------------------------------------
 * Replaces sampling/rejection.py:101-153 sample_capped_chain_from_probs (_sample_capped_chain,
 * :12-98): target_probs [B,16,V] and draft_probs [B,15,V] fp32, contiguous.  Draft s+1 is
 * accepted while q in (0,1] and uniforms[b,s] * q < p (at most verify_lens[b]-1 drafts); the
 * bonus is the first index whose running exact (2^-40 fixed point) mass of max(p - clamp01(q), 0)
 * exceeds floor(uniform_final * total) (p itself after a fully accepted block or a zero
 * residual; V-1 when no index does).  Same five outputs as dsv_verify_logits.  V <= 2^20. */
int dsv_chain_from_probs(int32_t batch, int32_t vocab, const int64_t* candidates,
                         const float* target_probs, const float* draft_probs,
                         const int32_t* verify_lens, const float* uniforms,
                         const float* uniform_final, const int32_t* prefix_lens, int32_t* accept,
                         int32_t* commit, int64_t* bonus, int64_t* output, int32_t* new_seq,
                         dsv_stream_t stream);

/* ---- capped chain rejection with sparse q ---------------------------------------------------
 * Replaces sampling/sparse/accept.py:463-543 accept_sparse (_accept_sparse, _dense_bonus,
 * _packed_bonus): q is sparse, q_ids/q_values [B,15,16] (q of a token = the sum of its
 * entries); the target row of (b, s) is row_offsets[b] + s (b * 16 without row_offsets) of
 * dense_p [rows, V] (divided by denominator[row] when given: the reference's raw fallback,
 * IEEE division) or, with packed rows (p_ids/p_values [rows, width <= 64], p_lengths, and
 * p_overflow != 0 meaning "use the dense row"), the packed entries (bonus over the row's ids in
 * ascending order, as the reference).  Exact fixed-point residual CDF; same five outputs as
 * dsv_verify_logits.  dense_p may be NULL when every packed row is used (pure packed). */
int dsv_accept_sparse(int32_t batch, int32_t vocab, int32_t width, const int64_t* candidates,
                      const float* dense_p, const int32_t* p_ids, const float* p_values,
                      const int32_t* p_lengths, const int32_t* p_overflow, const int64_t* q_ids,
                      const float* q_values, const int32_t* verify_lens, const float* uniforms,
                      const float* uniform_final, const int32_t* prefix_lens,
                      const int64_t* row_offsets, const float* denominator, int32_t* accept,
                      int32_t* commit, int64_t* bonus, int64_t* output, int32_t* new_seq,
                      dsv_stream_t stream);

/* ---- compress_probs ------------------------------------------------------------------------
 * Replaces sampling/sparse/accept.py:422-460 compress_probs: per row of probs [rows, V] the
 * first `capacity` positive entries in index order (ids int32 / values, padded with -1 / 0),
 * their clamped count and an overflow flag (more than capacity positives, or any negative,
 * NaN or infinite entry). */
int dsv_compress_probs(int64_t rows, int32_t vocab, int32_t capacity, const float* probs,
                       int32_t* ids, float* values, int32_t* lengths, int32_t* overflow,
                       dsv_stream_t stream);

/* ---- small-support joint target ---------------------------------------------------------
 * Replaces sampling/sparse/target.py:95-178 build_sparse_target (its CPU branch :156-178 is the
 * definition; _pack_joint :23-53 and _overflow_dense :56-76 the reference's CUDA branch).  Row r
 * of logits [rows, vocab] (dtype 0 bf16, 1 fp32; row_stride elements apart) belongs to request
 * row_request[r] (or r / rows_per_request when row_request is NULL), with temperature, top_k
 * (clamped to [1, capacity]) and top_p of that request.  With p = softmax(l / T): kept = p > 0,
 * p >= the k-th largest p (every tie kept), and the mass of strictly larger p below top_p (or
 * top_p >= 1).  count <= capacity: ids [r, :] the kept ids ascending (-1 padded), values their
 * p renormalised over the kept set (0 padded), lengths[r] = count, overflow[r] = 0.  count >
 * capacity: overflow[r] = 1, lengths[r] = capacity, packed entries -1 / 0, and dense [r, :] =
 * p where p >= the k-th largest p, renormalised, else 0.  Dense rows of packed rows are not
 * written.  Canonical arithmetic (exp2c, exact 2^-40 fixed-point masses); capacity <= 64. */
int dsv_sparse_target(int64_t rows, int32_t vocab, int32_t dtype, const void* logits,
                      int64_t row_stride, const int64_t* row_request, int32_t rows_per_request,
                      const float* temperature, const int32_t* top_k, const float* top_p,
                      int32_t capacity, int32_t* ids, float* values, int32_t* lengths,
                      int32_t* overflow, float* dense, dsv_stream_t stream);

/* ---- logit adjustments ---------------------------------------------------------------------
 * Replaces sampling/compact.py:14-79 adjust_logits (the native transforms of SGLang's
 * SamplingBatchInfo, in its order) in place on logits [rows, vocab] (bf16 or fp32, rows
 * row_stride elements apart): + additive[req] (acc_additive_penalties / acc_linear_penalties),
 * then scaling[req] (l < 0 ? l * s : l / s, acc_scaling_penalties), then the grammar bitmask
 * (vocab_mask[req] bit i clear: -inf; mask_words 32-bit words per request), then + bias[req]
 * (logit_bias); each step rounded to the logit dtype as the torch op it replaces.  Request of
 * row r: row_to_request[r], or r / rows_per_request when row_to_request is NULL.  Any of the
 * four inputs may be NULL. */
int dsv_adjust_logits(void* logits, int32_t dtype, int64_t rows, int32_t vocab, int64_t row_stride,
                      const int64_t* row_to_request, int32_t rows_per_request,
                      const float* additive, const float* scaling, const uint32_t* vocab_mask,
                      int32_t mask_words, const float* bias, dsv_stream_t stream);

/* ---- greedy capped accept ----------------------------------------------------------------------
 * Replaces verification/caps.py:32-59 _accept_capped (and verification/ragged.py:51-76 _accept):
 * with top1 of (b, s) at top1[(b * 16 + s) * top1_stride] (e.g. column 0 of a [B*16, k] top-k
 * id array with top1_stride = k), accepted = first s < cap-1 with cand[b, s+1] != top1(b, s),
 * else cap-1; bonus = top1(b, accepted); output keeps the proposed tokens around the bonus.
 * Same five outputs as dsv_verify_logits. */
int dsv_accept_greedy(int32_t batch, const int64_t* candidates, const int64_t* top1,
                      int64_t top1_stride, const int32_t* verify_lens, const int32_t* prefix_lens,
                      int32_t* accept, int32_t* commit, int64_t* bonus, int64_t* output,
                      int32_t* new_seq, dsv_stream_t stream);

/* ---- request-seeded uniforms -------------------------------------------------------------------
 * Replaces sampling/random.py:22-91 seeded_uniforms (bit-exact with its _cpu_uniforms):
 * out[r, c] for r < n, c < width from seeds[r] (int64), positions[r] (int32, or int64 when
 * positions_int64) and stream_id (DRAFT 0, ACCEPT 1, BONUS 2, PREFILL 3). */
int dsv_uniforms(int32_t n, int32_t width, const int64_t* seeds, const void* positions,
                 int32_t positions_int64, int32_t stream_id, float* out, dsv_stream_t stream);

/* ---- SPS verify-length plan --------------------------------------------------------------------
 * Replaces verification/sps.py:35-58 allocate_verify_lens and the index of sps.py:61-99
 * device_plan: raw [B, 15] draft confidences, table [15, nbins] conditional acceptance,
 * optional boundaries [nbound] (bucketize; NULL: linear bins), budget in [B, 16 B].
 * Outputs verify_lens [B], qo_indptr [B+1] and index [budget] (index[qo[b] + t] = b * 16 + t).
 * B <= 1024; one launch. */
int dsv_sps_plan(int32_t batch, const float* raw, const float* table, int32_t nbins,
                 const float* boundaries, int32_t nbound, int32_t budget, int32_t* verify_lens,
                 int64_t* qo_indptr, int64_t* index, dsv_stream_t stream);

/* ---- accept-compact on its own -----------------------------------------------------------------
 * The compaction of dsv_compact_out after any accept step (e.g. dsv_accept_greedy): tokens
 * output[b, :commit_b] and KV slots of positions [0, commit_b) packed by the exclusive scan of
 * commit; positions [commit_b, verify_len_b) freed.  Slot positions outside slots_len read as
 * -1 and set bit 2 of the error word of `workspace` (any zeroed dsv workspace). */
int dsv_accept_compact(int32_t batch, const int32_t* commit, const int32_t* verify_lens,
                       const int64_t* output, const dsv_compact_out* compact, void* workspace,
                       dsv_stream_t stream);

/* ---- draft-side serial chains ------------------------------------------------------------------
 * The kernels that produce a block's draft tokens, q rows and confidences from the serial
 * last-write refinement (T = block_size, n = batch * (T - 1) drafted rows, K candidates each).
 *
 * dsv_serial_sample_chain replaces kernels/dspine.py:616-772 (_serial_sample_chain /
 * serial_sample_chain): per request, row by row, p = softmax(table[n, sender] * inv_temp[b]),
 * joint filter rank < top_k[b] (ties to the lower lane), mass ranked ahead <= top_p[b],
 * p >= min_p[b] * max p, q = kept p renormalised, draw = first lane whose running sum of q
 * exceeds u[n] * total (capped at the last kept lane); the drawn lane is the next row's sender.
 * Writes out_tok[n] (cand[n, draw], or greedy_tok[n] when greedy[b]) and out_q[n, :] (q, or
 * the one-hot of cand == greedy_tok for greedy requests).  confidence_out (optional, [n]):
 * max p of each sampled row before filtering; rows of greedy requests are left untouched.
 * table fp32 [n, K, K]; inv_temp, top_p, min_p fp32 [batch]; top_k, greedy int32 [batch];
 * u fp32 [n]; candidates, greedy_tok int64 [n, K] / [n]; 1 <= K <= 64. */
int dsv_serial_sample_chain(int32_t batch, int32_t block_size, int32_t k, const float* table,
                            const float* inv_temp, const int32_t* top_k, const float* top_p,
                            const float* min_p, const int32_t* greedy, const float* u,
                            const int64_t* candidates, const int64_t* greedy_tok,
                            int64_t* out_tok, float* out_q, float* confidence_out,
                            dsv_stream_t stream);

/* dsv_serial_table replaces kernels/dspine.py:210-287 _serial_table (serial_table :357-471):
 * for drafted row n (request b, block row r, state row b*T + 1 + r), candidate lanes c with
 * ids cand[n, c] and sender lanes j (the anchor input_ids[b*T] on block row 0, else
 * cand[n-1, j]):
 *   s[j, c] = W[c] . (raw[row] * norm_w) + rms[row] * sum_r sigmoid(query[row, r] + TSV[s_j, r]
 *             + gate_b[r]) * TSV[s_j, RK + r] * TG[id_c, r]
 * (W[c] = lm_head[id_c], or candidate_head[n*K + c] when head_candidates) and writes
 * idx[n, j] = the first lane of max_c s[j, c]; confidence (optional, fp32 [n, K]) =
 * 1 / sum_c exp((s[j, c] - max) / max(rms, 1e-6)).  bf16 raw [batch*T, hidden] (row pitch
 * raw_stride), norm_w [hidden], lm_head (row pitch lm_stride, a multiple of 8, 16-byte aligned),
 * tg [vocab, rk], tsv [vocab, 2 rk], query (pitch query_stride, even), gate_b [rk] (query, tg,
 * tsv, gate_b 4-byte aligned); rms fp32 [batch*T].
 * hidden a multiple of 512 up to 16384, rk a multiple of 128, K a power of two in [2, 64].
 * A row whose candidate or sender id lies outside [0, vocab) writes idx -1 (confidence NaN). */
int dsv_serial_table(int32_t batch, int32_t block_size, int32_t hidden, int32_t rk, int32_t k,
                     int64_t vocab, const void* raw, int64_t raw_stride, const void* norm_w,
                     const int64_t* candidates, const int64_t* input_ids, const void* lm_head,
                     int64_t lm_stride, int32_t head_candidates, const void* tg, const void* tsv,
                     const void* query, int64_t query_stride, const float* rms,
                     const void* gate_b, int64_t* idx, float* confidence, dsv_stream_t stream);

/* dsv_serial_chain replaces kernels/dspine.py:290-324 _serial_chain (serial_chain :474-502):
 * per request, j = idx[first row, 0]; row r writes out[r] = cand[r, j] (and, with confidence,
 * confidence_out[r] = confidence[r, previous j], previous starting at 0), then j = idx[r+1, j].
 * A lane outside [0, K) selects the value 0.  confidence and confidence_out go together. */
int dsv_serial_chain(int32_t batch, int32_t block_size, int32_t k, const int64_t* idx,
                     const int64_t* candidates, int64_t* out, const float* confidence,
                     float* confidence_out, dsv_stream_t stream);

/* ---- top-k ids of materialised logits ------------------------------------------------------
 * Replaces kernels/dspine.py:165-207 topk_ids (with _chunk_max :111-121 and _select_topk
 * :124-162): out[r, :] = the ids of the k largest values of row r of logits (dtype 0 bf16,
 * 1 fp32, 2 fp16; row pitch row_stride elements), ascending by id; ties at the k-th place go to
 * the lower id (the reference's two-stage selection over 64-wide chunks gives exactly this).
 * k a power of two in [1, 64]; ceil(vocab / 64) >= k (as the reference); vocab <= 262144.
 * -0 equals +0; NaN ranks below every number. */
int dsv_topk_ids(int64_t rows, int32_t vocab, int64_t row_stride, int32_t dtype,
                 const void* logits, int32_t k, int64_t* out, dsv_stream_t stream);

/* The row's top-k (value desc, id asc) for any k in [1, min(128, vocab)], the ids written in
 * that rank order: the ids of stable_local_topk's portable path (layers/fp8/coarse.py:19-35: a
 * stable descending argsort, the first k).  Same kernel as dsv_topk_ids. */
int dsv_topk_ranked(int64_t rows, int32_t vocab, int64_t row_stride, int32_t dtype,
                    const void* logits, int32_t k, int64_t* out, dsv_stream_t stream);

/* ---- FP8 coarse retrieval + BF16 rescore (layers/fp8/coarse.py, layers/fp8/gather.py) -------
 * dsv_fp8_quantize_rows replaces _scale + _quantize (coarse.py:41-55): per row
 * scale[r] = max|x[r, :]| / 448 (1 for an all-zero row), q[r, c] = e4m3(clamp(x / scale, -448,
 * 448)) with IEEE division and round-to-nearest-even (dtype 0 bf16, 1 fp32; q rows q_stride
 * bytes apart).  FullVFP8Coarse.__init__ (coarse.py:58-73) quantizes the head with it once;
 * retrieve_and_rescore quantizes the hidden rows with it every step. */
int dsv_fp8_quantize_rows(int64_t rows, int32_t cols, int64_t row_stride, int32_t dtype,
                          const void* x, void* q, int64_t q_stride, float* scale,
                          dsv_stream_t stream);

/* Replaces torch.ops.aten._scaled_mm(xq, wq.T, x_scale, w_scale, out_dtype=bf16,
 * use_fast_accum=False) of retrieve_and_rescore (coarse.py:78-93):
 * out[r, c] = bf16(sum_h xq[r, h] * wq[c, h] * x_scale[r] * w_scale[c]), fp32 accumulation on
 * the tensor cores (tcgen05 kind::f8f6f4).  hidden a multiple of 128; xq, wq 16-byte aligned
 * with row pitches (bytes) multiples of 16.  *err (device, caller-zeroed) gets bit 0 when a
 * pipeline wait timed out. */
int dsv_fp8_coarse_scores(int32_t rows, int32_t vocab, int32_t hidden, const void* xq,
                          int64_t x_stride, const float* x_scale, const void* wq, int64_t w_stride,
                          const float* w_scale, void* out, int64_t out_stride, uint32_t* err,
                          dsv_stream_t stream);

/* Replaces rescore + select16 (gather.py:53-79 with gather_dot :7-34 and global_top16 :37-50):
 * scores[r, c] = sum_h weight[ids[r, c], h] * hidden_rows[r, h] in fp32, stored as bf16
 * (scores_f32 = 0, the hidden dtype of the reference) or fp32; ids outside [0, vocab) score
 * -inf.  With out16 non-null, out16[r, :] = the 16 tokens of the 16 selection rounds of
 * global_top16 (largest stored score, lowest token among equals), ascending.  A null weight
 * runs the selection alone on the given scores (select16; out16 required).  weight bf16,
 * 16-byte aligned, pitch a multiple of 8; hidden a multiple of 8, at most 16384; cands <= 128. */
int dsv_rescore_select16(int32_t rows, int32_t cands, int32_t hidden, int32_t vocab,
                         const void* weight, int64_t w_stride, const int64_t* ids,
                         const void* hidden_rows, int64_t h_stride, int32_t hidden_dtype,
                         void* scores, int32_t scores_f32, int64_t* out16, dsv_stream_t stream);

/* ---- the same verification without a caller workspace ------------------------------------
 * No counterpart in the reference: for callers that cannot allocate device memory (or hand out
 * scratch) at verification time.  Same arguments, outputs and results as dsv_verify_logits,
 * without `workspace`/`workspace_bytes`; its scratch is a fixed 870 KB device array inside the
 * library (sized for 256 requests), and the call performs no cudaMalloc/cudaFree and no
 * allocating library call.
 *  - batch > 256 returns DSV_WORKSPACE_TOO_SMALL before anything is enqueued.
 *  - each call clears the scratch it uses (cudaMemsetAsync on `stream`) before its kernels.
 *  - device_error (optional, a device pointer to one uint32) receives this call's error word
 *    (bits as for dsv_workspace_error), copied on `stream` after the kernels.
 *  - the scratch is shared by every call on a device: calls that can overlap (other streams,
 *    other host threads) race on it and must be serialised by the caller.
 *  - the first call on each device looks up the scratch address (cudaGetSymbolAddress, which
 *    may load the module); make that first call outside any stream capture.
 *  - the current device must be the device of `stream` and of the tensors. */
int dsv_verify_logits_noalloc(int32_t batch, int32_t vocab, int32_t dtype,
                              const int64_t* candidates, const void* target_logits,
                              const int64_t* target_row, int64_t target_rows,
                              const void* draft_logits, const int64_t* draft_row,
                              int64_t draft_rows, int64_t row_stride, const float* temperature,
                              const int32_t* top_k, const float* top_p,
                              const int32_t* verify_lens, const float* uniforms,
                              const float* uniform_final, const int32_t* prefix_lens,
                              int32_t* accept, int32_t* commit, int64_t* bonus, int64_t* output,
                              int32_t* new_seq, const dsv_compact_out* compact,
                              uint32_t* device_error, dsv_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DSPINE_B200_H */
