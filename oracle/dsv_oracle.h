/*
 * dsv_oracle.h -- CPU restatement of Tencent/DSpine's draft-block verification path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA product is compared
 * against (tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm).  No
 * product code path links or calls it.
 *
 * Every function follows one reference function (file:line inside the reference project,
 * package sglang_dspine) and states where this restatement fixes arithmetic that the
 * reference leaves to its reduction order:
 *
 *   - all sums that feed a discrete decision (softmax denominators, the top-p boundary, the
 *     residual CDF of the bonus draw) are exact integer sums of fix(x) = rne(x * 2^40);
 *   - exp is dsv_exp2 below (Cody-Waite reduction + a degree-6 polynomial fitted for this
 *     project), so a probability's fp32 bits are a pure function of its inputs.
 *
 * With those two rules the reference's decisions (accept length, emitted tokens, bonus) are
 * a function of the inputs alone; the reference's own float sums approximate the exact ones
 * to ~1e-7 relative, so the two agree except where a uniform lands within that distance of
 * a CDF step.
 */
#ifndef DSV_ORACLE_H
#define DSV_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OR_FIX_BITS 40

/* scalar building blocks (exposed for tests) */
float or_exp2(float y);
uint64_t or_fix(float x);
uint32_t or_key_f32(float v);
/* floor(u * m) for u an fp32 in [0,1), m < 2^62; returns -1 for u < 0 and -2 for u >= 1 or NaN */
int64_t or_scale_floor(float u, uint64_t m);

/* Row descriptor of the target distribution of one logit row
 * (runtime/worker.py:440-508 build_dspine_target_probs / filter_target_probs, flashinfer
 * backend with min-p off; tests/ref_utils.py:79-108 ref_target_row). */
typedef struct {
    int32_t greedy;     /* 1: one-hot at argmax */
    int32_t argmax;     /* first index of the maximum logit */
    float m;            /* max logit */
    float c;            /* log2(e) / T */
    uint32_t kstar;     /* threshold key: kept iff key > kstar or (key == kstar and i <= tie_cut) */
    int32_t tie_cut;
    int32_t n_kept;
    uint64_t s_total;   /* sum of fix(e) over the row */
    uint64_t s_kept;    /* sum of fix(e) over the kept set */
    float inv_s;        /* 1 / float(s_kept * 2^-40) */
} or_row_desc;

void or_process_row(const float* logits, int32_t V, float temperature, int32_t top_k,
                    float top_p, or_row_desc* out);

/* Filter modes of runtime/worker.py:473-508 filter_target_probs (see or_process_row_ex). */
#define OR_JOINT 0  /* flashinfer backend, no min-p in the batch: joint top-k / top-p      */
#define OR_SEQ 1    /* flashinfer backend, min-p in the batch: top-k -> top-p -> min-p     */
#define OR_TORCH 2  /* pytorch backend: joint top-k / top-p, then min-p                    */

/* or_process_row with min-p and a filter mode (min_p <= 0: no min-p floor) */
void or_process_row_ex(const float* logits, int32_t V, float temperature, int32_t top_k,
                       float top_p, float min_p, int32_t mode, or_row_desc* out);
/* the min-p key floor of a row with max m and c = log2(e) / T: elements whose 32-bit ordered
 * key is >= the floor pass "p >= min_p * max p" */
uint32_t or_minp_floor(float m, float c, float min_p);
/* floor(u * m) as or_scale_floor, and *exact = 1 when u * m is an integer */
int64_t or_scale_floor_exact(float u, uint64_t m, int* exact);
/* p_i of a processed row (0 outside the kept set) */
float or_row_prob(const float* logits, const or_row_desc* d, int32_t i);

/* Dense target probabilities for rows = bs*T logit rows (request b = row / rows_per_request).
 * logits [rows, V] f32; temperature/top_k/top_p per request; out [rows, V] f32. */
void or_target_probs(const float* logits, int64_t rows, int32_t V, int32_t rows_per_request,
                     const float* temperature, const int32_t* top_k, const float* top_p,
                     float* out, int32_t nthreads);

/* or_target_probs with per-request min_p (NULL: none) and a filter mode */
void or_target_probs_ex(const float* logits, int64_t rows, int32_t V, int32_t rows_per_request,
                        const float* temperature, const int32_t* top_k, const float* top_p,
                        const float* min_p, int32_t mode, float* out, int32_t nthreads);

/* build_sparse_target (sampling/sparse/target.py:95-178): per row the kept set of the
 * small-support joint target (threshold = k-th largest p, ties kept; nucleus = the mass of
 * strictly larger p below top_p), packed ids ascending / values (capacity wide), lengths,
 * overflow, and for overflow rows the dense row p >= threshold renormalised.  temperature,
 * top_k, top_p per row. */
void or_sparse_target(const float* logits, int64_t rows, int32_t V, const float* temperature,
                      const int32_t* top_k, const float* top_p, int32_t capacity, int32_t* ids,
                      float* values, int32_t* lengths, int32_t* overflow, float* dense,
                      int32_t nthreads);

/* sample_capped_chain_from_probs (sampling/rejection.py:12-153) with the exact residual
 * CDF.  candidates [B,16] i64, target [B,16,V] f32, draft [B,15,V] f32, caps [B] i32,
 * uniforms [B,15] f32, uniform_final [B] f32, prefix [B] i32.
 * Outputs: accept i32 [B], commit i32 [B], bonus i64 [B], output i64 [B,16], new_seq i32 [B]. */
void or_chain_from_probs(int32_t B, int32_t V, const int64_t* candidates, const float* target,
                         const float* draft, const int32_t* caps, const float* uniforms,
                         const float* uniform_final, const int32_t* prefix, int32_t* accept,
                         int32_t* commit, int64_t* bonus, int64_t* output, int32_t* new_seq);

/* Fused verification from logits: build_dspine_target_probs on target rows, the same
 * processing on dense draft logits (q of the draft sampler), then the capped chain and
 * residual bonus.  Target row of request b, position s is tgt_row[b] + s; draft row is
 * drf_row[b] + s (s < 15).  draft == NULL (or a greedy request) means q is one-hot at the
 * drafted token.  Logit rows are f32 of length V with row stride `stride`. */
void or_verify_logits(int32_t B, int32_t V, const int64_t* candidates, const float* target,
                      const int64_t* tgt_row, const float* draft, const int64_t* drf_row,
                      int64_t stride, const float* temperature, const int32_t* top_k,
                      const float* top_p, const int32_t* caps, const float* uniforms,
                      const float* uniform_final, const int32_t* prefix, int32_t* accept,
                      int32_t* commit, int64_t* bonus, int64_t* output, int32_t* new_seq,
                      int32_t nthreads);

/* or_verify_logits with per-request min_p (NULL: none) and a filter mode */
void or_verify_logits_ex(int32_t B, int32_t V, const int64_t* candidates, const float* target,
                         const int64_t* tgt_row, const float* draft, const int64_t* drf_row,
                         int64_t stride, const float* temperature, const int32_t* top_k,
                         const float* top_p, const float* min_p, int32_t mode,
                         const int32_t* caps, const float* uniforms, const float* uniform_final,
                         const int32_t* prefix, int32_t* accept, int32_t* commit,
                         int64_t* bonus, int64_t* output, int32_t* new_seq, int32_t nthreads);

/* accept_sparse (sampling/sparse/accept.py:207-543): sparse q (K=16), dense p (optionally
 * RAW with a denominator) or packed p with dense overflow rows, optional row offsets.
 * dense_p may be NULL (pure packed).  packed arrays may be NULL (dense only). */
void or_accept_sparse(int32_t B, int32_t V, const int64_t* candidates, const float* dense_p,
                      const int32_t* p_ids, const float* p_vals, const int32_t* p_len,
                      const int32_t* overflow, int32_t cap_width, const int64_t* q_ids,
                      const float* q_vals, const int32_t* caps, const float* uniforms,
                      const float* uniform_final, const int32_t* prefix,
                      const int64_t* row_offsets, const float* denom, int32_t* accept,
                      int32_t* commit, int64_t* bonus, int64_t* output, int32_t* new_seq);

/* compress_probs (sampling/sparse/accept.py:7-78,422-460) */
void or_compress_probs(const float* p, int64_t rows, int32_t V, int32_t capacity,
                       int32_t* ids, float* values, int32_t* lengths, int32_t* overflow);

/* Greedy capped accept (verification/caps.py:32-59, verification/ragged.py:51-76):
 * top1 [B,16] i64 given, caps [B]. */
void or_accept_greedy(int32_t B, const int64_t* candidates, const int64_t* top1,
                      const int32_t* caps, const int32_t* prefix, int32_t* accept,
                      int32_t* commit, int64_t* bonus, int64_t* output, int32_t* new_seq);

/* argmax of each row, first index of the maximum (torch.argmax) */
void or_argmax_rows(const float* x, int64_t rows, int32_t V, int64_t stride, int64_t* out);

/* topk_ids (kernels/dspine.py:165-207): k largest by (value desc, id asc), ids ascending */
void or_topk_ids(const float* x, int64_t rows, int32_t V, int64_t stride, int32_t k,
                 int64_t* out);

/* k largest by (value desc, id asc) in that order, with their values */
void or_topk_sorted(const float* x, int64_t rows, int32_t V, int64_t stride, int32_t k,
                    float* vals, int64_t* ids);

/* seeded uniforms (sampling/random.py:22-43) */
void or_uniforms(const int64_t* seeds, const int64_t* positions, int32_t n, int32_t width,
                 int32_t stream, float* out);

/* allocate_verify_lens (verification/sps.py:35-58) with linear bins (boundaries == NULL)
 * or bucketize(boundaries, right=False). raw [B,15], table [15, nbins]. */
void or_sps_lens(int32_t B, const float* raw, const float* table, int32_t nbins,
                 const float* boundaries, int32_t nbound, int32_t budget, int32_t* lens);
/* device_plan's window index (verification/sps.py:27-32,61-99) */
void or_sps_index(int32_t B, const int32_t* lens, int32_t T, int64_t* qo_indptr,
                  int64_t* index);

/* Accepted-token + KV-slot compaction.  SGLang's _commit_accept is not vendored in the
 * reference (it is wrapped at runtime/worker.py:745-777); this restates its contract:
 * tokens Output[b, :Commit_b] and slots of verify positions [0, Commit_b) are kept.
 * commit [B], lens [B] (verify rows of request b), output [B,16] tokens, slots: request b's
 * verify slot s is slots[slot_row[b] + s].  Writes tok_out/slot_out packed by exclusive
 * scan of commit (offsets [B+1]) and the freed slots (lens-commit per request) likewise. */
void or_accept_compact(int32_t B, const int32_t* commit, const int32_t* lens,
                       const int64_t* output, const int32_t* slots, const int64_t* slot_row,
                       int64_t* tok_out, int32_t* slot_out, int32_t* offsets,
                       int32_t* free_out, int32_t* free_offsets);

/* merge_topk (sampling/tp_head.py:9-14): values/ids [n, m]; first k by (value desc, then
 * stable by id asc, then by position) */
void or_merge_topk(int64_t n, int32_t m, const float* values, const int64_t* ids, int32_t k,
                   float* out_vals, int64_t* out_ids);

#ifdef __cplusplus
}
#endif
#endif
