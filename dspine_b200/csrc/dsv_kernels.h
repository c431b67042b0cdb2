// dsv_kernels.h -- argument blocks and launchers shared by the kernels and the C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dsv {

struct TaskResult {
    int32_t d;       // accept decision of draft s+1 against target row s
    int32_t bonus;   // draw on row s if the chain stops there (-1: not drawn)
    float p;         // target probability of the drafted token (diagnostics)
    float q;         // draft probability of the drafted token (diagnostics)
};

struct WsHeader {
    unsigned int next;       // dynamic task counter
    unsigned int exited;     // clusters that left the task loop
    unsigned int finalized;  // requests finalized in this launch
    unsigned int err;        // bit 0: bulk copy timed out; bit 1: bad row; bit 2: bad slot;
                             // bit 3: a selection found no boundary; bit 4: tie cut not found;
                             // bit 5: shared-memory layout check of the row kernel failed;
                             // bit 6: a chain task's request was never published (time limit)
                             // bit 7: the second half of a split row gave up waiting for the
                             //        first (time limit); bits 0, 5-7 leave counters / flags
                             //        possibly set: the workspace must be zeroed again
    unsigned int next2;      // unused (kept zero; the header layout is fixed)
    unsigned int ready_tail; // row kernel: requests published to the ready list
    unsigned int chain_next; // row kernel: chain tasks taken
    unsigned int pad_;
    unsigned long long bytes_read;  // row kernel: logit bytes read from memory by the rows'
                                    // first passes, summed over launches (never reset by a
                                    // launch; verification drops rows that cannot change an
                                    // outcome, so this is what was read)
};
static_assert(sizeof(WsHeader) <= 64, "workspace header");

// Descriptor of one processed logit row (streaming path): p_i = exp2c((l_i - m) c) * inv_s
// for kept elements (key > kstar, or key == kstar and index <= tie_cut), else 0; greedy rows
// are one-hot at argmax.
constexpr uint32_t kDescGreedy = 1u;
struct RowDesc {
    float m;
    float c;
    float inv_s;
    uint32_t kstar;      // ordered 16-bit key of the boundary value
    int32_t tie_cut;
    int32_t argmax;
    uint32_t flags;
    uint32_t pad;
};

// Workspace layout: [WsHeader (64 B)][done: u32 x B, padded to 64 B][TaskResult x B x 16]
//                   [RowDesc x B x 16 x 2]
constexpr inline size_t verify_done_bytes(int B) { return ((size_t)B * 4 + 63) & ~(size_t)63; }
constexpr inline size_t verify_desc_offset(int B) {
    return 64 + verify_done_bytes(B) + (size_t)B * 16 * sizeof(TaskResult);
}
constexpr inline size_t verify_gmax_offset(int B) {
    return verify_desc_offset(B) + (size_t)B * 16 * 2 * sizeof(RowDesc);
}
// [u64 x B x 16]: greedy rows' packed (max key << 32 | ~first index), reset after use
// [u32 x B]: streaming path: the ready list (request + 1 per sampled request whose rows are
// done, in completion order; reset after use)
constexpr inline size_t verify_order_offset(int B) {
    return verify_gmax_offset(B) + (size_t)B * 16 * sizeof(unsigned long long);
}
// [u32 x 2 x B]: streaming path: per request its rows done and its chain steps decided (reset
// by the last CTA of each launch); cluster path: [2 b] = 16 - the earliest rejected step of
// request b (reset when the request is finalised)
constexpr inline size_t verify_racc_offset(int B) {
    return verify_order_offset(B) + (((size_t)B * 4 + 63) & ~(size_t)63);
}
// [u64 x 32 x 8 x B]: streaming path: residual mass per (request, slice, warp)
constexpr inline size_t verify_wmass_offset(int B) {
    return verify_racc_offset(B) + (((size_t)B * 8 + 63) & ~(size_t)63);
}
// [2 KB]: phase timers of profiling builds (-DDSV_PROFILE); unused otherwise.  Profiling
// builds add a 128 KB task trace after them.
#ifdef DSV_PROFILE
constexpr size_t kProfBytes = 2048 + 128 * 1024;
#else
constexpr size_t kProfBytes = 2048;
#endif
constexpr inline size_t verify_prof_offset(int B) {
    return verify_wmass_offset(B) + (size_t)B * 32 * 8 * 8;
}
// everything above: the workspace without split rows (the no-allocation entry point's scratch)
constexpr inline size_t verify_base_bytes(int B) {
    return verify_prof_offset(B) + kProfBytes;
}
// Split rows (streaming path): nucleus rows beyond the first wave of the row kernel are
// processed as two halves by two CTAs; the first half publishes its per-key histogram here.
// [kSplitCap slots of kSplitSlotBytes][u32 flag x kSplitCap]
#ifndef DSV_SPLIT_CAP
#define DSV_SPLIT_CAP 256
#endif
constexpr int kSplitCap = DSV_SPLIT_CAP;
constexpr size_t kSplitSlotBytes = 8192 * 4 + 16 + 512 * 2 + 48;  // counts, meta, band, pad
constexpr inline size_t verify_split_offset(int B) { return verify_base_bytes(B); }
constexpr inline size_t verify_workspace_bytes(int B) {
    return verify_split_offset(B) + (size_t)kSplitCap * (kSplitSlotBytes + 4);
}

struct VerifyArgs {
    int B, V;
    int slice;                 // vocabulary elements per CTA of a cluster
    int num_clusters;
    const int64_t* cand;       // [B,16]
    const void* tgt;           // target logits, rows of `stride` elements
    const int64_t* tgt_row;    // [B] first target row of request b
    long long tgt_rows;        // rows in the target tensor (bounds)
    const void* drf;           // draft logits or null (q one-hot at the draft)
    const int64_t* drf_row;    // [B] first draft row of request b
    long long drf_rows;
    long long stride;
    const float* temperature;  // [B]
    const int32_t* top_k;      // [B]
    const float* top_p;        // [B]
    const float* min_p;        // [B] or null (no min-p floor)
    int mode;                  // FilterMode (dsv_common.cuh)
    const int32_t* caps;       // [B] verify lengths
    const float* u;            // [B,15]
    const float* uf;           // [B]
    const int32_t* prefix;     // [B]
    int32_t* accept;
    int32_t* commit;
    int64_t* bonus;
    int64_t* output;           // [B,16]
    int32_t* new_seq;
    // optional accept-compact
    const int32_t* slots;      // KV slot of verify position s of request b: slots[slot_row[b]+s]
    long long slots_len;
    const int64_t* slot_row;
    int64_t* tok_out;          // [sum commit]
    int32_t* slot_out;         // [sum commit]
    int32_t* offsets;          // [B+1]
    int32_t* free_out;         // [sum (cap - commit)]
    int32_t* free_offsets;     // [B+1]
    // workspace
    WsHeader* ws;
    unsigned int* done;
    TaskResult* res;
    RowDesc* desc;             // [B,16,2] row descriptors (streaming path)
    unsigned long long* gmax;  // [B,16] greedy rows: max key << 32 | (0xFFFFFFFF - first index)
    unsigned long long* prof;  // profiling builds: phase timers
    unsigned int* order;       // [B] streaming path: chain-kernel dispatch order
    unsigned int* racc;        // [B,2] streaming path: rows finished, accepted length
    unsigned long long* wmass; // [B,32,8] streaming path: residual mass per slice and warp
    unsigned char* split;      // split-row slots (kSplitCap x kSplitSlotBytes) or null
    unsigned int* split_flag;  // [kSplitCap]: 1 once the first half is published
    int split_cap;             // rows that may be split in this launch (0: none)
    // standalone target probabilities (dsv_target_probs): caps == null means every request
    // has cap_all rows, tgt_row == null means request b starts at row b * row_step, cand ==
    // null skips the chain decision
    int cap_all;
    long long row_step;
};

// build_sparse_target (sparse_target.cu): per row the packed kept set of the small-support joint
// target, or the dense renormalised row when it overflows the capacity
struct SparseTargetArgs {
    long long rows;
    int V;
    int capacity;                  // packed width (<= 64); top-k values are clamped to it
    const void* logits;            // rows of `stride` elements
    long long stride;
    const int64_t* row_request;    // [rows] request of each row, or null: row / rows_per_request
    int rows_per_request;
    const float* temperature;      // per request
    const int32_t* top_k;
    const float* top_p;
    int32_t* ids;                  // [rows, capacity]
    float* values;                 // [rows, capacity]
    int32_t* lengths;              // [rows]
    int32_t* overflow;             // [rows]
    float* dense;                  // [rows, V]: overflow rows only
};
int launch_sparse_target(const SparseTargetArgs& a, int dtype, cudaStream_t stream);

// launchers (return a dsv::Status)
int launch_verify(const VerifyArgs& a, int dtype, cudaStream_t stream);
// streaming path (bf16 rows, B <= 1024, V <= 262144): rows kernel + chain kernel
bool stream_supported(const VerifyArgs& a, int dtype);
int launch_stream(VerifyArgs a, cudaStream_t stream);
// descriptors of every target row (rows kernel only) and the dense probabilities they define
int launch_target_probs(VerifyArgs a, float* out, cudaStream_t stream);
// the same probabilities from the cluster kernel of verify.cu (fp32 logits, or any vocabulary):
// rows tgt_rows, request of row t = t / row_step
int launch_probs_cluster(const VerifyArgs& a, int dtype, float* out, cudaStream_t stream);

// ---- LM head fused with top-k (lmhead.cu) ---------------------------------------------------
struct LmHeadArgs {
    int M, N, K, k;            // rows, vocabulary columns of this weight, hidden, top-k (<= 32)
    const void* x;             // [M, K] bf16, rows x_stride elements apart
    long long x_stride;
    const void* w;             // [N, K] bf16, rows w_stride elements apart
    long long w_stride;
    long long id_offset;       // added to every column index (first vocabulary id of a shard)
    long long pad_id;          // id written for empty slots (k > N)
    int sort_ids;              // 0: rank order (value desc, id asc); 1: ids ascending
    int64_t* out_ids;          // [M, k]
    float* out_val;            // [M, k] bf16-rounded logits
    float* out_lse;            // [M] or null
    void* workspace;           // lmhead_workspace_bytes(M, N, k), 16-byte aligned
};
int lmhead_tk(int k);  // register list length serving k (0: unsupported)
size_t lmhead_workspace_bytes(int M, int N, int k);
int launch_lmhead(const LmHeadArgs& h, cudaStream_t stream);

// merge of P per-shard lists (value desc, id asc) + their logsumexps: list p of row r at
// val[p * val_ps + r * k], ids[p * id_ps + r * k], lse[p * lse_ps + r]
struct TopkMergeArgs {
    int M, P, k;
    const float* val;
    long long val_ps;
    const int64_t* ids;
    long long id_ps;
    const float* lse;
    long long lse_ps;
    long long pad_id;
    int sort_ids;
    int64_t* out_ids;
    float* out_val;
    float* out_lse;
};
int launch_topk_merge(const TopkMergeArgs& m, cudaStream_t stream);

// ---- chain rejection from dense probabilities (probs.cu) -------------------------------------
struct ChainProbsArgs {
    int B, V;
    const int64_t* cand;   // [B,16]
    const float* target;   // [B,16,V]
    const float* draft;    // [B,15,V]
    const int32_t* caps;   // [B]
    const float* u;        // [B,15]
    const float* uf;       // [B]
    const int32_t* prefix; // [B]
    int32_t* accept;
    int32_t* commit;
    int64_t* bonus;
    int64_t* output;
    int32_t* new_seq;
};
int chain_probs_max_vocab();

// sparse-q chain rejection (probs.cu): dense, packed or overflow-mixed target rows
struct SparseAcceptArgs {
    int B, V, width;             // width: packed entries per row (0 without packed rows)
    const int64_t* cand;         // [B,16]
    const float* dense;          // [rows, V] or null
    const int32_t* p_ids;        // [rows, width] or null
    const float* p_vals;
    const int32_t* p_len;        // [rows]
    const int32_t* overflow;     // [rows]: the row is dense
    const int64_t* q_ids;        // [B,15,16]
    const float* q_vals;
    const int32_t* caps;
    const float* u;              // [B,15]
    const float* uf;             // [B]
    const int32_t* prefix;
    const int64_t* row_offsets;  // [B] or null (b * 16)
    const float* denom;          // [rows] or null: raw dense rows divided by it
    int32_t* accept;
    int32_t* commit;
    int64_t* bonus;
    int64_t* output;
    int32_t* new_seq;
};
int launch_sparse_accept(const SparseAcceptArgs& a, cudaStream_t stream);
int launch_compress(const float* p, long long rows, int V, int capacity, int32_t* ids, float* vals,
                    int32_t* lens, int32_t* ovf, cudaStream_t stream);
int launch_chain_probs(const ChainProbsArgs& c, cudaStream_t stream);

// ---- draft-side serial chains (serial.cu) ---------------------------------------------------
struct SampleChainArgs {
    int bs, tm1, k;               // requests, drafted rows per request (T-1), candidates per row
    const float* table;           // [bs*tm1, k, k]
    const float* inv_temp;        // [bs]
    const int32_t* top_k;         // [bs]
    const float* top_p;           // [bs]
    const float* min_p;           // [bs]
    const int32_t* greedy;        // [bs]
    const float* u;               // [bs*tm1]
    const int64_t* cand;          // [bs*tm1, k]
    const int64_t* greedy_tok;    // [bs*tm1]
    int64_t* out_tok;             // [bs*tm1]
    float* out_q;                 // [bs*tm1, k]
    float* confidence;            // [bs*tm1] or null
};
struct TableArgs {
    int n, t, h, rk, k;           // drafted rows, block width T, hidden, RK, candidates per row
    long long vocab;              // rows of tg / tsv (and of lm_w unless head_candidates)
    const __nv_bfloat16* raw;     // [bs*T, h]
    long long raw_stride;
    const __nv_bfloat16* norm_w;  // [h]
    const int64_t* cand;          // [n, k]
    const int64_t* input_ids;     // [bs*T]
    const __nv_bfloat16* lm_w;    // [vocab, h] or candidate head [n*k, h]
    long long w_stride;
    int head_candidates;
    const __nv_bfloat16* tg;      // [vocab, rk]
    const __nv_bfloat16* tsv;     // [vocab, 2*rk]
    const __nv_bfloat16* query;   // [bs*T, >= rk]
    long long q_stride;
    const float* rms;             // [bs*T]
    const __nv_bfloat16* gate_b;  // [rk]
    int64_t* idx;                 // [n, k]
    float* confidence;            // [n, k] or null
};
int serial_max_k();
size_t serial_table_smem(int h, int k);
size_t serial_chain_smem(int tm1, int k);
int launch_sample_chain(const SampleChainArgs& a, cudaStream_t stream);
int launch_serial_table(const TableArgs& a, cudaStream_t stream);
int launch_serial_chain(int bs, int tm1, int k, const int64_t* idx, const int64_t* cand,
                        int64_t* out, const float* conf, float* conf_out, cudaStream_t stream);

// ---- FP8 coarse retrieval (lmhead.cu, fp8.cu) ---------------------------------------------
struct Coarse8Args {
    int M, N, K;               // rows, weight rows (vocabulary), hidden (multiple of 128)
    const void* xq;            // [M, K] e4m3, rows x_stride bytes apart
    long long x_stride;
    const float* sx;           // [M]
    const void* wq;            // [N, K] e4m3, rows w_stride bytes apart
    long long w_stride;
    const float* sw;           // [N]
    void* out;                 // [M, N] bf16 scores, rows out_stride elements apart
    long long out_stride;
    unsigned int* err;         // error word (bit 0: a pipeline wait timed out)
};
int launch_coarse8(const Coarse8Args& a, cudaStream_t stream);
int launch_fp8_quantize(const void* x, int dtype, long long rows, int cols, long long stride,
                        uint8_t* q, long long q_stride, float* scale, cudaStream_t stream);
int launch_rescore16(int M, int C, int H, int V, const void* w, long long w_stride, const int64_t* ids,
                     const void* hidden, int hidden_dtype, long long h_stride, void* scores,
                     int scores_f32, int64_t* out16, cudaStream_t stream);
int fp8_max_candidates();
int fp8_max_hidden();

// ---- top-k ids of materialised logits (topk.cu) -------------------------------------------
int topk_max_k();
int topk_max_vocab();
int launch_topk_ids(const void* logits, int dtype, long long rows, int V, long long stride, int k,
                    int64_t* out, cudaStream_t stream);
int topk_ranked_max_k();
int launch_topk_ranked(const void* logits, int dtype, long long rows, int V, long long stride, int k,
                       int64_t* out, cudaStream_t stream);

// ---- per-request steps (small.cu) -----------------------------------------------------------
struct GreedyArgs {
    int B;
    const int64_t* cand;       // [B,16]
    const int64_t* top1;       // top-1 id of (b, s) at top1[(b * 16 + s) * top1_stride]
    long long top1_stride;
    const int32_t* caps;       // [B]
    const int32_t* prefix;     // [B]
    int32_t* accept;
    int32_t* commit;
    int64_t* bonus;
    int64_t* output;           // [B,16]
    int32_t* new_seq;
};
int launch_greedy(const GreedyArgs& g, cudaStream_t stream);

// in-place logit adjustments (small.cu)
struct AdjustArgs {
    void* logits;                  // [rows, V] bf16 or fp32, rows `stride` elements apart
    long long rows, stride;
    int V;
    const int64_t* row_to_request; // [rows] or null: request = row / rows_per_request
    int rows_per_request;
    const float* additive;         // [requests, V] or null
    const float* scaling;          // [requests, V] or null
    const uint32_t* mask;          // [requests, mask_words] bitmask (1 = allowed) or null
    int mask_words;
    const float* bias;             // [requests, V] or null
};
int launch_adjust(const AdjustArgs& a, int dtype, cudaStream_t stream);
int launch_uniforms(int n, int width, const int64_t* seeds, const void* positions, int pos64,
                    int stream_id, float* out, cudaStream_t stream);
int sps_max_batch();
int launch_sps(int B, const float* raw, const float* table, int nbins, const float* bounds,
               int nbound, int budget, int32_t* lens, int64_t* qo, int64_t* index,
               cudaStream_t stream);
int launch_compact(int B, const int32_t* commit, const int32_t* lens, const int64_t* output,
                   const int32_t* slots, long long slots_len, const int64_t* slot_row,
                   int64_t* tok_out, int32_t* slot_out, int32_t* offsets, int32_t* free_out,
                   int32_t* free_offsets, unsigned int* err, cudaStream_t stream);

}  // namespace dsv
