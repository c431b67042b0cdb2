// capi.cu -- extern "C" entry points: host-side validation, then the kernel launchers.
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <mutex>

#include "../../include/dspine_b200.h"
#include "dsv_common.cuh"
#include "dsv_kernels.h"

namespace {

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

std::atomic<uint64_t> g_launches{0};

// count the kernels an entry point enqueued (only after a successful launch)
inline int counted(int status, int kernels) {
    if (status == DSV_OK) g_launches.fetch_add((uint64_t)kernels, std::memory_order_relaxed);
    return status;
}

// ---- scratch of dsv_verify_logits_noalloc -------------------------------------------------
// A file-scope device array sized for kNoAllocMaxBatch requests (870 KB).  It is part of the
// module image: the driver places it when the library's kernels are loaded on a device, and it
// starts zeroed.  Its address is looked up once per device and cached.
constexpr int kNoAllocMaxBatch = 256;
constexpr size_t kNoAllocBytes = dsv::verify_base_bytes(kNoAllocMaxBatch);  // no split rows
__device__ __align__(256) unsigned char g_noalloc_ws[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// address of g_noalloc_ws on the current device, or nullptr if it cannot be obtained
void* noalloc_scratch() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    if (g_noalloc_addr[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_ws) != cudaSuccess) return nullptr;
        g_noalloc_addr[dev] = p;
    }
    return g_noalloc_addr[dev];
}

}  // namespace

extern "C" {

const char* dsv_version(void) { return "dspine_b200 0.1.0 (sm_100a)"; }

uint64_t dsv_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char* dsv_status_string(int s) {
    switch (s) {
        case DSV_OK: return "ok";
        case DSV_BAD_SHAPE: return "bad shape";
        case DSV_BAD_DTYPE: return "bad dtype";
        case DSV_BAD_POINTER: return "bad pointer";
        case DSV_BAD_ALIGNMENT: return "bad alignment";
        case DSV_LAUNCH_FAILED: return "kernel launch failed";
        case DSV_WORKSPACE_TOO_SMALL: return "workspace too small";
        case DSV_DEVICE_TIMEOUT: return "device wait timed out";
        case DSV_UNSUPPORTED: return "unsupported configuration";
        default: return "unknown status";
    }
}

int dsv_verify_workspace_size(int32_t batch, size_t* bytes) {
    if (bytes == nullptr) return DSV_BAD_POINTER;
    if (batch < 0) return DSV_BAD_SHAPE;
    *bytes = dsv::verify_workspace_bytes(batch);
    return DSV_OK;
}

int dsv_workspace_init(void* ws, size_t bytes, dsv_stream_t stream) {
    if (ws == nullptr) return DSV_BAD_POINTER;
    if (cudaMemsetAsync(ws, 0, bytes, (cudaStream_t)stream) != cudaSuccess) return DSV_LAUNCH_FAILED;
    return DSV_OK;
}

int dsv_workspace_error(void* ws, uint32_t* err, dsv_stream_t stream) {
    if (ws == nullptr || err == nullptr) return DSV_BAD_POINTER;
    dsv::WsHeader* h = reinterpret_cast<dsv::WsHeader*>(ws);
    uint32_t v = 0;
    if (cudaMemcpyAsync(&v, &h->err, sizeof(v), cudaMemcpyDeviceToHost, (cudaStream_t)stream) != cudaSuccess)
        return DSV_LAUNCH_FAILED;
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return DSV_LAUNCH_FAILED;
    if (cudaMemsetAsync(&h->err, 0, sizeof(v), (cudaStream_t)stream) != cudaSuccess) return DSV_LAUNCH_FAILED;
    *err = v;
    return DSV_OK;
}

int dsv_copy_row_ranges(void* dst, const void* src, size_t row_bytes, int32_t n,
                        const int64_t* first_row, const int64_t* n_rows, dsv_stream_t stream) {
    if (n < 0) return DSV_BAD_SHAPE;
    if (n == 0) return DSV_OK;
    if (dst == nullptr || src == nullptr || first_row == nullptr || n_rows == nullptr)
        return DSV_BAD_POINTER;
    char* d = static_cast<char*>(dst);
    const char* s = static_cast<const char*>(src);
    int64_t r0 = -1, nr = 0;  // the range being merged
    for (int32_t i = 0; i <= n; ++i) {
        if (i < n) {
            if (first_row[i] < 0 || n_rows[i] < 0) return DSV_BAD_SHAPE;
            if (n_rows[i] == 0) continue;
            if (r0 >= 0 && r0 + nr == first_row[i]) {
                nr += n_rows[i];
                continue;
            }
        }
        if (r0 >= 0 && nr > 0) {
            const size_t off = (size_t)r0 * row_bytes;
            if (cudaMemcpyAsync(d + off, s + off, (size_t)nr * row_bytes, cudaMemcpyHostToDevice,
                                (cudaStream_t)stream) != cudaSuccess)
                return DSV_LAUNCH_FAILED;
        }
        if (i < n) {
            r0 = first_row[i];
            nr = n_rows[i];
        }
    }
    return DSV_OK;
}

int dsv_workspace_bytes_read(const void* ws, uint64_t* bytes, dsv_stream_t stream) {
    if (ws == nullptr || bytes == nullptr) return DSV_BAD_POINTER;
    const dsv::WsHeader* h = reinterpret_cast<const dsv::WsHeader*>(ws);
    unsigned long long v = 0;
    if (cudaMemcpyAsync(&v, &h->bytes_read, sizeof(v), cudaMemcpyDeviceToHost, (cudaStream_t)stream) !=
        cudaSuccess)
        return DSV_LAUNCH_FAILED;
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return DSV_LAUNCH_FAILED;
    *bytes = v;
    return DSV_OK;
}

int dsv_verify_logits_ex(int32_t batch, int32_t vocab, int32_t dtype, const int64_t* candidates,
                         const void* target_logits, const int64_t* target_row,
                         int64_t target_rows, const void* draft_logits, const int64_t* draft_row,
                         int64_t draft_rows, int64_t row_stride, const float* temperature,
                         const int32_t* top_k, const float* top_p, const float* min_p,
                         int32_t filter_mode, const int32_t* verify_lens, const float* uniforms,
                         const float* uniform_final, const int32_t* prefix_lens, int32_t* accept,
                         int32_t* commit, int64_t* bonus, int64_t* output, int32_t* new_seq,
                         const dsv_compact_out* compact, void* workspace,
                         size_t workspace_bytes, dsv_stream_t stream) {
    if (batch < 0 || vocab < 1 || row_stride < vocab || target_rows < 0) return DSV_BAD_SHAPE;
    if (filter_mode < DSV_FILTER_JOINT || filter_mode > DSV_FILTER_TORCH) return DSV_UNSUPPORTED;
    if (dtype != DSV_BF16 && dtype != DSV_F32) return DSV_BAD_DTYPE;
    if (batch == 0) return DSV_OK;
    if (target_rows < 1 || (draft_logits && draft_rows < 1)) return DSV_BAD_SHAPE;
    if (!candidates || !target_logits || !target_row || !temperature || !top_k || !top_p ||
        !verify_lens || !uniforms || !uniform_final || !prefix_lens || !accept || !commit ||
        !bonus || !output || !new_seq || !workspace)
        return DSV_BAD_POINTER;
    if (draft_logits && (!draft_row || draft_rows < 0)) return DSV_BAD_POINTER;
    if (compact && compact->slots_len < 0) return DSV_BAD_SHAPE;
    if (compact && (!compact->slots || !compact->slot_row || !compact->tokens ||
                    !compact->kept_slots || !compact->offsets || !compact->freed_slots ||
                    !compact->freed_offsets))
        return DSV_BAD_POINTER;
    // the split-row region is optional: without it no row is split
    if (workspace_bytes < dsv::verify_base_bytes(batch)) return DSV_WORKSPACE_TOO_SMALL;
    if (!aligned(workspace, 16)) return DSV_BAD_ALIGNMENT;
    const size_t esz = dtype == DSV_BF16 ? 2 : 4;
    if (!aligned(target_logits, esz) || (draft_logits && !aligned(draft_logits, esz)))
        return DSV_BAD_ALIGNMENT;

    dsv::VerifyArgs a = {};
    a.B = batch;
    a.V = vocab;
    a.cand = candidates;
    a.tgt = target_logits;
    a.tgt_row = target_row;
    a.tgt_rows = target_rows;
    a.drf = draft_logits;
    a.drf_row = draft_row;
    a.drf_rows = draft_rows;
    a.stride = row_stride;
    a.temperature = temperature;
    a.top_k = top_k;
    a.top_p = top_p;
    a.min_p = min_p;
    a.mode = filter_mode;
    a.caps = verify_lens;
    a.u = uniforms;
    a.uf = uniform_final;
    a.prefix = prefix_lens;
    a.accept = accept;
    a.commit = commit;
    a.bonus = bonus;
    a.output = output;
    a.new_seq = new_seq;
    if (compact) {
        a.slots = compact->slots;
        a.slots_len = compact->slots_len;
        a.slot_row = compact->slot_row;
        a.tok_out = compact->tokens;
        a.slot_out = compact->kept_slots;
        a.offsets = compact->offsets;
        a.free_out = compact->freed_slots;
        a.free_offsets = compact->freed_offsets;
    }
    char* base = reinterpret_cast<char*>(workspace);
    a.ws = reinterpret_cast<dsv::WsHeader*>(base);
    a.done = reinterpret_cast<unsigned int*>(base + 64);
    a.res = reinterpret_cast<dsv::TaskResult*>(base + 64 + dsv::verify_done_bytes(batch));
    a.desc = reinterpret_cast<dsv::RowDesc*>(base + dsv::verify_desc_offset(batch));
    a.gmax = reinterpret_cast<unsigned long long*>(base + dsv::verify_gmax_offset(batch));
    a.prof = reinterpret_cast<unsigned long long*>(base + dsv::verify_prof_offset(batch));
    a.order = reinterpret_cast<unsigned int*>(base + dsv::verify_order_offset(batch));
    a.racc = reinterpret_cast<unsigned int*>(base + dsv::verify_racc_offset(batch));
    a.wmass = reinterpret_cast<unsigned long long*>(base + dsv::verify_wmass_offset(batch));
    if (workspace_bytes >= dsv::verify_workspace_bytes(batch)) {
        a.split = reinterpret_cast<unsigned char*>(base + dsv::verify_split_offset(batch));
        a.split_flag = reinterpret_cast<unsigned int*>(a.split + (size_t)dsv::kSplitCap * dsv::kSplitSlotBytes);
        a.split_cap = dsv::kSplitCap;
    }
    if (dsv::stream_supported(a, dtype))
        return counted(dsv::launch_stream(a, (cudaStream_t)stream), 1);
    return counted(dsv::launch_verify(a, dtype, (cudaStream_t)stream), 1);
}

int dsv_verify_logits(int32_t batch, int32_t vocab, int32_t dtype, const int64_t* candidates,
                      const void* target_logits, const int64_t* target_row, int64_t target_rows,
                      const void* draft_logits, const int64_t* draft_row, int64_t draft_rows,
                      int64_t row_stride, const float* temperature, const int32_t* top_k,
                      const float* top_p, const int32_t* verify_lens, const float* uniforms,
                      const float* uniform_final, const int32_t* prefix_lens, int32_t* accept,
                      int32_t* commit, int64_t* bonus, int64_t* output, int32_t* new_seq,
                      const dsv_compact_out* compact, void* workspace, size_t workspace_bytes,
                      dsv_stream_t stream) {
    return dsv_verify_logits_ex(batch, vocab, dtype, candidates, target_logits, target_row,
                                target_rows, draft_logits, draft_row, draft_rows, row_stride,
                                temperature, top_k, top_p, nullptr, DSV_FILTER_JOINT, verify_lens,
                                uniforms, uniform_final, prefix_lens, accept, commit, bonus,
                                output, new_seq, compact, workspace, workspace_bytes, stream);
}

int dsv_lmhead_workspace_size(int32_t rows, int32_t vocab, int32_t k, size_t* bytes) {
    if (bytes == nullptr) return DSV_BAD_POINTER;
    if (rows < 0 || vocab < 1 || k < 1 || k > 32) return DSV_BAD_SHAPE;
    *bytes = dsv::lmhead_workspace_bytes(rows, vocab, k);
    return DSV_OK;
}

int dsv_lmhead_topk(int32_t rows, int32_t vocab, int32_t hidden, int32_t k,
                    const void* hidden_states, int64_t hidden_stride, const void* weight,
                    int64_t weight_stride, int64_t id_offset, int64_t pad_id, int32_t sort_ids,
                    int64_t* ids, float* values, float* lse, void* workspace,
                    size_t workspace_bytes, dsv_stream_t stream) {
    if (rows < 0 || vocab < 1 || k < 1 || k > 32) return DSV_BAD_SHAPE;
    if (hidden < 64 || hidden % 64 != 0) return DSV_BAD_SHAPE;
    if (hidden_stride < hidden || weight_stride < hidden) return DSV_BAD_SHAPE;
    if (rows == 0) return DSV_OK;
    if (!hidden_states || !weight || !ids || !values || !workspace) return DSV_BAD_POINTER;
    // tensor maps: 16-byte aligned bases and row pitches
    if (!aligned(hidden_states, 16) || !aligned(weight, 16) || hidden_stride % 8 != 0 ||
        weight_stride % 8 != 0 || !aligned(workspace, 16))
        return DSV_BAD_ALIGNMENT;
    if (workspace_bytes < dsv::lmhead_workspace_bytes(rows, vocab, k)) return DSV_WORKSPACE_TOO_SMALL;
    dsv::LmHeadArgs h = {};
    h.M = rows;
    h.N = vocab;
    h.K = hidden;
    h.k = k;
    h.x = hidden_states;
    h.x_stride = hidden_stride;
    h.w = weight;
    h.w_stride = weight_stride;
    h.id_offset = id_offset;
    h.pad_id = pad_id;
    h.sort_ids = sort_ids != 0;
    h.out_ids = ids;
    h.out_val = values;
    h.out_lse = lse;
    h.workspace = workspace;
    return counted(dsv::launch_lmhead(h, (cudaStream_t)stream), 2);
}

int dsv_tp_merge(int32_t rows, int32_t shards, int32_t k, const float* values,
                 int64_t values_shard_stride, const int64_t* ids, int64_t ids_shard_stride,
                 const float* lse, int64_t lse_shard_stride, int64_t pad_id, int32_t sort_ids,
                 int64_t* out_ids, float* out_values, float* out_lse, dsv_stream_t stream) {
    if (rows < 0 || shards < 1 || shards > 256 || k < 1 || k > 32) return DSV_BAD_SHAPE;
    if (values_shard_stride < (int64_t)rows * k || ids_shard_stride < (int64_t)rows * k ||
        lse_shard_stride < rows)
        return DSV_BAD_SHAPE;
    if (rows == 0) return DSV_OK;
    if (!values || !ids || !lse || !out_ids || !out_values) return DSV_BAD_POINTER;
    if (!aligned(ids, 8) || !aligned(values, 4) || !aligned(lse, 4)) return DSV_BAD_ALIGNMENT;
    dsv::TopkMergeArgs m = {};
    m.M = rows;
    m.P = shards;
    m.k = k;
    m.val = values;
    m.val_ps = values_shard_stride;
    m.ids = ids;
    m.id_ps = ids_shard_stride;
    m.lse = lse;
    m.lse_ps = lse_shard_stride;
    m.pad_id = pad_id;
    m.sort_ids = sort_ids != 0;
    m.out_ids = out_ids;
    m.out_val = out_values;
    m.out_lse = out_lse;
    return counted(dsv::launch_topk_merge(m, (cudaStream_t)stream), 1);
}

int dsv_chain_from_probs(int32_t batch, int32_t vocab, const int64_t* candidates,
                         const float* target_probs, const float* draft_probs,
                         const int32_t* verify_lens, const float* uniforms,
                         const float* uniform_final, const int32_t* prefix_lens, int32_t* accept,
                         int32_t* commit, int64_t* bonus, int64_t* output, int32_t* new_seq,
                         dsv_stream_t stream) {
    if (batch < 0 || vocab < 1 || vocab > dsv::chain_probs_max_vocab()) return DSV_BAD_SHAPE;
    if (batch == 0) return DSV_OK;
    if (!candidates || !target_probs || !draft_probs || !verify_lens || !uniforms ||
        !uniform_final || !prefix_lens || !accept || !commit || !bonus || !output || !new_seq)
        return DSV_BAD_POINTER;
    if (!aligned(target_probs, 4) || !aligned(draft_probs, 4)) return DSV_BAD_ALIGNMENT;
    dsv::ChainProbsArgs c = {batch, vocab, candidates, target_probs, draft_probs, verify_lens,
                             uniforms, uniform_final, prefix_lens, accept, commit, bonus,
                             output, new_seq};
    return counted(dsv::launch_chain_probs(c, (cudaStream_t)stream), 1);
}

int dsv_accept_sparse(int32_t batch, int32_t vocab, int32_t width, const int64_t* candidates,
                      const float* dense_p, const int32_t* p_ids, const float* p_values,
                      const int32_t* p_lengths, const int32_t* p_overflow, const int64_t* q_ids,
                      const float* q_values, const int32_t* verify_lens, const float* uniforms,
                      const float* uniform_final, const int32_t* prefix_lens,
                      const int64_t* row_offsets, const float* denominator, int32_t* accept,
                      int32_t* commit, int64_t* bonus, int64_t* output, int32_t* new_seq,
                      dsv_stream_t stream) {
    if (batch < 0 || vocab < 1 || vocab > dsv::chain_probs_max_vocab()) return DSV_BAD_SHAPE;
    if (p_ids && (width < 1 || width > 64)) return DSV_BAD_SHAPE;
    if (batch == 0) return DSV_OK;
    if (!candidates || !q_ids || !q_values || !verify_lens || !uniforms || !uniform_final ||
        !prefix_lens || !accept || !commit || !bonus || !output || !new_seq)
        return DSV_BAD_POINTER;
    if (!dense_p && !p_ids) return DSV_BAD_POINTER;
    if (p_ids && (!p_values || !p_lengths || !p_overflow)) return DSV_BAD_POINTER;
    dsv::SparseAcceptArgs a = {};
    a.B = batch;
    a.V = vocab;
    a.width = p_ids ? width : 0;
    a.cand = candidates;
    a.dense = dense_p;
    a.p_ids = p_ids;
    a.p_vals = p_values;
    a.p_len = p_lengths;
    a.overflow = p_overflow;
    a.q_ids = q_ids;
    a.q_vals = q_values;
    a.caps = verify_lens;
    a.u = uniforms;
    a.uf = uniform_final;
    a.prefix = prefix_lens;
    a.row_offsets = row_offsets;
    a.denom = denominator;
    a.accept = accept;
    a.commit = commit;
    a.bonus = bonus;
    a.output = output;
    a.new_seq = new_seq;
    return counted(dsv::launch_sparse_accept(a, (cudaStream_t)stream), 1);
}

int dsv_compress_probs(int64_t rows, int32_t vocab, int32_t capacity, const float* probs,
                       int32_t* ids, float* values, int32_t* lengths, int32_t* overflow,
                       dsv_stream_t stream) {
    if (rows < 0 || vocab < 1 || capacity < 1 || rows > 0x7fffffff) return DSV_BAD_SHAPE;
    if (rows == 0) return DSV_OK;
    if (!probs || !ids || !values || !lengths || !overflow) return DSV_BAD_POINTER;
    return counted(dsv::launch_compress(probs, rows, vocab, capacity, ids, values, lengths, overflow,
                                        (cudaStream_t)stream),
                   1);
}

int dsv_sparse_target(int64_t rows, int32_t vocab, int32_t dtype, const void* logits,
                      int64_t row_stride, const int64_t* row_request, int32_t rows_per_request,
                      const float* temperature, const int32_t* top_k, const float* top_p,
                      int32_t capacity, int32_t* ids, float* values, int32_t* lengths,
                      int32_t* overflow, float* dense, dsv_stream_t stream) {
    if (rows < 0 || vocab < 1 || row_stride < vocab || capacity < 1 || capacity > 64)
        return DSV_BAD_SHAPE;
    if (!row_request && rows_per_request < 1) return DSV_BAD_SHAPE;
    if (dtype != DSV_BF16 && dtype != DSV_F32) return DSV_BAD_DTYPE;
    if (rows == 0) return DSV_OK;
    if (!logits || !temperature || !top_k || !top_p || !ids || !values || !lengths || !overflow ||
        !dense)
        return DSV_BAD_POINTER;
    dsv::SparseTargetArgs a = {rows, vocab, capacity, logits, row_stride, row_request,
                               rows_per_request, temperature, top_k, top_p, ids, values,
                               lengths, overflow, dense};
    return counted(dsv::launch_sparse_target(a, dtype, (cudaStream_t)stream), 1);
}

int dsv_adjust_logits(void* logits, int32_t dtype, int64_t rows, int32_t vocab, int64_t row_stride,
                      const int64_t* row_to_request, int32_t rows_per_request,
                      const float* additive, const float* scaling, const uint32_t* vocab_mask,
                      int32_t mask_words, const float* bias, dsv_stream_t stream) {
    if (rows < 0 || vocab < 1 || row_stride < vocab || rows > 0x7fffffff) return DSV_BAD_SHAPE;
    if (dtype != DSV_BF16 && dtype != DSV_F32) return DSV_BAD_DTYPE;
    if (!row_to_request && rows_per_request < 1) return DSV_BAD_SHAPE;
    if (vocab_mask && mask_words * 32 < vocab) return DSV_BAD_SHAPE;
    if (rows == 0) return DSV_OK;
    if (!logits) return DSV_BAD_POINTER;
    dsv::AdjustArgs a = {logits, rows, row_stride, vocab, row_to_request, rows_per_request,
                         additive, scaling, vocab_mask, mask_words, bias};
    return counted(dsv::launch_adjust(a, dtype, (cudaStream_t)stream), 1);
}

int dsv_accept_greedy(int32_t batch, const int64_t* candidates, const int64_t* top1,
                      int64_t top1_stride, const int32_t* verify_lens, const int32_t* prefix_lens,
                      int32_t* accept, int32_t* commit, int64_t* bonus, int64_t* output,
                      int32_t* new_seq, dsv_stream_t stream) {
    if (batch < 0 || top1_stride < 1) return DSV_BAD_SHAPE;
    if (batch == 0) return DSV_OK;
    if (!candidates || !top1 || !verify_lens || !prefix_lens || !accept || !commit || !bonus ||
        !output || !new_seq)
        return DSV_BAD_POINTER;
    dsv::GreedyArgs g = {batch, candidates, top1, top1_stride, verify_lens, prefix_lens,
                         accept, commit, bonus, output, new_seq};
    return counted(dsv::launch_greedy(g, (cudaStream_t)stream), 1);
}

int dsv_uniforms(int32_t n, int32_t width, const int64_t* seeds, const void* positions,
                 int32_t positions_int64, int32_t stream_id, float* out, dsv_stream_t stream) {
    if (n < 0 || width < 1 || width >= 65536 || stream_id < 0 || stream_id > 3) return DSV_BAD_SHAPE;
    if (n == 0) return DSV_OK;
    if (!seeds || !positions || !out) return DSV_BAD_POINTER;
    return counted(dsv::launch_uniforms(n, width, seeds, positions, positions_int64 != 0,
                                        stream_id, out, (cudaStream_t)stream),
                   1);
}

int dsv_sps_plan(int32_t batch, const float* raw, const float* table, int32_t nbins,
                 const float* boundaries, int32_t nbound, int32_t budget, int32_t* verify_lens,
                 int64_t* qo_indptr, int64_t* index, dsv_stream_t stream) {
    if (batch < 1 || batch > dsv::sps_max_batch() || nbins < 1) return DSV_BAD_SHAPE;
    if (budget < batch || budget > batch * 16) return DSV_BAD_SHAPE;
    if (boundaries && nbound < 0) return DSV_BAD_SHAPE;
    if (!raw || !table || !verify_lens || !qo_indptr || !index) return DSV_BAD_POINTER;
    return counted(dsv::launch_sps(batch, raw, table, nbins, boundaries, boundaries ? nbound : 0,
                                   budget, verify_lens, qo_indptr, index, (cudaStream_t)stream),
                   1);
}

int dsv_accept_compact(int32_t batch, const int32_t* commit, const int32_t* verify_lens,
                       const int64_t* output, const dsv_compact_out* compact, void* workspace,
                       dsv_stream_t stream) {
    if (batch < 0) return DSV_BAD_SHAPE;
    if (batch == 0) return DSV_OK;
    if (!commit || !verify_lens || !output || !compact || !workspace) return DSV_BAD_POINTER;
    if (compact->slots_len < 0) return DSV_BAD_SHAPE;
    if (!compact->slots || !compact->slot_row || !compact->tokens || !compact->kept_slots ||
        !compact->offsets || !compact->freed_slots || !compact->freed_offsets)
        return DSV_BAD_POINTER;
    if (!aligned(workspace, 16)) return DSV_BAD_ALIGNMENT;
    unsigned int* err = reinterpret_cast<unsigned int*>(static_cast<char*>(workspace) +
                                                        offsetof(dsv::WsHeader, err));
    return counted(dsv::launch_compact(batch, commit, verify_lens, output, compact->slots,
                                       compact->slots_len, compact->slot_row, compact->tokens,
                                       compact->kept_slots, compact->offsets,
                                       compact->freed_slots, compact->freed_offsets, err,
                                       (cudaStream_t)stream),
                   1);
}

int dsv_target_probs_ex(int64_t rows, int32_t vocab, int32_t dtype, int32_t rows_per_request,
                        const void* logits, int64_t row_stride, const float* temperature,
                        const int32_t* top_k, const float* top_p, const float* min_p,
                        int32_t filter_mode, float* probs, void* workspace,
                        size_t workspace_bytes, dsv_stream_t stream) {
    if (rows < 0 || vocab < 1 || rows_per_request < 1 || row_stride < vocab ||
        rows % rows_per_request != 0)
        return DSV_BAD_SHAPE;
    if (dtype != DSV_BF16 && dtype != DSV_F32) return DSV_BAD_DTYPE;
    if (filter_mode < DSV_FILTER_JOINT || filter_mode > DSV_FILTER_TORCH) return DSV_UNSUPPORTED;
    const bool rows_path = dtype == DSV_BF16 && vocab <= 262000 && rows_per_request <= 16;
    if (rows == 0) return DSV_OK;
    if (!logits || !temperature || !top_k || !top_p || !probs || !workspace) return DSV_BAD_POINTER;
    if (!aligned(logits, dtype == DSV_BF16 ? 2 : 4) || !aligned(workspace, 16))
        return DSV_BAD_ALIGNMENT;
    const long long nreq = rows / rows_per_request;
    char* base = reinterpret_cast<char*>(workspace);
    if (!rows_path) {
        // one cluster per row (verify.cu): only the task counters of the workspace are used
        if (workspace_bytes < 64) return DSV_WORKSPACE_TOO_SMALL;
        dsv::VerifyArgs a = {};
        a.B = (int)(nreq < 0x7fffffff ? nreq : 0x7fffffff);
        a.V = vocab;
        a.tgt = logits;
        a.tgt_rows = rows;
        a.row_step = rows_per_request;
        a.stride = row_stride;
        a.temperature = temperature;
        a.top_k = top_k;
        a.top_p = top_p;
        a.min_p = min_p;
        a.mode = filter_mode;
        a.ws = reinterpret_cast<dsv::WsHeader*>(base);
        return counted(dsv::launch_probs_cluster(a, dtype, probs, (cudaStream_t)stream), 1);
    }
    const int chunk = 1024;
    const int wsb = (int)(nreq < chunk ? nreq : chunk);
    if (workspace_bytes < dsv::verify_base_bytes(wsb)) return DSV_WORKSPACE_TOO_SMALL;
    int launched = 0;
    for (long long r0 = 0; r0 < nreq; r0 += chunk) {
        const int B = (int)((nreq - r0) < chunk ? (nreq - r0) : chunk);
        dsv::VerifyArgs a = {};
        a.B = B;
        a.V = vocab;
        a.tgt = static_cast<const uint16_t*>(logits) + r0 * rows_per_request * row_stride;
        a.tgt_row = nullptr;
        a.row_step = rows_per_request;
        a.tgt_rows = (long long)B * rows_per_request;
        a.stride = row_stride;
        a.temperature = temperature + r0;
        a.top_k = top_k + r0;
        a.top_p = top_p + r0;
        a.min_p = min_p ? min_p + r0 : nullptr;
        a.mode = filter_mode;
        a.caps = nullptr;
        a.cap_all = rows_per_request;
        a.ws = reinterpret_cast<dsv::WsHeader*>(base);
        a.done = reinterpret_cast<unsigned int*>(base + 64);
        a.res = reinterpret_cast<dsv::TaskResult*>(base + 64 + dsv::verify_done_bytes(wsb));
        a.desc = reinterpret_cast<dsv::RowDesc*>(base + dsv::verify_desc_offset(wsb));
        a.gmax = reinterpret_cast<unsigned long long*>(base + dsv::verify_gmax_offset(wsb));
        a.order = reinterpret_cast<unsigned int*>(base + dsv::verify_order_offset(wsb));
        a.racc = reinterpret_cast<unsigned int*>(base + dsv::verify_racc_offset(wsb));
        a.wmass = reinterpret_cast<unsigned long long*>(base + dsv::verify_wmass_offset(wsb));
        a.prof = reinterpret_cast<unsigned long long*>(base + dsv::verify_prof_offset(wsb));
        const int st = dsv::launch_target_probs(a, probs + r0 * rows_per_request * (long long)vocab,
                                                (cudaStream_t)stream);
        if (st != DSV_OK) return counted(st, launched);
        launched += 2;
    }
    return counted(DSV_OK, launched);
}

int dsv_target_probs(int64_t rows, int32_t vocab, int32_t rows_per_request, const void* logits,
                     int64_t row_stride, const float* temperature, const int32_t* top_k,
                     const float* top_p, float* probs, void* workspace, size_t workspace_bytes,
                     dsv_stream_t stream) {
    if (vocab > 262000 || rows_per_request > 16) return DSV_BAD_SHAPE;
    return dsv_target_probs_ex(rows, vocab, DSV_BF16, rows_per_request, logits, row_stride,
                               temperature, top_k, top_p, nullptr, DSV_FILTER_JOINT, probs,
                               workspace, workspace_bytes, stream);
}

int dsv_topk_ids(int64_t rows, int32_t vocab, int64_t row_stride, int32_t dtype,
                 const void* logits, int32_t k, int64_t* out, dsv_stream_t stream) {
    if (rows < 0 || vocab < 1 || vocab > dsv::topk_max_vocab() || row_stride < vocab) return DSV_BAD_SHAPE;
    if (k < 1 || k > dsv::topk_max_k() || (k & (k - 1)) || (vocab + 63) / 64 < k) return DSV_BAD_SHAPE;
    if (dtype < 0 || dtype > 2) return DSV_BAD_DTYPE;
    if (rows == 0) return DSV_OK;
    if (!logits || !out) return DSV_BAD_POINTER;
    if (!aligned(logits, dtype == 1 ? 4 : 2)) return DSV_BAD_ALIGNMENT;
    return counted(dsv::launch_topk_ids(logits, dtype, rows, vocab, row_stride, k, out,
                                        (cudaStream_t)stream),
                   1);
}

int dsv_topk_ranked(int64_t rows, int32_t vocab, int64_t row_stride, int32_t dtype,
                    const void* logits, int32_t k, int64_t* out, dsv_stream_t stream) {
    if (rows < 0 || vocab < 1 || vocab > dsv::topk_max_vocab() || row_stride < vocab) return DSV_BAD_SHAPE;
    if (k < 1 || k > dsv::topk_ranked_max_k() || k > vocab) return DSV_BAD_SHAPE;
    if (dtype < 0 || dtype > 2) return DSV_BAD_DTYPE;
    if (rows == 0) return DSV_OK;
    if (!logits || !out) return DSV_BAD_POINTER;
    if (!aligned(logits, dtype == 1 ? 4 : 2)) return DSV_BAD_ALIGNMENT;
    return counted(dsv::launch_topk_ranked(logits, dtype, rows, vocab, row_stride, k, out,
                                           (cudaStream_t)stream),
                   1);
}

int dsv_fp8_quantize_rows(int64_t rows, int32_t cols, int64_t row_stride, int32_t dtype,
                          const void* x, void* q, int64_t q_stride, float* scale,
                          dsv_stream_t stream) {
    if (rows < 0 || cols < 1 || row_stride < cols || q_stride < cols) return DSV_BAD_SHAPE;
    if (dtype < 0 || dtype > 1) return DSV_BAD_DTYPE;
    if (rows == 0) return DSV_OK;
    if (!x || !q || !scale) return DSV_BAD_POINTER;
    if (!aligned(x, dtype == 1 ? 4 : 2) || !aligned(scale, 4)) return DSV_BAD_ALIGNMENT;
    return counted(dsv::launch_fp8_quantize(x, dtype, rows, cols, row_stride, static_cast<uint8_t*>(q),
                                            q_stride, scale, (cudaStream_t)stream),
                   1);
}

int dsv_fp8_coarse_scores(int32_t rows, int32_t vocab, int32_t hidden, const void* xq,
                          int64_t x_stride, const float* x_scale, const void* wq, int64_t w_stride,
                          const float* w_scale, void* out, int64_t out_stride, uint32_t* err,
                          dsv_stream_t stream) {
    if (rows < 0 || vocab < 1 || hidden < 128 || hidden % 128) return DSV_BAD_SHAPE;
    if (x_stride < hidden || w_stride < hidden || out_stride < vocab) return DSV_BAD_SHAPE;
    if (rows == 0) return DSV_OK;
    if (!xq || !x_scale || !wq || !w_scale || !out || !err) return DSV_BAD_POINTER;
    // TMA: 16-byte aligned bases and row pitches
    if (!aligned(xq, 16) || !aligned(wq, 16) || (x_stride % 16) || (w_stride % 16)) return DSV_BAD_ALIGNMENT;
    if (!aligned(out, 2) || !aligned(x_scale, 4) || !aligned(w_scale, 4) || !aligned(err, 4))
        return DSV_BAD_ALIGNMENT;
    dsv::Coarse8Args a = {};
    a.M = rows;
    a.N = vocab;
    a.K = hidden;
    a.xq = xq;
    a.x_stride = x_stride;
    a.sx = x_scale;
    a.wq = wq;
    a.w_stride = w_stride;
    a.sw = w_scale;
    a.out = out;
    a.out_stride = out_stride;
    a.err = err;
    return counted(dsv::launch_coarse8(a, (cudaStream_t)stream), 1);
}

int dsv_rescore_select16(int32_t rows, int32_t cands, int32_t hidden, int32_t vocab,
                         const void* weight, int64_t w_stride, const int64_t* ids,
                         const void* hidden_rows, int64_t h_stride, int32_t hidden_dtype,
                         void* scores, int32_t scores_f32, int64_t* out16, dsv_stream_t stream) {
    if (rows < 0 || cands < 1 || cands > dsv::fp8_max_candidates() || vocab < 1) return DSV_BAD_SHAPE;
    if (out16 && cands < 16) return DSV_BAD_SHAPE;
    if (weight) {
        if (hidden < 8 || hidden % 8 || hidden > dsv::fp8_max_hidden()) return DSV_BAD_SHAPE;
        if (w_stride < hidden || h_stride < hidden) return DSV_BAD_SHAPE;
        if (hidden_dtype < 0 || hidden_dtype > 1) return DSV_BAD_DTYPE;
    } else {
        hidden = 0;  // selection only
        if (!out16) return DSV_BAD_POINTER;
    }
    if (rows == 0) return DSV_OK;
    if (!ids || !scores || (weight && !hidden_rows)) return DSV_BAD_POINTER;
    if ((weight && (!aligned(weight, 16) || (w_stride % 8) || !aligned(hidden_rows, hidden_dtype ? 4 : 2))) ||
        !aligned(ids, 8) || !aligned(scores, scores_f32 ? 4 : 2) || (out16 && !aligned(out16, 8)))
        return DSV_BAD_ALIGNMENT;
    return counted(dsv::launch_rescore16(rows, cands, hidden, vocab, weight, w_stride, ids, hidden_rows,
                                         hidden_dtype, h_stride, scores, scores_f32, out16,
                                         (cudaStream_t)stream),
                   1);
}

int dsv_serial_sample_chain(int32_t batch, int32_t block_size, int32_t k, const float* table,
                            const float* inv_temp, const int32_t* top_k, const float* top_p,
                            const float* min_p, const int32_t* greedy, const float* u,
                            const int64_t* candidates, const int64_t* greedy_tok,
                            int64_t* out_tok, float* out_q, float* confidence_out,
                            dsv_stream_t stream) {
    if (batch < 0 || block_size < 2 || k < 1 || k > dsv::serial_max_k()) return DSV_BAD_SHAPE;
    if ((int64_t)batch * (block_size - 1) > INT32_MAX) return DSV_BAD_SHAPE;
    if (batch == 0) return DSV_OK;
    if (!table || !inv_temp || !top_k || !top_p || !min_p || !greedy || !u || !candidates ||
        !greedy_tok || !out_tok || !out_q)
        return DSV_BAD_POINTER;
    dsv::SampleChainArgs a = {batch, block_size - 1, k, table, inv_temp, top_k, top_p, min_p,
                              greedy, u, candidates, greedy_tok, out_tok, out_q, confidence_out};
    return counted(dsv::launch_sample_chain(a, (cudaStream_t)stream), 1);
}

int dsv_serial_table(int32_t batch, int32_t block_size, int32_t hidden, int32_t rk, int32_t k,
                     int64_t vocab, const void* raw, int64_t raw_stride, const void* norm_w,
                     const int64_t* candidates, const int64_t* input_ids, const void* lm_head,
                     int64_t lm_stride, int32_t head_candidates, const void* tg, const void* tsv,
                     const void* query, int64_t query_stride, const float* rms,
                     const void* gate_b, int64_t* idx, float* confidence, dsv_stream_t stream) {
    if (batch < 0 || block_size < 2) return DSV_BAD_SHAPE;
    if (hidden < 512 || hidden % 512 || hidden > 16384) return DSV_BAD_SHAPE;
    if (rk < 128 || rk % 128 || k < 2 || k > dsv::serial_max_k() || (k & (k - 1))) return DSV_BAD_SHAPE;
    if (vocab < 1 || raw_stride < hidden || lm_stride < hidden || query_stride < rk) return DSV_BAD_SHAPE;
    const int64_t n = (int64_t)batch * (block_size - 1);
    if (n > INT32_MAX) return DSV_BAD_SHAPE;
    if (batch == 0) return DSV_OK;
    if (!raw || !norm_w || !candidates || !input_ids || !lm_head || !tg || !tsv || !query ||
        !rms || !gate_b || !idx)
        return DSV_BAD_POINTER;
    if (!aligned(lm_head, 16) || lm_stride % 8) return DSV_BAD_ALIGNMENT;
    if (!aligned(query, 4) || query_stride % 2 || !aligned(tg, 4) || !aligned(tsv, 4) ||
        !aligned(gate_b, 4))
        return DSV_BAD_ALIGNMENT;
    dsv::TableArgs a;
    a.n = (int)n;
    a.t = block_size;
    a.h = hidden;
    a.rk = rk;
    a.k = k;
    a.vocab = vocab;
    a.raw = static_cast<const __nv_bfloat16*>(raw);
    a.raw_stride = raw_stride;
    a.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
    a.cand = candidates;
    a.input_ids = input_ids;
    a.lm_w = static_cast<const __nv_bfloat16*>(lm_head);
    a.w_stride = lm_stride;
    a.head_candidates = head_candidates != 0;
    a.tg = static_cast<const __nv_bfloat16*>(tg);
    a.tsv = static_cast<const __nv_bfloat16*>(tsv);
    a.query = static_cast<const __nv_bfloat16*>(query);
    a.q_stride = query_stride;
    a.rms = rms;
    a.gate_b = static_cast<const __nv_bfloat16*>(gate_b);
    a.idx = idx;
    a.confidence = confidence;
    return counted(dsv::launch_serial_table(a, (cudaStream_t)stream), 1);
}

int dsv_serial_chain(int32_t batch, int32_t block_size, int32_t k, const int64_t* idx,
                     const int64_t* candidates, int64_t* out, const float* confidence,
                     float* confidence_out, dsv_stream_t stream) {
    if (batch < 0 || block_size < 2 || k < 1) return DSV_BAD_SHAPE;
    if (dsv::serial_chain_smem(block_size - 1, k) > 200 * 1024) return DSV_UNSUPPORTED;
    if ((confidence == nullptr) != (confidence_out == nullptr)) return DSV_BAD_POINTER;
    if (batch == 0) return DSV_OK;
    if (!idx || !candidates || !out) return DSV_BAD_POINTER;
    return counted(dsv::launch_serial_chain(batch, block_size - 1, k, idx, candidates, out,
                                            confidence, confidence_out, (cudaStream_t)stream),
                   1);
}

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
                              uint32_t* device_error, dsv_stream_t stream) {
    if (batch < 0) return DSV_BAD_SHAPE;
    if (batch > kNoAllocMaxBatch) return DSV_WORKSPACE_TOO_SMALL;
    if (batch == 0) return DSV_OK;
    char* ws = static_cast<char*>(noalloc_scratch());
    if (ws == nullptr) return DSV_LAUNCH_FAILED;
    const size_t used = dsv::verify_base_bytes(batch);  // scratch without split rows
    cudaStream_t st = (cudaStream_t)stream;
    // counters, the error word and the greedy maxima must start at zero; clearing the whole
    // used prefix also drops whatever an earlier call that failed on the device left behind
    if (cudaMemsetAsync(ws, 0, used, st) != cudaSuccess) return DSV_LAUNCH_FAILED;
    const int status = dsv_verify_logits(
        batch, vocab, dtype, candidates, target_logits, target_row, target_rows, draft_logits,
        draft_row, draft_rows, row_stride, temperature, top_k, top_p, verify_lens, uniforms,
        uniform_final, prefix_lens, accept, commit, bonus, output, new_seq, compact, ws, used,
        stream);
    if (status != DSV_OK) return status;
    if (device_error != nullptr &&
        cudaMemcpyAsync(device_error, ws + offsetof(dsv::WsHeader, err), sizeof(uint32_t),
                        cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return DSV_LAUNCH_FAILED;
    return DSV_OK;
}

}  // extern "C"
