// verify.cu -- fused draft-block verification from logits (sm_100a).
//
// Reference path (package sglang_dspine):
//   runtime/worker.py:440-508   build_dspine_target_probs / filter_target_probs   (p, q)
//   sampling/rejection.py:12-98  _sample_capped_chain                               (chain+bonus)
//   runtime/worker.py:511-581   dspine_accept_sampling                              (the caller)
//
// Work unit ("task") = (request b, verify position s): target row s and, for sampled requests
// with s < cap-1, draft row s.  A task is split across a thread-block cluster of kC CTAs:
// CTA r owns the vocabulary slice [r*S, r*S+S) of both rows, bulk-copied into shared memory
// once (cp.async.bulk + mbarrier).  Every later pass reads shared memory; cross-CTA
// reductions go through distributed shared memory between cluster barriers.  Per task:
//   pass A   max key / first argmax of each row
//   levels   radix histograms over logit keys (count + exact fixed-point mass) that narrow
//            the joint top-k / top-p boundary to one key value and a tie count
//   ties     if ties straddle the boundary: per-CTA tie counts and the drafted token's rank
//   decide   p and q of the drafted token -> d_s = q>0 && q<=1 && u*q < p
//   bonus    if the chain can stop on this row (d_s false or s == cap-1): the residual
//            (p - q)+ (or p) inverse-CDF draw, exact in 2^-40 fixed point
// The last task of a request to finish walks d_0..d_{cap-2}, takes the bonus drawn on the row
// where the chain stopped, and writes the five outputs.  The last request to finish packs the
// accepted tokens and KV slots when compaction outputs are given.
//
// Every branch that contains a cluster barrier depends only on values all CTAs of the cluster
// compute identically (task id, request parameters, exactly reduced statistics).

#include <cooperative_groups.h>

#include <mutex>

#include "dsv_common.cuh"
#include "dsv_kernels.h"

namespace cg = cooperative_groups;

namespace dsv {

namespace {

#ifndef DSV_VERIFY_THREADS
#define DSV_VERIFY_THREADS 1024
#endif
// threads per CTA: one CTA per SM (two staged fp32 slices fill its shared memory), so the
// per-element exp and fixed-point work of the passes needs all the SM's warps (config 0,
// fp32: 0.145 ms per call at 1024 threads against 0.157 at 512 and 0.226 at 256)
constexpr int kNT = DSV_VERIFY_THREADS;
constexpr int kNW = kNT / 32;
constexpr int kBins = 256;

// Published per barrier parity; read by the other CTAs of the cluster after the barrier.
struct __align__(16) Pub {
    uint32_t hcnt[2][kBins];
    unsigned long long hmass[2][kBins];
    unsigned long long ssum[2];
    unsigned long long rmass;
    uint32_t maxkey[2];
    int32_t argmax[2];
    uint32_t tie_cnt[2];
    int32_t cand_rank[2];
};

struct RowState {
    int greedy;
    int k_on, p_on;
    int k;
    float top_p;
    float mp;           // min-p (0: no floor)
    int thr_preset;     // thr was set before the walk (sequential mode: from the top-k mass)
    float c;            // log2(e) / T
    float m;            // max logit
    int argmax;
    int done;           // kept set determined
    int keep_all;
    uint32_t prefix;    // radix prefix of the boundary bucket
    int shift;
    uint32_t cnt_above;
    unsigned long long mass_above;
    long long thr;
    uint32_t kstar;
    int tstar;
    int partial;
    unsigned long long s_total;
    unsigned long long s_kept;
    float inv_s;
    uint32_t tie_prefix;
    uint32_t tie_local;
    int local_cut;      // kept ties of this slice: index <= local_cut
    int cand_kept;      // drafted token is a kept tie (partial rows)
    long long row;
};

struct Task {
    int b, s, cap;
    int has_draft, onehot_q;
    float u, uf;
    long long cand;
    int need_bonus, pure;
    int d;
    float p, q;
};

struct Shared {
    Pub pub[2];
    uint32_t rcnt[2][kBins];
    unsigned long long rmh[2][kBins];
    RowState rs[2];
    Task tk;
    uint64_t bar;
    int task_slot[2];
    uint32_t red_k[kNW];
    int red_i[kNW];
    unsigned long long red_u64[kNW];
    uint32_t red_u32[kNW];
    int flag_final;
    int flag_compact;
    int cut_found;
    int skip;          // rank 0: the task (or its bonus) cannot change the request's outcome
    unsigned long long seg[1];  // segment sums; sized at launch
};

template <typename T>
struct Ctx {
    const VerifyArgs* a;
    Shared* sh;
    T* buf[2];
    int lo, n, nvec;
    int rank;
    int bar_i;          // cluster barriers passed (uniform across the cluster)
    uint32_t phase;     // mbarrier phase of this CTA
};

// ---------------------------------------------------------------------------------------
// block reductions

__device__ __forceinline__ void block_max_key(Shared* sh, uint32_t& key, int& idx) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        uint32_t k2 = __shfl_xor_sync(0xffffffffu, key, o);
        int i2 = __shfl_xor_sync(0xffffffffu, idx, o);
        if (k2 > key || (k2 == key && i2 < idx)) { key = k2; idx = i2; }
    }
    if (lane == 0) { sh->red_k[w] = key; sh->red_i[w] = idx; }
    __syncthreads();
    key = 0;
    idx = 0x7fffffff;
    for (int q = 0; q < kNW; ++q) {
        uint32_t k2 = sh->red_k[q];
        int i2 = sh->red_i[q];
        if (k2 > key || (k2 == key && i2 < idx)) { key = k2; idx = i2; }
    }
    __syncthreads();
}

__device__ __forceinline__ uint32_t block_sum_u32(Shared* sh, uint32_t v) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    v = warp_sum_u32(v);
    if (lane == 0) sh->red_u32[w] = v;
    __syncthreads();
    uint32_t t = 0;
    for (int q = 0; q < kNW; ++q) t += sh->red_u32[q];
    __syncthreads();
    return t;
}

// ---------------------------------------------------------------------------------------
// element helpers

__device__ __forceinline__ float row_e(const RowState& rs, float lf) {
    return exp2c(__fmul_rn(__fsub_rn(lf, rs.m), rs.c));
}

__device__ __forceinline__ bool key_kept(const RowState& rs, uint32_t key, int gidx) {
    if (rs.keep_all || key > rs.kstar) return true;
    if (key < rs.kstar) return false;
    return !rs.partial || gidx <= rs.local_cut;
}

template <typename T>
__device__ __forceinline__ float row_prob(const RowState& rs, uint32_t u, int gidx) {
    using E = Elem<T>;
    if (rs.greedy) return gidx == rs.argmax ? 1.0f : 0.0f;
    if (!key_kept(rs, E::key(u), gidx)) return 0.0f;
    return __fmul_rn(row_e(rs, E::to_float(u)), rs.inv_s);
}

// residual weight (p - q)+ of element gidx, or p when the draw is pure
template <typename T>
__device__ __forceinline__ float elem_w(const Shared* sh, uint32_t up, uint32_t uq, int gidx) {
    const Task& tk = sh->tk;
    float p = row_prob<T>(sh->rs[0], up, gidx);
    if (tk.pure || p == 0.0f) return p;
    float q;
    if (tk.onehot_q) q = (gidx == tk.cand) ? 1.0f : 0.0f;
    else q = row_prob<T>(sh->rs[1], uq, gidx);
    q = (q >= 0.0f && q <= 1.0f) ? q : 0.0f;
    return fmaxf(__fsub_rn(p, q), 0.0f);
}

// ---------------------------------------------------------------------------------------
// stages

template <typename T>
__device__ bool load_slices(Ctx<T>& cx, int nrows) {
    using E = Elem<T>;
    const VerifyArgs& a = *cx.a;
    Shared* sh = cx.sh;
    const int tid = threadIdx.x;
    bool ok = true;
    __syncthreads();
    if (cx.n <= 0) return ok;
    const T* src[2];
    int bulk[2] = {0, 0};
    uint32_t total = 0;
    for (int r = 0; r < nrows; ++r) {
        const T* base = reinterpret_cast<const T*>(r == 0 ? a.tgt : a.drf);
        src[r] = base + sh->rs[r].row * a.stride + cx.lo;
        const int full = (cx.n / E::kEV) * E::kEV;
        if ((reinterpret_cast<uintptr_t>(src[r]) & 15u) == 0 && full > 0) {
            bulk[r] = full;
            total += (uint32_t)full * (uint32_t)sizeof(T);
        }
    }
    if (total) {
        if (tid == 0) {
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&sh->bar, total);
            for (int r = 0; r < nrows; ++r) {
                if (!bulk[r]) continue;
                const char* s = reinterpret_cast<const char*>(src[r]);
                char* d = reinterpret_cast<char*>(cx.buf[r]);
                const uint32_t bytes = (uint32_t)bulk[r] * (uint32_t)sizeof(T);
                for (uint32_t off = 0; off < bytes; off += 32768u)
                    bulk_g2s(d + off, s + off, min(32768u, bytes - off), &sh->bar);
            }
        }
    }
    for (int r = 0; r < nrows; ++r)
        for (int i = bulk[r] + tid; i < cx.n; i += kNT) cx.buf[r][i] = src[r][i];
    if (total) {
        if (!mbar_wait_bounded(&sh->bar, cx.phase & 1u)) {
            ok = false;
            if (tid == 0) atomicOr(&a.ws->err, 1u);
        }
        cx.phase++;
    }
    __syncthreads();
    return ok;
}

// pass A: max key and its first index per row; reduced across the cluster.
template <typename T, int kC>
__device__ void pass_max(Ctx<T>& cx, cg::cluster_group& cluster, int nrows) {
    using E = Elem<T>;
    Shared* sh = cx.sh;
    Pub& pb = sh->pub[cx.bar_i & 1];
    for (int r = 0; r < nrows; ++r) {
        uint32_t best = 0;
        int bidx = 0x7fffffff;
        const uint4* vb = reinterpret_cast<const uint4*>(cx.buf[r]);
        for (int v = threadIdx.x; v < cx.nvec; v += kNT) {
            uint32_t u[E::kEV];
            E::unpack(vb[v], u);
#pragma unroll
            for (int j = 0; j < E::kEV; ++j) {
                const int li = v * E::kEV + j;
                if (li < cx.n) {
                    const uint32_t key = E::key(u[j]);
                    if (key > best) { best = key; bidx = cx.lo + li; }
                }
            }
        }
        block_max_key(sh, best, bidx);
        if (threadIdx.x == 0) { pb.maxkey[r] = best; pb.argmax[r] = bidx; }
    }
    cluster.sync();
    const int pi = cx.bar_i & 1;
    cx.bar_i++;
    if (threadIdx.x < nrows) {
        const int r = threadIdx.x;
        uint32_t best = 0;
        int bidx = 0x7fffffff;
#pragma unroll
        for (int q = 0; q < kC; ++q) {
            const Pub* rp = cluster.map_shared_rank(&sh->pub[pi], q);
            const uint32_t k2 = rp->maxkey[r];
            const int i2 = rp->argmax[r];
            if (k2 > best || (k2 == best && i2 < bidx)) { best = k2; bidx = i2; }
        }
        RowState& rs = sh->rs[r];
        rs.argmax = bidx;
        rs.m = E::key_to_float(best);
    }
    __syncthreads();
}

// one radix level: histogram of digit (key >> shift) & 255 among keys with the row's prefix
template <typename T>
__device__ void hist_pass(Ctx<T>& cx, Pub& pb, bool first, const bool* mask) {
    using E = Elem<T>;
    Shared* sh = cx.sh;
    for (int i = threadIdx.x; i < 2 * kBins; i += kNT) {
        (&pb.hcnt[0][0])[i] = 0u;
        (&pb.hmass[0][0])[i] = 0ull;
    }
    if (threadIdx.x < 2) pb.ssum[threadIdx.x] = 0ull;
    __syncthreads();
    for (int r = 0; r < 2; ++r) {
        if (!mask[r]) continue;
        const RowState& rs = sh->rs[r];
        const int shift = rs.shift;
        const uint32_t prefix = rs.prefix;
        const bool filtered = rs.k_on || rs.p_on;
        unsigned long long acc = 0;
        const uint4* vb = reinterpret_cast<const uint4*>(cx.buf[r]);
        for (int v = threadIdx.x; v < cx.nvec; v += kNT) {
            uint32_t u[E::kEV];
            E::unpack(vb[v], u);
#pragma unroll
            for (int j = 0; j < E::kEV; ++j) {
                const int li = v * E::kEV + j;
                if (li < cx.n) {
                    const uint32_t key = E::key(u[j]);
                    if (first || (key >> (shift + 8)) == prefix) {
                        const float y = __fmul_rn(__fsub_rn(E::to_float(u[j]), rs.m), rs.c);
                        // fix(exp2(y)) == 0 exactly for y <= -41
                        const uint64_t F = (y > -41.0f) ? fix01(exp2c(y)) : 0ull;
                        if (filtered) {
                            const uint32_t d = (key >> shift) & 255u;
                            atomicAdd(&pb.hcnt[r][d], 1u);
                            if (F) atomicAdd(&pb.hmass[r][d], (unsigned long long)F);
                        } else {
                            acc += F;
                        }
                    }
                }
            }
        }
        if (!filtered) {
            acc = warp_sum_u64(acc);
            if ((threadIdx.x & 31) == 0) atomicAdd(&pb.ssum[r], acc);
        }
    }
}

// After the level barrier: reduce all CTAs' histograms, then warp r walks row r's buckets
// from the top and narrows the boundary (or finishes the row).
template <int kC>
__device__ void level_scan(Shared* sh, cg::cluster_group& cluster, int pi, bool first,
                           const bool* mask) {
    for (int i = threadIdx.x; i < 2 * kBins; i += kNT) {
        const int r = i / kBins, d = i % kBins;
        if (!mask[r]) continue;
        uint32_t c = 0;
        unsigned long long m = 0;
#pragma unroll
        for (int q = 0; q < kC; ++q) {
            const Pub* rp = cluster.map_shared_rank(&sh->pub[pi], q);
            c += rp->hcnt[r][d];
            m += rp->hmass[r][d];
        }
        sh->rcnt[r][d] = c;
        sh->rmh[r][d] = m;
    }
    if (threadIdx.x < 2 && mask[threadIdx.x] && first) {
        RowState& rs = sh->rs[threadIdx.x];
        if (!rs.k_on && !rs.p_on) {
            unsigned long long s = 0;
#pragma unroll
            for (int q = 0; q < kC; ++q) s += cluster.map_shared_rank(&sh->pub[pi], q)->ssum[threadIdx.x];
            rs.s_total = s;
            rs.s_kept = s;
            rs.keep_all = 1;
            rs.done = 1;
            rs.inv_s = inv_from_fix(s);
        }
    }
    __syncthreads();
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (w < 2 && mask[w] && !sh->rs[w].done) {
        RowState& rs = sh->rs[w];
        // lane covers buckets 255-8*lane down to 248-8*lane (descending key order)
        uint32_t lc = 0;
        unsigned long long lm = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int d = 255 - 8 * lane - j;
            lc += sh->rcnt[w][d];
            lm += sh->rmh[w][d];
        }
        long long thr = rs.thr;
        if (first) {
            const unsigned long long tot = warp_sum_u64(lm);
            if (!rs.thr_preset) {
                thr = 0x7fffffffffffffffll;
                if (rs.p_on) {
                    thr = scale_floor(rs.top_p, tot);
                    if (thr < 0) thr = 0;  // top_p <= 0: only the first element survives
                }
            }
            if (lane == 0) { rs.s_total = tot; rs.thr = thr; }
        }
        const uint32_t ic = warp_incl_u32(lc);
        const unsigned long long im = warp_incl_u64(lm);
        uint32_t N = rs.cnt_above + (ic - lc);
        unsigned long long A = rs.mass_above + (im - lm);
        int found = -1;
        uint32_t fN = 0, fc = 0;
        unsigned long long fA = 0, fm = 0;
        for (int j = 0; j < 8; ++j) {
            const int d = 255 - 8 * lane - j;
            const uint32_t c = sh->rcnt[w][d];
            const unsigned long long m = sh->rmh[w][d];
            const bool trig = (rs.k_on && (N + c >= (uint32_t)rs.k)) ||
                              (rs.p_on && (long long)(A + m) > thr);
            if (c && trig) { found = d; fN = N; fA = A; fc = c; fm = m; break; }
            N += c;
            A += m;
        }
        const unsigned bal = __ballot_sync(0xffffffffu, found >= 0);
        if (bal == 0) {
            if (lane == 0) {  // no limit binds: every element is kept
                rs.keep_all = 1;
                rs.done = 1;
                rs.s_kept = rs.s_total;
                rs.inv_s = inv_from_fix(rs.s_total);
            }
        } else {
            const int src = __ffs(bal) - 1;
            found = __shfl_sync(0xffffffffu, found, src);
            fN = __shfl_sync(0xffffffffu, fN, src);
            fA = __shfl_sync(0xffffffffu, fA, src);
            fc = __shfl_sync(0xffffffffu, fc, src);
            fm = __shfl_sync(0xffffffffu, fm, src);
            if (lane == 0) {
                if (rs.shift == 0) {
                    // one key value: fc elements of equal mass f
                    rs.kstar = (rs.prefix << 8) | (uint32_t)found;
                    const unsigned long long f = fm / fc;
                    const long long g = fc;
                    long long t = g;
                    if (rs.k_on) { const long long tk = (long long)rs.k - (long long)fN; if (tk < t) t = tk; }
                    if (rs.p_on && f > 0) {
                        const long long tp = (thr - (long long)fA) / (long long)f + 1;
                        if (tp < t) t = tp;
                    }
                    if (t < 1) t = 1;
                    rs.tstar = (int)t;
                    rs.partial = (t < g);
                    rs.s_kept = fA + (unsigned long long)t * f;
                    rs.inv_s = inv_from_fix(rs.s_kept);
                    rs.done = 1;
                } else {
                    rs.prefix = (rs.prefix << 8) | (uint32_t)found;
                    rs.cnt_above = fN;
                    rs.mass_above = fA;
                    rs.shift -= 8;
                }
            }
        }
    }
    __syncthreads();
}

template <typename T, int kC>
__device__ void radix_levels(Ctx<T>& cx, cg::cluster_group& cluster, int nrows) {
    Shared* sh = cx.sh;
    bool first = true;
    for (;;) {
        bool mask[2] = {!sh->rs[0].done, nrows > 1 && !sh->rs[1].done};
        if (!mask[0] && !mask[1]) break;
        hist_pass<T>(cx, sh->pub[cx.bar_i & 1], first, mask);
        cluster.sync();
        const int pi = cx.bar_i & 1;
        cx.bar_i++;
        level_scan<kC>(sh, cluster, pi, first, mask);
        first = false;
    }
}

// min-p: count the elements at or above each row's floor (minp_floor32 of its maximum) over
// the cluster and cap the row's top-k at that count (the kept set stays a prefix of the rank
// order).  All CTAs of the cluster call it.
template <typename T, int kC>
__device__ void minp_pass(Ctx<T>& cx, cg::cluster_group& cluster, int nrows) {
    using E = Elem<T>;
    Shared* sh = cx.sh;
    Pub& pb = sh->pub[cx.bar_i & 1];
    for (int r = 0; r < nrows; ++r) {
        const RowState& rs = sh->rs[r];
        uint32_t cnt = 0;
        if (!rs.done && rs.mp > 0.0f) {
            const uint32_t f32 = minp_floor32(rs.m, rs.c, rs.mp);
            const uint32_t kf = E::kKeyBits == 16 ? key16_floor(f32) : f32;
            const bool none = E::kKeyBits == 16 && kf > 0xFFFFu;
            const uint4* vb = reinterpret_cast<const uint4*>(cx.buf[r]);
            for (int v = threadIdx.x; v < cx.nvec && !none; v += kNT) {
                uint32_t u[E::kEV];
                E::unpack(vb[v], u);
#pragma unroll
                for (int j = 0; j < E::kEV; ++j) {
                    const int li = v * E::kEV + j;
                    if (li < cx.n && E::key(u[j]) >= kf) ++cnt;
                }
            }
        }
        cnt = block_sum_u32(sh, cnt);
        if (threadIdx.x == 0) pb.tie_cnt[r] = cnt;
    }
    cluster.sync();
    const int pi = cx.bar_i & 1;
    cx.bar_i++;
    if (threadIdx.x < nrows) {
        RowState& rs = sh->rs[threadIdx.x];
        if (!rs.done && rs.mp > 0.0f) {
            uint32_t total = 0;
#pragma unroll
            for (int q = 0; q < kC; ++q)
                total += cluster.map_shared_rank(&sh->pub[pi], q)->tie_cnt[threadIdx.x];
            long long k = rs.k_on ? (long long)rs.k : (long long)cx.a->V;
            if ((long long)total < k) k = (long long)total;
            if (k < 1) k = 1;
            if (k < (long long)cx.a->V) {
                rs.k = (int)k;
                rs.k_on = 1;
            }
        }
    }
    __syncthreads();
}

// sequential mode (flashinfer with min-p in the batch): top-p is taken against the mass of the
// row's top-k elements.  A walk with the top-k alone gives that mass; the rows are then reset
// for the final walk with the threshold preset.
__device__ void seq_prepare(Shared* sh, int nrows, int key_bits, bool first_stage) {
    if (threadIdx.x < nrows) {
        RowState& rs = sh->rs[threadIdx.x];
        if (first_stage) {
            rs.p_on = 0;
        } else {
            long long thr = scale_floor(rs.top_p, rs.s_kept);
            if (thr < 0) thr = 0;
            rs.thr = thr;
            rs.thr_preset = 1;
            rs.p_on = 1;
            rs.done = 0;
            rs.keep_all = 0;
            rs.prefix = 0;
            rs.shift = key_bits - 8;
            rs.cnt_above = 0;
            rs.mass_above = 0;
            rs.kstar = 0;
            rs.tstar = 0;
            rs.partial = 0;
            rs.s_kept = 0;
            rs.inv_s = 0.0f;
        }
    }
    __syncthreads();
}

// The kept set of the task's rows: the sequential mode's top-k mass first, the min-p cap, then
// the radix walk.  Both rows of a task belong to one request, so they share the mode.
template <typename T, int kC>
__device__ void select_rows(Ctx<T>& cx, cg::cluster_group& cluster, int nrows) {
    Shared* sh = cx.sh;
    const RowState& r0 = sh->rs[0];
    const bool seq = cx.a->mode == kModeSeq && !r0.done && r0.k_on && r0.p_on;
    const bool minp = r0.mp > 0.0f && !r0.done;
    __syncthreads();  // every thread has read the row state before seq_prepare changes it
    if (seq) {
        seq_prepare(sh, nrows, Elem<T>::kKeyBits, true);
        radix_levels<T, kC>(cx, cluster, nrows);
        seq_prepare(sh, nrows, Elem<T>::kKeyBits, false);
    }
    if (minp) minp_pass<T, kC>(cx, cluster, nrows);
    radix_levels<T, kC>(cx, cluster, nrows);
}

// Ties straddle the boundary of a row: count them per CTA, locate the drafted token among
// them, and decide whether the drafted token is kept.
template <typename T, int kC>
__device__ void tie_pass(Ctx<T>& cx, cg::cluster_group& cluster, int nrows) {
    using E = Elem<T>;
    Shared* sh = cx.sh;
    Pub& pb = sh->pub[cx.bar_i & 1];
    const long long cnd = sh->tk.cand;
    for (int r = 0; r < nrows; ++r) {
        const RowState& rs = sh->rs[r];
        uint32_t cnt = 0, before = 0;
        if (rs.partial) {
            const uint4* vb = reinterpret_cast<const uint4*>(cx.buf[r]);
            for (int v = threadIdx.x; v < cx.nvec; v += kNT) {
                uint32_t u[E::kEV];
                E::unpack(vb[v], u);
#pragma unroll
                for (int j = 0; j < E::kEV; ++j) {
                    const int li = v * E::kEV + j;
                    if (li < cx.n && E::key(u[j]) == rs.kstar) {
                        ++cnt;
                        if (cx.lo + li < cnd) ++before;
                    }
                }
            }
        }
        cnt = block_sum_u32(sh, cnt);
        before = block_sum_u32(sh, before);
        if (threadIdx.x == 0) {
            pb.tie_cnt[r] = cnt;
            int rk = -1;
            if (rs.partial && cnd >= cx.lo && cnd < cx.lo + cx.n) {
                const uint32_t uc = E::raw(cx.buf[r], (int)(cnd - cx.lo));
                if (E::key(uc) == rs.kstar) rk = (int)before;
            }
            pb.cand_rank[r] = rk;
        }
    }
    cluster.sync();
    const int pi = cx.bar_i & 1;
    cx.bar_i++;
    if (threadIdx.x < nrows) {
        RowState& rs = sh->rs[threadIdx.x];
        if (rs.partial) {
            uint32_t run = 0, pre = 0, mine = 0, cpre = 0;
            int crank = -1;
#pragma unroll
            for (int q = 0; q < kC; ++q) {
                const Pub* rp = cluster.map_shared_rank(&sh->pub[pi], q);
                const uint32_t tc = rp->tie_cnt[threadIdx.x];
                const int cr = rp->cand_rank[threadIdx.x];
                if (cr >= 0) { crank = cr; cpre = run; }
                if (q == cx.rank) { pre = run; mine = tc; }
                run += tc;
            }
            rs.tie_prefix = pre;
            rs.tie_local = mine;
            rs.cand_kept = (crank >= 0) && ((uint32_t)crank + cpre < (uint32_t)rs.tstar);
        }
    }
    __syncthreads();
}

// p / q of the drafted token and the accept decision (thread 0; every CTA computes it)
template <typename T>
__device__ void decide(Ctx<T>& cx, int nrows) {
    using E = Elem<T>;
    const VerifyArgs& a = *cx.a;
    Shared* sh = cx.sh;
    Task& tk = sh->tk;
    if (threadIdx.x == 0) {
        const long long cnd = tk.cand;
        const bool valid = cnd >= 0 && cnd < a.V;
        float pq[2] = {0.0f, 0.0f};
        if (valid) {
            for (int r = 0; r < 2; ++r) {
                const RowState& rs = sh->rs[r];
                if (r == 1 && tk.onehot_q) { pq[1] = 1.0f; break; }
                if (r >= nrows) break;
                if (rs.greedy) { pq[r] = (cnd == rs.argmax) ? 1.0f : 0.0f; continue; }
                const T* rowp = reinterpret_cast<const T*>(r == 0 ? a.tgt : a.drf) + rs.row * a.stride;
                const uint32_t uc = E::raw(rowp, (int)cnd);
                const uint32_t key = E::key(uc);
                bool kept;
                if (rs.keep_all || key > rs.kstar) kept = true;
                else if (key < rs.kstar) kept = false;
                else kept = !rs.partial || rs.cand_kept;
                pq[r] = kept ? __fmul_rn(row_e(rs, E::to_float(uc)), rs.inv_s) : 0.0f;
            }
        }
        int d = 0;
        if (tk.s < tk.cap - 1) {
            const float p = pq[0], q = pq[1];
            d = (q > 0.0f && q <= 1.0f && __fmul_rn(tk.u, q) < p) ? 1 : 0;
        }
        tk.d = d;
        tk.p = pq[0];
        tk.q = pq[1];
        tk.need_bonus = (!d) || (tk.s == tk.cap - 1);
        tk.pure = (tk.s == tk.cap - 1);
    }
    __syncthreads();
}

// The boundary CTA of a partial row finds its local tie cut: the first (tstar - tie_prefix)
// ties of its slice, in index order, are kept.
template <typename T>
__device__ void local_cuts(Ctx<T>& cx, int nrows) {
    using E = Elem<T>;
    Shared* sh = cx.sh;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    for (int r = 0; r < nrows; ++r) {
        RowState& rs = sh->rs[r];
        if (!rs.partial) continue;
        const long long want = (long long)rs.tstar - (long long)rs.tie_prefix;
        if (want <= 0 || want >= (long long)rs.tie_local) {
            __syncthreads();
            if (tid == 0) rs.local_cut = (want <= 0) ? -1 : 0x7fffffff;
            __syncthreads();
            continue;
        }
        if (tid == 0) sh->cut_found = -1;
        __syncthreads();
        uint32_t base = 0;
        const uint4* vb = reinterpret_cast<const uint4*>(cx.buf[r]);
        for (int v0 = 0; v0 < cx.nvec; v0 += kNT) {
            const int v = v0 + tid;
            uint32_t u[E::kEV];
            uint32_t cntv = 0;
            if (v < cx.nvec) {
                E::unpack(vb[v], u);
#pragma unroll
                for (int j = 0; j < E::kEV; ++j) {
                    const int li = v * E::kEV + j;
                    if (li < cx.n && E::key(u[j]) == rs.kstar) ++cntv;
                }
            }
            const uint32_t inc = warp_incl_u32(cntv);
            if (lane == 31) sh->red_u32[w] = inc;
            __syncthreads();
            uint32_t wpre = 0, tot = 0;
            for (int q = 0; q < kNW; ++q) {
                const uint32_t x = sh->red_u32[q];
                if (q < w) wpre += x;
                tot += x;
            }
            const uint32_t excl = base + wpre + inc - cntv;
            if (cntv && excl < (uint32_t)want && excl + cntv >= (uint32_t)want) {
                uint32_t k = excl;
#pragma unroll
                for (int j = 0; j < E::kEV; ++j) {
                    const int li = v * E::kEV + j;
                    if (li < cx.n && E::key(u[j]) == rs.kstar) {
                        ++k;
                        if (k == (uint32_t)want) sh->cut_found = cx.lo + li;
                    }
                }
            }
            __syncthreads();
            base += tot;
            if (base >= (uint32_t)want) break;
        }
        __syncthreads();
        if (tid == 0) rs.local_cut = sh->cut_found;
        __syncthreads();
    }
}

// residual pass over this CTA's slice: per (round, warp) segment sums of fix(w); returns the
// CTA total (valid in every thread)
template <typename T>
__device__ unsigned long long residual_pass(Ctx<T>& cx, bool use_q) {
    using E = Elem<T>;
    Shared* sh = cx.sh;
    const int tid = threadIdx.x;
    const uint4* vp = reinterpret_cast<const uint4*>(cx.buf[0]);
    const uint4* vq = reinterpret_cast<const uint4*>(cx.buf[1]);
    unsigned long long local = 0;
    int round = 0;
    for (int v0 = 0; v0 < cx.nvec; v0 += kNT, ++round) {
        const int v = v0 + tid;
        unsigned long long acc = 0;
        if (v < cx.nvec) {
            uint32_t up[E::kEV], uq[E::kEV];
            E::unpack(vp[v], up);
            if (use_q) {
                E::unpack(vq[v], uq);
            } else {
#pragma unroll
                for (int j = 0; j < E::kEV; ++j) uq[j] = 0;
            }
#pragma unroll
            for (int j = 0; j < E::kEV; ++j) {
                const int li = v * E::kEV + j;
                if (li < cx.n) acc += fixv(elem_w<T>(sh, up[j], uq[j], cx.lo + li));
            }
        }
        acc = warp_sum_u64(acc);
        if ((tid & 31) == 0) sh->seg[round * kNW + (tid >> 5)] = acc;
        local += acc;
    }
    if ((tid & 31) == 0) sh->red_u64[tid >> 5] = local;
    __syncthreads();
    unsigned long long tot = 0;
    for (int q = 0; q < kNW; ++q) tot += sh->red_u64[q];
    __syncthreads();
    return tot;
}

// find the element where the local cumulative fix(w) first exceeds tl (warp 0)
template <typename T>
__device__ int crossing(Ctx<T>& cx, bool use_q, unsigned long long tl) {
    using E = Elem<T>;
    Shared* sh = cx.sh;
    const int lane = threadIdx.x & 31;
    const int nrounds = (cx.nvec + kNT - 1) / kNT;
    const int nseg = nrounds * kNW;
    unsigned long long run = 0;
    int segf = -1;
    for (int j0 = 0; j0 < nseg; j0 += 32) {
        const int j = j0 + lane;
        const unsigned long long x = j < nseg ? sh->seg[j] : 0ull;
        const unsigned long long inc = warp_incl_u64(x);
        const unsigned bal = __ballot_sync(0xffffffffu, run + inc > tl);
        if (bal) {
            const int src = __ffs(bal) - 1;
            run += __shfl_sync(0xffffffffu, inc - x, src);
            segf = j0 + src;
            break;
        }
        run += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (segf < 0) return -1;
    const int v = (segf / kNW) * kNT + (segf % kNW) * 32 + lane;
    const uint4* vp = reinterpret_cast<const uint4*>(cx.buf[0]);
    const uint4* vq = reinterpret_cast<const uint4*>(cx.buf[1]);
    unsigned long long wv[E::kEV];
    unsigned long long lsum = 0;
    if (v < cx.nvec) {
        uint32_t up[E::kEV], uq[E::kEV];
        E::unpack(vp[v], up);
        if (use_q) {
            E::unpack(vq[v], uq);
        } else {
#pragma unroll
            for (int j = 0; j < E::kEV; ++j) uq[j] = 0;
        }
#pragma unroll
        for (int j = 0; j < E::kEV; ++j) {
            const int li = v * E::kEV + j;
            wv[j] = (li < cx.n) ? fixv(elem_w<T>(sh, up[j], uq[j], cx.lo + li)) : 0ull;
            lsum += wv[j];
        }
    } else {
#pragma unroll
        for (int j = 0; j < E::kEV; ++j) wv[j] = 0;
    }
    const unsigned long long inc = warp_incl_u64(lsum);
    const unsigned long long start = run + inc - lsum;
    const bool hit = lsum > 0 && start <= tl && start + lsum > tl;
    const unsigned bal = __ballot_sync(0xffffffffu, hit);
    int idx = -1;
    if (hit && lane == __ffs(bal) - 1) {
        unsigned long long cum = start;
#pragma unroll
        for (int j = 0; j < E::kEV; ++j) {
            cum += wv[j];
            if (idx < 0 && cum > tl) idx = cx.lo + v * E::kEV + j;
        }
    }
    if (bal) idx = __shfl_sync(0xffffffffu, idx, __ffs(bal) - 1);
    return idx;
}

template <typename T, int kC>
__device__ void bonus_draw(Ctx<T>& cx, cg::cluster_group& cluster, int nrows) {
    const VerifyArgs& a = *cx.a;
    Shared* sh = cx.sh;
    Task& tk = sh->tk;
    const int tid = threadIdx.x;
    local_cuts<T>(cx, nrows);
    const bool has_q_rows = tk.has_draft;
    for (int attempt = 0; attempt < 2; ++attempt) {
        const bool use_q = has_q_rows && !tk.pure;
        const unsigned long long mine = residual_pass<T>(cx, use_q);
        if (tid == 0) sh->pub[cx.bar_i & 1].rmass = mine;
        cluster.sync();
        const int pi = cx.bar_i & 1;
        cx.bar_i++;
        unsigned long long M = 0, pre = 0;
#pragma unroll
        for (int q = 0; q < kC; ++q) {
            const unsigned long long x = cluster.map_shared_rank(&sh->pub[pi], q)->rmass;
            if (q < cx.rank) pre += x;
            M += x;
        }
        if (!tk.pure && M == 0) {
            // zero residual mass: draw from p instead (same decision in every CTA)
            __syncthreads();
            if (tid == 0) tk.pure = 1;
            __syncthreads();
            continue;
        }
        const long long thr = scale_floor(tk.uf, M);
        TaskResult* res = &a.res[tk.b * kT + tk.s];
        if (thr == -2 || thr >= (long long)M) {
            if (cx.rank == 0 && tid == 0) res->bonus = a.V - 1;
        } else if (thr < 0) {
            if (cx.rank == 0 && tid == 0) res->bonus = 0;
        } else if ((long long)pre <= thr && thr < (long long)(pre + mine)) {
            if (tid < 32) {
                const int idx = crossing<T>(cx, use_q, (unsigned long long)(thr - (long long)pre));
                if (tid == 0) res->bonus = idx;
            }
        }
        break;
    }
    __threadfence();
    cluster.sync();  // the bonus writer's store precedes rank 0's completion signal
    cx.bar_i++;
}

// ---------------------------------------------------------------------------------------
// accept-compact of the whole batch (one CTA): exclusive scan of commit and of cap - commit

__device__ void compact_block(const VerifyArgs& a, Shared* sh) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    int run_c = 0, run_f = 0;
    if (tid == 0) { a.offsets[0] = 0; a.free_offsets[0] = 0; }
    for (int b0 = 0; b0 < a.B; b0 += kNT) {
        const int b = b0 + tid;
        int cm = 0, fr = 0;
        if (b < a.B) {
            int cap = a.caps[b];
            cap = cap < 1 ? 1 : (cap > kT ? kT : cap);
            cm = __ldcg(&a.commit[b]);
            fr = cap - cm;
            if (fr < 0) fr = 0;
        }
        const uint32_t ic = warp_incl_u32((uint32_t)cm);
        const uint32_t iff = warp_incl_u32((uint32_t)fr);
        if (lane == 31) { sh->red_u32[w] = ic; sh->red_k[w] = iff; }
        __syncthreads();
        int wc = 0, wf = 0, tc = 0, tf = 0;
        for (int q = 0; q < kNW; ++q) {
            if (q < w) { wc += (int)sh->red_u32[q]; wf += (int)sh->red_k[q]; }
            tc += (int)sh->red_u32[q];
            tf += (int)sh->red_k[q];
        }
        __syncthreads();
        if (b < a.B) {
            const int oc = run_c + wc + (int)ic - cm;
            const int of = run_f + wf + (int)iff - fr;
            a.offsets[b + 1] = oc + cm;
            a.free_offsets[b + 1] = of + fr;
            const long long srow = a.slot_row[b];
            bool bad = false;
            for (int i = 0; i < cm; ++i) {
                a.tok_out[oc + i] = __ldcg(&a.output[b * kT + i]);
                const long long si = srow + i;
                const bool in = si >= 0 && si < a.slots_len;
                bad |= !in;
                a.slot_out[oc + i] = in ? a.slots[si] : -1;
            }
            for (int j = 0; j < fr; ++j) {
                const long long si = srow + cm + j;
                const bool in = si >= 0 && si < a.slots_len;
                bad |= !in;
                a.free_out[of + j] = in ? a.slots[si] : -1;
            }
            if (bad) atomicOr(&a.ws->err, 4u);
        }
        run_c += tc;
        run_f += tf;
    }
}

__device__ void finalize_request(const VerifyArgs& a, int b, int cap) {
    int acc = 0;
    for (int s = 0; s < cap - 1; ++s) {
        if (!__ldcg(&a.res[b * kT + s].d)) break;
        ++acc;
    }
    const int bo = __ldcg(&a.res[b * kT + acc].bonus);
    a.accept[b] = acc;
    a.commit[b] = acc + 1;
    a.bonus[b] = bo;
    for (int i = 0; i < kT; ++i) {
        long long v = 0;
        if (i < acc) v = a.cand[b * kT + i + 1];
        else if (i == acc) v = bo;
        a.output[b * kT + i] = v;
    }
    a.new_seq[b] = a.prefix[b] + acc + 1;
}

}  // namespace

// ---------------------------------------------------------------------------------------
// Early exit: a chain stops at its first rejected step, so a task past a known rejection of
// its request cannot change any output.  racc[2 b] holds 16 - r for the earliest rejected step
// r found so far (0: none; reset by the request's finalisation).  The decision to drop is
// rank 0's, shared through DSMEM after a cluster barrier, so every CTA of the cluster takes
// the same branches.
template <int kC>
__device__ bool cluster_past_rejection(const VerifyArgs& a, Shared* sh, cg::cluster_group& cluster,
                                       int& bar_i, int b, int s) {
    if (cluster.block_rank() == 0 && threadIdx.x == 0)
        sh->skip = a.cand != nullptr && 16 - s < (int)*(volatile unsigned*)&a.racc[2 * b];
    cluster.sync();
    bar_i++;
    return *cluster.map_shared_rank(&sh->skip, 0) != 0;
}

template <typename T, int kC>
__global__ void __launch_bounds__(kNT) verify_kernel(VerifyArgs a) {
    using E = Elem<T>;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int tid = threadIdx.x;

    const size_t slice_bytes = ((size_t)a.slice * sizeof(T) + 127) & ~(size_t)127;
    Ctx<T> cx;
    cx.a = &a;
    cx.buf[0] = reinterpret_cast<T*>(smem_raw);
    cx.buf[1] = reinterpret_cast<T*>(smem_raw + slice_bytes);
    cx.sh = reinterpret_cast<Shared*>(smem_raw + 2 * slice_bytes);
    cx.rank = (int)cluster.block_rank();
    cx.lo = cx.rank * a.slice;
    cx.n = max(0, min(a.slice, a.V - cx.lo));
    cx.nvec = (cx.n + E::kEV - 1) / E::kEV;
    cx.bar_i = 0;
    cx.phase = 0;
    Shared* sh = cx.sh;

    if (tid == 0) {
        mbar_init(&sh->bar, 1);
        fence_mbar_init();
        if (cx.rank == 0) sh->task_slot[0] = (int)atomicAdd(&a.ws->next, 1u);
    }
    cluster.sync();
    cx.bar_i++;
    const int total = a.B * kT;
    int t = *cluster.map_shared_rank(&sh->task_slot[0], 0);
    int iter = 0;

    while (t < total) {
        __syncthreads();
        if (cx.rank == 0 && tid == 0)
            sh->task_slot[(iter + 1) & 1] = (int)atomicAdd(&a.ws->next, 1u);
        const int b = t % a.B;
        const int s = t / a.B;
        int cap = a.caps[b];
        cap = cap < 1 ? 1 : (cap > kT ? kT : cap);
        if (s < cap) {
            const float Tb = a.temperature[b];
            const int topk = a.top_k[b];
            const float c = log2e_over(Tb);
            const bool greedy = is_greedy(Tb, topk, c);
            const bool has_draft = !greedy && a.drf != nullptr && s < cap - 1;
            const int nrows = has_draft ? 2 : 1;
            long long trow = a.tgt_row[b] + s;
            long long drow = has_draft ? a.drf_row[b] + s : 0;
            const bool rows_ok = trow >= 0 && trow < a.tgt_rows && (!has_draft || (drow >= 0 && drow < a.drf_rows));
            if (!rows_ok) {
                if (tid == 0) atomicOr(&a.ws->err, 2u);
                trow = 0;
                drow = 0;
            }
            if (tid == 0) {
                Task& tk = sh->tk;
                tk.b = b;
                tk.s = s;
                tk.cap = cap;
                tk.has_draft = has_draft;
                tk.onehot_q = greedy || a.drf == nullptr;
                tk.u = (s < kT - 1) ? a.u[b * (kT - 1) + s] : 0.0f;
                tk.uf = a.uf[b];
                tk.cand = (s < kT - 1) ? a.cand[b * kT + s + 1] : -1;
                tk.need_bonus = 0;
                tk.pure = 0;
                for (int r = 0; r < 2; ++r) {
                    RowState& rs = sh->rs[r];
                    rs.greedy = greedy;
                    rs.k = topk;
                    rs.k_on = !greedy && topk < a.V;
                    rs.top_p = a.top_p[b];
                    rs.p_on = !greedy && (rs.top_p < 1.0f);
                    rs.mp = (!greedy && a.mode != kModeJoint && a.min_p) ? a.min_p[b] : 0.0f;
                    rs.thr_preset = 0;
                    rs.c = c;
                    rs.done = greedy;
                    rs.keep_all = 0;
                    rs.prefix = 0;
                    rs.shift = E::kKeyBits - 8;
                    rs.cnt_above = 0;
                    rs.mass_above = 0;
                    rs.thr = 0;
                    rs.kstar = 0;
                    rs.tstar = 0;
                    rs.partial = 0;
                    rs.s_total = 0;
                    rs.s_kept = 0;
                    rs.inv_s = 0.0f;
                    rs.tie_prefix = 0;
                    rs.tie_local = 0;
                    rs.local_cut = -1;
                    rs.cand_kept = 0;
                    rs.row = (r == 0) ? trow : drow;
                }
            }
            __syncthreads();
            const bool drop = cluster_past_rejection<kC>(a, sh, cluster, cx.bar_i, b, s);
            if (!drop) {
                load_slices<T>(cx, nrows);
                if (tid == 0 && cx.n > 0)  // the workspace's count of logit bytes read
                    atomicAdd(&a.ws->bytes_read, (unsigned long long)cx.n * sizeof(T) * (unsigned)nrows);
                pass_max<T, kC>(cx, cluster, nrows);
            }
            if (drop) {
                // nothing to compute: only the completion signal below
            } else if (greedy) {
                // one-hot p at the argmax, one-hot q at the drafted token: closed form
                if (cx.rank == 0 && tid == 0) {
                    const Task& tk = sh->tk;
                    const int g = sh->rs[0].argmax;
                    const bool valid = tk.cand >= 0 && tk.cand < a.V;
                    int d = 0;
                    if (s < cap - 1) {
                        const float p = (valid && tk.cand == g) ? 1.0f : 0.0f;
                        const float q = valid ? 1.0f : 0.0f;
                        d = (q > 0.0f && q <= 1.0f && __fmul_rn(tk.u, q) < p) ? 1 : 0;
                    }
                    TaskResult* res = &a.res[b * kT + s];
                    res->d = d;
                    res->p = 0.0f;
                    res->q = 0.0f;
                    if (!d && s < cap - 1) atomicMax(&a.racc[2 * b], (unsigned)(16 - s));
                    int bonus = -1;
                    if (!d || s == cap - 1) {
                        const long long thr = scale_floor(tk.uf, 1ull << kFixBits);
                        bonus = (thr == -2) ? a.V - 1 : (thr < 0 ? 0 : g);
                    }
                    res->bonus = bonus;
                }
            } else {
                select_rows<T, kC>(cx, cluster, nrows);
                const bool anyp = sh->rs[0].partial || (nrows > 1 && sh->rs[1].partial);
                if (anyp) tie_pass<T, kC>(cx, cluster, nrows);
                decide<T>(cx, nrows);
                if (cx.rank == 0 && tid == 0) {
                    TaskResult* res = &a.res[b * kT + s];
                    res->d = sh->tk.d;
                    res->p = sh->tk.p;
                    res->q = sh->tk.q;
                    res->bonus = -1;
                    if (!sh->tk.d && s < cap - 1) atomicMax(&a.racc[2 * b], (unsigned)(16 - s));
                }
                // the bonus of a rejected step counts only if no earlier step is rejected
                if (sh->tk.need_bonus && !cluster_past_rejection<kC>(a, sh, cluster, cx.bar_i, b, s))
                    bonus_draw<T, kC>(cx, cluster, nrows);
            }

            // completion signal; the last task of the request finalizes it
            if (cx.rank == 0) {
                __syncthreads();
                if (tid == 0) {
                    __threadfence();
                    const unsigned old = atomicAdd(&a.done[b], 1u);
                    sh->flag_final = (old == (unsigned)(cap - 1));
                    sh->flag_compact = 0;
                    if (sh->flag_final) {
                        __threadfence();
                        finalize_request(a, b, cap);
                        a.done[b] = 0;
                        a.racc[2 * b] = 0u;  // the earliest rejection, for the next launch
                        __threadfence();
                        const unsigned fo = atomicAdd(&a.ws->finalized, 1u);
                        sh->flag_compact = (fo == (unsigned)(a.B - 1));
                    }
                }
                __syncthreads();
                if (sh->flag_compact) {
                    __threadfence();
                    if (a.tok_out != nullptr) compact_block(a, sh);
                    __syncthreads();
                    if (tid == 0) a.ws->finalized = 0;
                }
            }
        } else {
            cluster.sync();  // every iteration passes at least one cluster barrier
            cx.bar_i++;
        }
        t = *cluster.map_shared_rank(&sh->task_slot[(iter + 1) & 1], 0);
        ++iter;
    }
    // exit: the last cluster out resets the task counter for the next launch
    if (cx.rank == 0 && tid == 0) {
        __threadfence();
        const unsigned old = atomicAdd(&a.ws->exited, 1u);
        if (old == (unsigned)(a.num_clusters - 1)) {
            a.ws->next = 0;
            a.ws->exited = 0;
            __threadfence();
        }
    }
    // no CTA may leave while a peer can still read its shared memory
    cluster.sync();
}

// ---------------------------------------------------------------------------------------
// Dense target probabilities of logit rows (dsv_target_probs for fp32 logits): the same
// cluster-per-row selection as verify_kernel (slices staged in shared memory, radix walk,
// tie cut), then every CTA writes its slice of p.  Row t belongs to request t / row_step.

template <typename T, int kC>
__global__ void __launch_bounds__(kNT) probs_kernel(VerifyArgs a, float* out) {
    using E = Elem<T>;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int tid = threadIdx.x;
    const size_t slice_bytes = ((size_t)a.slice * sizeof(T) + 127) & ~(size_t)127;
    Ctx<T> cx;
    cx.a = &a;
    cx.buf[0] = reinterpret_cast<T*>(smem_raw);
    cx.buf[1] = reinterpret_cast<T*>(smem_raw + slice_bytes);
    cx.sh = reinterpret_cast<Shared*>(smem_raw + 2 * slice_bytes);
    cx.rank = (int)cluster.block_rank();
    cx.lo = cx.rank * a.slice;
    cx.n = max(0, min(a.slice, a.V - cx.lo));
    cx.nvec = (cx.n + E::kEV - 1) / E::kEV;
    cx.bar_i = 0;
    cx.phase = 0;
    Shared* sh = cx.sh;
    if (tid == 0) {
        mbar_init(&sh->bar, 1);
        fence_mbar_init();
        if (cx.rank == 0) sh->task_slot[0] = (int)atomicAdd(&a.ws->next, 1u);
    }
    cluster.sync();
    cx.bar_i++;
    const long long total = a.tgt_rows;
    long long t = *cluster.map_shared_rank(&sh->task_slot[0], 0);
    int iter = 0;
    while (t < total) {
        __syncthreads();
        if (cx.rank == 0 && tid == 0)
            sh->task_slot[(iter + 1) & 1] = (int)atomicAdd(&a.ws->next, 1u);
        const int b = (int)(t / a.row_step);
        const float Tb = a.temperature[b];
        const int topk = a.top_k[b];
        const float c = log2e_over(Tb);
        const bool greedy = is_greedy(Tb, topk, c);
        if (tid == 0) {
            Task& tk = sh->tk;
            tk.cand = -1;
            tk.onehot_q = 1;
            tk.pure = 1;
            RowState& rs = sh->rs[0];
            rs.greedy = greedy;
            rs.k = topk;
            rs.k_on = !greedy && topk < a.V;
            rs.top_p = a.top_p[b];
            rs.p_on = !greedy && (rs.top_p < 1.0f);
            rs.mp = (!greedy && a.mode != kModeJoint && a.min_p) ? a.min_p[b] : 0.0f;
            rs.thr_preset = 0;
            rs.c = c;
            rs.done = greedy;
            rs.keep_all = 0;
            rs.prefix = 0;
            rs.shift = E::kKeyBits - 8;
            rs.cnt_above = 0;
            rs.mass_above = 0;
            rs.thr = 0;
            rs.kstar = 0;
            rs.tstar = 0;
            rs.partial = 0;
            rs.s_total = 0;
            rs.s_kept = 0;
            rs.inv_s = 0.0f;
            rs.tie_prefix = 0;
            rs.tie_local = 0;
            rs.local_cut = -1;
            rs.cand_kept = 0;
            rs.row = t;
        }
        __syncthreads();
        load_slices<T>(cx, 1);
        pass_max<T, kC>(cx, cluster, 1);
        if (!greedy) {
            select_rows<T, kC>(cx, cluster, 1);
            if (sh->rs[0].partial) {
                tie_pass<T, kC>(cx, cluster, 1);
                local_cuts<T>(cx, 1);
            }
        }
        // this CTA's slice of the row's probabilities
        const RowState& rs = sh->rs[0];
        float* orow = out + t * (long long)a.V + cx.lo;
        for (int i = tid; i < cx.n; i += kNT) {
            const uint32_t u = E::raw(cx.buf[0], i);
            orow[i] = row_prob<T>(rs, u, cx.lo + i);
        }
        t = *cluster.map_shared_rank(&sh->task_slot[(iter + 1) & 1], 0);
        ++iter;
        cluster.sync();  // the next task's state is written only after every CTA is done here
        cx.bar_i++;
    }
    if (cx.rank == 0 && tid == 0) {
        __threadfence();
        const unsigned old = atomicAdd(&a.ws->exited, 1u);
        if (old == (unsigned)(a.num_clusters - 1)) {
            a.ws->next = 0;
            a.ws->exited = 0;
            __threadfence();
        }
    }
    cluster.sync();
}

// ---------------------------------------------------------------------------------------
// launcher

namespace {

template <typename T>
size_t verify_smem_bytes(int slice) {
    const size_t slice_bytes = ((size_t)slice * sizeof(T) + 127) & ~(size_t)127;
    const int nvec = (slice + Elem<T>::kEV - 1) / Elem<T>::kEV;
    const int nseg = ((nvec + kNT - 1) / kNT) * kNW;
    return 2 * slice_bytes + sizeof(Shared) + (size_t)nseg * sizeof(unsigned long long);
}

template <typename T, int kC>
int launch_verify_t(VerifyArgs a, cudaStream_t stream) {
    const int EV = Elem<T>::kEV;
    int slice = (a.V + kC - 1) / kC;
    slice = ((slice + EV - 1) / EV) * EV;
    a.slice = slice;
    const size_t smem = verify_smem_bytes<T>(slice);
    if (smem > 227 * 1024) return kUnsupported;
    auto kern = verify_kernel<T, kC>;
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return kLaunchFailed;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kC;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kNT, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // persistent grid: as many clusters as can be co-resident (cached per device/shape)
    static int cached_dev[16] = {-1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1, -1};
    static size_t cached_smem[16];
    static int cached_n[16];
    static std::mutex mu;
    const int slot = (dev & 7) * 2 + (sizeof(T) == 4 ? 1 : 0);
    int nclus = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (cached_dev[slot] == dev && cached_smem[slot] == smem) {
            nclus = cached_n[slot];
        } else {
            cfg.gridDim = dim3(kC, 1, 1);
            if (cudaOccupancyMaxActiveClusters(&nclus, kern, &cfg) != cudaSuccess || nclus <= 0)
                return kLaunchFailed;
            cached_dev[slot] = dev;
            cached_smem[slot] = smem;
            cached_n[slot] = nclus;
        }
    }
    const int tasks = a.B * kT;
    if (nclus > tasks) nclus = tasks;
    if (nclus < 1) nclus = 1;
    a.num_clusters = nclus;
    cfg.gridDim = dim3(nclus * kC, 1, 1);
    if (cudaLaunchKernelEx(&cfg, kern, a) != cudaSuccess) return kLaunchFailed;
    return kOk;
}

template <typename T, int kC>
int launch_probs_t(VerifyArgs a, float* out, cudaStream_t stream) {
    const int EV = Elem<T>::kEV;
    int slice = (a.V + kC - 1) / kC;
    slice = ((slice + EV - 1) / EV) * EV;
    a.slice = slice;
    const size_t smem = verify_smem_bytes<T>(slice);
    if (smem > 227 * 1024) return kUnsupported;
    auto kern = probs_kernel<T, kC>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return kLaunchFailed;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kC;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kNT, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(kC, 1, 1);
    int nclus = 0;
    if (cudaOccupancyMaxActiveClusters(&nclus, kern, &cfg) != cudaSuccess || nclus <= 0)
        return kLaunchFailed;
    if ((long long)nclus > a.tgt_rows) nclus = (int)a.tgt_rows;
    if (nclus < 1) nclus = 1;
    a.num_clusters = nclus;
    cfg.gridDim = dim3(nclus * kC, 1, 1);
    if (cudaLaunchKernelEx(&cfg, kern, a, out) != cudaSuccess) return kLaunchFailed;
    return kOk;
}

}  // namespace

int launch_probs_cluster(const VerifyArgs& a, int dtype, float* out, cudaStream_t stream) {
    if (dtype == 0) return launch_probs_t<__nv_bfloat16, 8>(a, out, stream);
    if (dtype == 1) return launch_probs_t<float, 8>(a, out, stream);
    return kBadDtype;
}

int launch_verify(const VerifyArgs& a, int dtype, cudaStream_t stream) {
    if (dtype == 0) return launch_verify_t<__nv_bfloat16, 8>(a, stream);
    if (dtype == 1) return launch_verify_t<float, 8>(a, stream);
    return kBadDtype;
}

}  // namespace dsv
