// probs.cu -- capped chain rejection from materialised probabilities (sm_100a).
//
// chain_probs_kernel replaces sampling/rejection.py:12-153 (_sample_capped_chain /
// sample_capped_chain_from_probs): target p [B,16,V] and draft q [B,15,V] fp32.
// sparse_accept_kernel replaces sampling/sparse/accept.py:94-543 (accept_sparse, _accept_sparse,
// _dense_bonus, _packed_bonus): dense or packed target rows, 16-entry sparse draft rows.
// One request is one thread-block cluster of kCl CTAs:
//   1. every CTA: warp 0 lane s tests draft s+1 (q in (0,1] and u_s * q < p); the first
//      rejection is the lowest set bit of a ballot.  Every CTA of the cluster computes the same
//      acceptance length from the same inputs, so nothing is exchanged for it.
//   2. the bonus row (residual max(p - clamp01(q), 0), or p after a fully accepted block or a
//      zero residual mass) is read once: CTA r streams segment r (consecutive 1024-element
//      tiles, 16-byte loads, four tiles in flight per thread) and keeps the exact 2^-40
//      fixed-point mass of every 128-element warp tile in shared memory.  With sparse q the
//      stream sums p alone and the residual replaces p at the (at most 16) draft tokens
//      afterwards, so no element pays for the 16-entry lookup.
//   3. the segment totals cross the cluster through distributed shared memory; every CTA forms
//      M and floor(u * M) exactly, and only the CTA whose segment holds the crossing finds it:
//      the crossing warp tile from its warp-tile prefix, then the element by one warp scan (the
//      first index whose running mass exceeds the threshold; V-1 when none, as the reference's
//      default).  That CTA writes the request's outputs.
#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "dsv_common.cuh"
#include "dsv_kernels.h"

namespace dsv {
namespace pr {

namespace cg = cooperative_groups;

constexpr int kT = 16;
constexpr int kCl = 8;                 // CTAs per request (one cluster)
constexpr int kDT = 256;               // threads per CTA
constexpr int kDW = kDT / 32;          // warps per CTA
constexpr int kTile = kDT * 4;         // elements per tile: one float4 per thread
constexpr int kMaxVocab = 1 << 20;
constexpr int kMaxSegTiles = (kMaxVocab / kTile + kCl - 1) / kCl;
constexpr int kMaxPackedWidth = 64;    // packed target rows (compress_probs capacity)

struct DrawShared {
    unsigned long long wt[kMaxSegTiles * kDW];  // warp-tile masses of this CTA's segment
    unsigned long long seg;                     // segment total, read by the cluster
    unsigned long long segs[kCl];               // every segment's total
    int64_t q_id[16];                           // the sparse draft row
    float q_v[16];
    long long bonus;
    int acc;
};

// tiles [t0, t1) of CTA `rank`: consecutive, as even as whole tiles allow
__device__ __forceinline__ void segment(int V, int rank, int& t0, int& t1) {
    const int ntiles = (V + kTile - 1) / kTile;
    const int per = (ntiles + kCl - 1) / kCl;
    t0 = min(rank * per, ntiles);
    t1 = min(t0 + per, ntiles);
}

// 4 consecutive elements from i (i a multiple of 4); 0 at and past V.  vec: 16-byte loads (the
// row is 16-byte aligned and V a multiple of 4, so i < V means all four are in the row).
__device__ __forceinline__ float4 load4(const float* x, int i, int V, bool vec) {
    if (x == nullptr || i >= V) return make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (vec) return __ldcs(reinterpret_cast<const float4*>(x + i));
    float4 r;
    r.x = x[i];
    r.y = i + 1 < V ? x[i + 1] : 0.0f;
    r.z = i + 2 < V ? x[i + 2] : 0.0f;
    r.w = i + 3 < V ? x[i + 3] : 0.0f;
    return r;
}

__device__ __forceinline__ float resid1(float pv, float qv) {
    const float qq = (qv >= 0.0f && qv <= 1.0f) ? qv : 0.0f;
    return fmaxf(pv - qq, 0.0f);
}

// Residual of dense rows (chain_probs): max(p - clamp01(q), 0), or p (pure).
struct DenseResid {
    const float* p;
    const float* q;
    bool pure, vec;
    static constexpr int kInFlight = 4;  // two rows: eight loads
    struct Raw {
        float4 p, q;
    };
    __device__ __forceinline__ Raw load(int i, int V) const {
        Raw r;
        r.p = load4(p, i, V, vec);
        r.q = pure ? make_float4(0.0f, 0.0f, 0.0f, 0.0f) : load4(q, i, V, vec);
        return r;
    }
    __device__ __forceinline__ uint64_t mass(const Raw& r) const {
        if (pure) return fixv(r.p.x) + fixv(r.p.y) + fixv(r.p.z) + fixv(r.p.w);
        return fixv(resid1(r.p.x, r.q.x)) + fixv(resid1(r.p.y, r.q.y)) +
               fixv(resid1(r.p.z, r.q.z)) + fixv(resid1(r.p.w, r.q.w));
    }
    __device__ __forceinline__ float at(int i) const { return pure ? p[i] : resid1(p[i], q[i]); }
};

// The target probability of a dense row (accept_sparse): p, or p / denominator (IEEE division,
// the reference's raw fallback); a missing row is all zero.
struct DenseP {
    const float* p;
    float den;
    bool raw, vec;
    static constexpr int kInFlight = 4;  // eight was slower (33 vs 29 us on 64 requests)
    struct Raw {
        float4 p;
    };
    __device__ __forceinline__ float val(float x) const { return raw ? __fdiv_rn(x, den) : x; }
    __device__ __forceinline__ Raw load(int i, int V) const { return Raw{load4(p, i, V, vec)}; }
    __device__ __forceinline__ uint64_t mass(const Raw& r) const {
        return fixv(val(r.p.x)) + fixv(val(r.p.y)) + fixv(val(r.p.z)) + fixv(val(r.p.w));
    }
    __device__ __forceinline__ float at(int i) const { return p ? val(p[i]) : 0.0f; }
};

// Warp-tile masses of tiles [t0, t1) into wt: element t*1024 + warp*128 + lane*4 + e, so the
// warp tiles follow index order at wt[(t - t0) * kDW + warp].  W::kInFlight tiles are loaded
// before any is reduced.  All threads.
template <class W>
__device__ __forceinline__ void stream_segment(const W& w, int V, int t0, int t1,
                                               unsigned long long* wt) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int off = warp * 128 + lane * 4;
    constexpr int kInFlight = W::kInFlight;
    for (int t = t0; t < t1; t += kInFlight) {
        typename W::Raw r[kInFlight];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) r[u] = w.load(t + u < t1 ? (t + u) * kTile + off : V, V);
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) {
            const uint64_t s = warp_sum_u64(w.mass(r[u]));
            if (lane == 0 && t + u < t1) wt[(t + u - t0) * kDW + warp] = s;
        }
    }
}

// After wt holds this CTA's warp-tile masses: the segment totals cross the cluster, every CTA
// forms M (into *mass) and floor(u * M), and the CTA whose segment holds the crossing returns the
// bonus index: the first index whose running mass exceeds floor(u * M) (the weight of index i is
// full(i), the same weights wt sums).  V - 1 when nothing crosses (u >= 1 or NaN, M = 0) and 0
// for u < 0, both from rank 0; -1 in every other CTA.  All threads of every CTA of the cluster.
template <class Full>
__device__ long long finish_draw(cg::cluster_group& cluster, DrawShared* sh, int V, int t0, int t1,
                                 float u, const Full& full, unsigned long long* mass) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rank = (int)cluster.block_rank();
    const int n = (t1 - t0) * kDW;
    if (warp == 0) {
        uint64_t s = 0;
        for (int j = lane; j < n; j += 32) s += sh->wt[j];
        s = warp_sum_u64(s);
        if (lane == 0) sh->seg = s;
    }
    cluster.sync();  // every segment total is published
    if (tid < kCl) sh->segs[tid] = *cluster.map_shared_rank(&sh->seg, tid);
    cluster.sync();  // every CTA has read them (seg may be rewritten, the CTA may exit)
    unsigned long long M = 0;
#pragma unroll
    for (int r = 0; r < kCl; ++r) M += sh->segs[r];
    *mass = M;
    const long long thr = scale_floor(u, M);
    if (thr == -1) return rank == 0 ? 0 : -1;
    if (thr == -2 || M == 0) return rank == 0 ? V - 1 : -1;
    // the crossing segment: the first whose inclusive prefix exceeds thr (thr < M: one exists)
    int cs = 0;
    unsigned long long before = 0;
    for (int r = 0; r < kCl; ++r) {
        if ((long long)(before + sh->segs[r]) > thr) {
            cs = r;
            break;
        }
        before += sh->segs[r];
    }
    if (rank != cs) return -1;
    if (warp == 0) {
        long long bo = V - 1;
        unsigned long long run = before;
        int found = -1;
        unsigned long long base = 0;
        for (int j0 = 0; j0 < n; j0 += 32) {
            const int j = j0 + lane;
            const uint64_t v = j < n ? sh->wt[j] : 0;
            const uint64_t incl = warp_incl_u64(v);
            const unsigned m = __ballot_sync(0xffffffffu, (long long)(run + incl) > thr);
            if (m) {
                const int l = __ffs(m) - 1;
                found = j0 + l;
                base = run + __shfl_sync(0xffffffffu, incl - v, l);
                break;
            }
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (found >= 0) {
            const int i0 = (t0 + found / kDW) * kTile + (found % kDW) * 128 + lane * 4;
            uint64_t f[4];
            uint64_t s = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                f[e] = i0 + e < V ? fixv(full(i0 + e)) : 0;
                s += f[e];
            }
            const uint64_t incl = warp_incl_u64(s);
            const unsigned m = __ballot_sync(0xffffffffu, (long long)(base + incl) > thr);
            if (m) {
                const int l = __ffs(m) - 1;
                long long hit = V - 1;
                if (lane == l) {
                    unsigned long long c = base + incl - s;
                    for (int e = 0; e < 4; ++e) {
                        c += f[e];
                        if ((long long)c > thr) {
                            hit = i0 + e;
                            break;
                        }
                    }
                }
                bo = __shfl_sync(0xffffffffu, hit, l);
            }
        }
        if (lane == 0) sh->bonus = bo;
    }
    __syncthreads();
    return sh->bonus;
}

__device__ __forceinline__ void write_outputs(int b, int acc, long long bo, const int64_t* cand,
                                              const int32_t* prefix, int32_t* accept,
                                              int32_t* commit, int64_t* bonus, int64_t* output,
                                              int32_t* new_seq) {
    const int tid = threadIdx.x;
    if (tid < kT) {
        const int64_t v = tid < acc ? cand[(int64_t)b * kT + tid + 1] : (tid == acc ? bo : 0);
        output[(int64_t)b * kT + tid] = v;
    }
    if (tid == 0) {
        accept[b] = acc;
        commit[b] = acc + 1;
        bonus[b] = bo;
        new_seq[b] = prefix[b] + acc + 1;
    }
}

__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kDT)
    chain_probs_kernel(int V, const int64_t* __restrict__ cand, const float* __restrict__ target,
                       const float* __restrict__ draft, const int32_t* __restrict__ caps,
                       const float* __restrict__ U, const float* __restrict__ UF,
                       const int32_t* __restrict__ prefix, int32_t* accept, int32_t* commit,
                       int64_t* bonus, int64_t* output, int32_t* new_seq) {
    __shared__ DrawShared sh;
    cg::cluster_group cluster = cg::this_cluster();
    const int b = blockIdx.x / kCl;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int cap = caps[b];
    cap = cap < 1 ? 1 : (cap > kT ? kT : cap);

    if (warp == 0) {
        bool reject = true;
        if (lane < cap - 1) {
            const int64_t tok = cand[(int64_t)b * kT + lane + 1];
            float p = 0.0f, q = 0.0f;
            if (tok >= 0 && tok < V) {
                p = target[((int64_t)b * kT + lane) * V + tok];
                q = draft[((int64_t)b * (kT - 1) + lane) * V + tok];
            }
            reject = !(q > 0.0f && q <= 1.0f && U[b * (kT - 1) + lane] * q < p);
        }
        const unsigned m = __ballot_sync(0xffffffffu, reject && lane < cap - 1);
        if (lane == 0) sh.acc = m ? __ffs(m) - 1 : cap - 1;
    }
    __syncthreads();
    const int a = sh.acc;
    int t0, t1;
    segment(V, (int)cluster.block_rank(), t0, t1);
    const bool vec = ((reinterpret_cast<uintptr_t>(target) | reinterpret_cast<uintptr_t>(draft)) & 15u) == 0 &&
                     (V & 3) == 0;
    DenseResid w{target + ((int64_t)b * kT + a) * V,
                 draft + ((int64_t)b * (kT - 1) + (a < kT - 1 ? a : 0)) * V, a == cap - 1, vec};
    long long bo = -1;
    for (int attempt = 0; attempt < 2; ++attempt) {
        stream_segment(w, V, t0, t1, sh.wt);
        __syncthreads();
        unsigned long long M = 0;
        bo = finish_draw(cluster, &sh, V, t0, t1, UF[b], [&](int i) { return w.at(i); }, &M);
        if (!w.pure && M == 0) {  // zero residual: draw from p (every CTA sees the same M)
            w.pure = true;
            continue;
        }
        break;
    }
    if (bo < 0) return;
    write_outputs(b, a, bo, cand, prefix, accept, commit, bonus, output, new_seq);
}

// ---- sparse q: sampling/sparse/accept.py:94-543 (_accept_sparse, accept_sparse) --------------

// sum of the q entries of a 16-entry sparse row equal to `token` (clamped to [0,1] when asked),
// in entry order (sampling/sparse/accept.py:275-277)
__device__ __forceinline__ float q_sparse(const int64_t* qid, const float* qv, long long token,
                                          bool clamp) {
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        if (qid[k] != token) continue;
        float v = qv[k];
        if (clamp) v = (v >= 0.0f && v <= 1.0f) ? v : 0.0f;
        s = __fadd_rn(s, v);
    }
    return s;
}

__device__ __forceinline__ float packed_p(const int32_t* ids, const float* vals, int len, int width,
                                          long long token) {
    float s = 0.0f;
    for (int l = 0; l < width && l < len; ++l)
        if ((long long)ids[l] == token) s = __fadd_rn(s, vals[l]);
    return s;
}

// Residual at the draft tokens: wt summed fix(p) over the segment; at each distinct draft token
// inside it the residual's mass replaces p's.  Warp 0 (lanes 0..15: the 16 entries).
__device__ __forceinline__ void sparse_corrections(DrawShared* sh, const DenseP& w, int V, int t0,
                                                   int t1) {
    const int lane = threadIdx.x & 31;
    const long long tok = lane < 16 ? sh->q_id[lane] : -1;
    bool first = lane < 16;
    for (int j = 0; j < 16; ++j)
        if (j < lane && sh->q_id[j] == tok) first = false;
    if (first && tok >= (long long)t0 * kTile && tok < (long long)t1 * kTile && tok < V && tok >= 0) {
        const float p = w.at((int)tok);
        const float r = fmaxf(__fsub_rn(p, q_sparse(sh->q_id, sh->q_v, tok, true)), 0.0f);
        const unsigned long long d = fixv(r) - fixv(p);  // modulo 2^64: the tile total stays >= 0
        atomicAdd(&sh->wt[(tok - (long long)t0 * kTile) >> 7], d);
    }
}

__global__ void __cluster_dims__(kCl, 1, 1) __launch_bounds__(kDT)
    sparse_accept_kernel(SparseAcceptArgs a) {
    __shared__ DrawShared sh;
    cg::cluster_group cluster = cg::this_cluster();
    const int b = blockIdx.x / kCl;
    const int rank = (int)cluster.block_rank();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int V = a.V;
    int cap = a.caps[b];
    cap = cap < 1 ? 1 : (cap > kT ? kT : cap);
    const long long base = a.row_offsets ? a.row_offsets[b] : (long long)b * kT;
    const bool packed = a.p_ids != nullptr;
    const bool raw = a.denom != nullptr;

    if (warp == 0) {
        bool reject = true;
        if (lane < cap - 1) {
            const long long row = base + lane;
            const long long qi = (long long)b * (kT - 1) + lane;
            const long long tok = a.cand[(long long)b * kT + lane + 1];
            const bool dense = packed ? (a.overflow[row] != 0) : true;
            float p = 0.0f;
            if (tok >= 0 && tok < V) {
                if (dense) {
                    p = a.dense ? a.dense[row * V + tok] : 0.0f;
                    if (raw) p = __fdiv_rn(p, a.denom[row]);
                } else {
                    p = packed_p(a.p_ids + row * a.width, a.p_vals + row * a.width, a.p_len[row],
                                 a.width, tok);
                }
            }
            const float q = q_sparse(a.q_ids + qi * 16, a.q_vals + qi * 16, tok, false);
            reject = !(q > 0.0f && q <= 1.0f && __fmul_rn(a.u[qi], q) < p);
        }
        const unsigned m = __ballot_sync(0xffffffffu, reject && lane < cap - 1);
        if (lane == 0) sh.acc = m ? __ffs(m) - 1 : cap - 1;
    }
    __syncthreads();
    const int acc = sh.acc;
    const bool pure0 = acc == cap - 1;
    const long long row = base + acc;
    const long long qi = (long long)b * (kT - 1) + (acc < kT - 1 ? acc : 0);
    const bool dense = packed ? (a.overflow[row] != 0) : true;
    const float uf = a.uf[b];
    long long bo = V - 1;
    if (packed && !dense) {
        // packed target row: its ids in ascending order (unused slots rank as V, the
        // reference's padding), residual against q, exact CDF (accept.py:186-204); rank 0 alone
        if (rank != 0) return;
        if (tid == 0) {
            const int32_t* ids = a.p_ids + row * a.width;
            const float* vals = a.p_vals + row * a.width;
            const int len = a.p_len[row];
            const int n = a.width;
            long long ord[kMaxPackedWidth];
            for (int l = 0; l < n; ++l) ord[l] = l < len ? (long long)ids[l] : (long long)V;
            for (int i = 1; i < n; ++i) {
                const long long x = ord[i];
                int j = i - 1;
                while (j >= 0 && ord[j] > x) {
                    ord[j + 1] = ord[j];
                    --j;
                }
                ord[j + 1] = x;
            }
            const int64_t* qid = a.q_ids + qi * 16;
            const float* qv = a.q_vals + qi * 16;
            bool pure = pure0;
            for (int attempt = 0; attempt < 2; ++attempt) {
                unsigned long long M = 0;
                for (int j = 0; j < n; ++j) {
                    const float p = ord[j] < V ? packed_p(ids, vals, len, n, ord[j]) : 0.0f;
                    const float r = pure ? p : fmaxf(__fsub_rn(p, q_sparse(qid, qv, ord[j], true)), 0.0f);
                    M += fixv(r);
                }
                if (!pure && M == 0) {
                    pure = true;
                    continue;
                }
                const long long thr = scale_floor(uf, M);
                if (thr != -2) {
                    unsigned long long C = 0;
                    for (int j = 0; j < n; ++j) {
                        const float p = ord[j] < V ? packed_p(ids, vals, len, n, ord[j]) : 0.0f;
                        const float r = pure ? p : fmaxf(__fsub_rn(p, q_sparse(qid, qv, ord[j], true)), 0.0f);
                        C += fixv(r);
                        if ((long long)C > thr) {
                            if (ord[j] < V) bo = ord[j];
                            break;
                        }
                    }
                }
                break;
            }
            sh.bonus = bo;
        }
        __syncthreads();
        bo = sh.bonus;
    } else {
        // dense target row (or the dense fallback of an overflowed packed row)
        if (tid < 16) {
            sh.q_id[tid] = a.q_ids[qi * 16 + tid];
            sh.q_v[tid] = a.q_vals[qi * 16 + tid];
        }
        int t0, t1;
        segment(V, rank, t0, t1);
        const float* prow = a.dense ? a.dense + row * V : nullptr;
        const DenseP w{prow, raw ? a.denom[row] : 1.0f, raw,
                       (reinterpret_cast<uintptr_t>(a.dense) & 15u) == 0 && (V & 3) == 0};
        bool pure = pure0;
        auto full = [&](int i) -> float {
            const float p = w.at(i);
            if (pure) return p;
            return fmaxf(__fsub_rn(p, q_sparse(sh.q_id, sh.q_v, i, true)), 0.0f);
        };
        bo = -1;
        for (int attempt = 0; attempt < 2; ++attempt) {
            stream_segment(w, V, t0, t1, sh.wt);
            __syncthreads();
            if (!pure) {
                if (warp == 0) sparse_corrections(&sh, w, V, t0, t1);
                __syncthreads();
            }
            unsigned long long M = 0;
            bo = finish_draw(cluster, &sh, V, t0, t1, uf, full, &M);
            if (!pure && M == 0) {  // zero residual: draw from p
                pure = true;
                continue;
            }
            break;
        }
        if (bo < 0) return;
    }
    write_outputs(b, acc, bo, a.cand, a.prefix, a.accept, a.commit, a.bonus, a.output, a.new_seq);
}

// ---- compress_probs: sampling/sparse/accept.py:422-460 --------------------------------------

// One CTA of kCT threads per row: the first `capacity` positive entries in index order (ids,
// values), their number (clamped) and the overflow flag (more than capacity, or a negative /
// NaN / inf entry).  One streaming pass (16-byte loads, four in flight per thread, no barrier)
// counts the positives and appends up to kCBuf of them to a shared list; a row with at most
// capacity positives sorts that list by index.  Only a row with more positives walks the row
// again, tile by tile in index order, until it has its first `capacity` positives (for a dense
// row these lie at the very start).
constexpr int kCT = 256;
constexpr int kCBuf = 64;

__global__ void __launch_bounds__(kCT)
    compress_kernel(const float* __restrict__ p, int V, int capacity, int32_t* ids, float* vals,
                    int32_t* lens, int32_t* ovf) {
    __shared__ unsigned int s_n, s_bad;
    __shared__ int s_idx[kCBuf];
    __shared__ float s_val[kCBuf];
    __shared__ unsigned int wcnt[kCT / 32];
    const long long r = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* x = p + r * (long long)V;
    if (tid == 0) {
        s_n = 0;
        s_bad = 0;
    }
    __syncthreads();
    bool bad = false;
    unsigned int cnt = 0;  // this thread's positives; the list takes them while it has room
    volatile unsigned int* vn = &s_n;
    auto visit = [&](float v, int i) {
        bad |= (v < 0.0f) || (v != v) || (fabsf(v) == INFINITY);
        if (v > 0.0f) {
            ++cnt;
            if (*vn < (unsigned)kCBuf) {
                const unsigned int slot = atomicAdd(&s_n, 1u);
                if (slot < (unsigned)kCBuf) {
                    s_idx[slot] = i;
                    s_val[slot] = v;
                }
            }
        }
    };
    const bool vec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
    const int nv = vec ? V / 4 : 0;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    int j = tid;
    for (; j + 3 * kCT < nv; j += 4 * kCT) {
        float4 q[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) q[u] = __ldcs(x4 + j + u * kCT);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int i = 4 * (j + u * kCT);
            visit(q[u].x, i);
            visit(q[u].y, i + 1);
            visit(q[u].z, i + 2);
            visit(q[u].w, i + 3);
        }
    }
    for (; j < nv; j += kCT) {
        const float4 q = __ldcs(x4 + j);
        visit(q.x, 4 * j);
        visit(q.y, 4 * j + 1);
        visit(q.z, 4 * j + 2);
        visit(q.w, 4 * j + 3);
    }
    for (int i = 4 * nv + tid; i < V; i += kCT) visit(x[i], i);
    if (bad) atomicOr(&s_bad, 1u);
    // the exact count (the list stops taking entries once full, so s_n may fall short of it)
    cnt = __reduce_add_sync(0xffffffffu, cnt);
    if (lane == 0) wcnt[warp] = cnt;
    __syncthreads();
    unsigned int n = 0;
#pragma unroll
    for (int w = 0; w < kCT / 32; ++w) n += wcnt[w];
    __syncthreads();  // wcnt is reused by the ordered walk
    if (n <= (unsigned)capacity && n <= (unsigned)kCBuf) {
        // every positive is in the list: rank by index
        for (int q = tid; q < capacity; q += kCT) {
            int id = -1;
            float v = 0.0f;
            if (q < (int)n) {
                const int me = s_idx[q];
                int rank = 0;
                for (unsigned int t = 0; t < n; ++t) rank += s_idx[t] < me;
                id = me;
                v = s_val[q];
                ids[r * capacity + rank] = id;
                vals[r * capacity + rank] = v;
            } else {
                ids[r * capacity + q] = -1;
                vals[r * capacity + q] = 0.0f;
            }
        }
    } else {
        // more positives than capacity: the first `capacity` in index order, tile by tile
        for (int q = tid; q < capacity; q += kCT) {
            ids[r * capacity + q] = -1;
            vals[r * capacity + q] = 0.0f;
        }
        __syncthreads();
        unsigned int run = 0;
        for (int t0 = 0; t0 < V && run < (unsigned)capacity; t0 += kCT) {
            const int i = t0 + tid;
            const float v = i < V ? x[i] : 0.0f;
            const bool pos = v > 0.0f;
            const unsigned m = __ballot_sync(0xffffffffu, pos);
            if (lane == 0) wcnt[warp] = __popc(m);
            __syncthreads();
            unsigned before = run, all = 0;
            for (int w = 0; w < kCT / 32; ++w) {
                if (w < warp) before += wcnt[w];
                all += wcnt[w];
            }
            const unsigned slot = before + __popc(m & ((1u << lane) - 1u));
            if (pos && slot < (unsigned)capacity) {
                ids[r * capacity + slot] = i;
                vals[r * capacity + slot] = v;
            }
            __syncthreads();
            run += all;
        }
    }
    if (tid == 0) {
        lens[r] = (int32_t)(n < (unsigned)capacity ? n : (unsigned)capacity);
        ovf[r] = (n > (unsigned)capacity || s_bad) ? 1 : 0;
    }
}

}  // namespace pr

int chain_probs_max_vocab() { return pr::kMaxVocab; }

int launch_sparse_accept(const SparseAcceptArgs& a, cudaStream_t st) {
    pr::sparse_accept_kernel<<<(unsigned)a.B * pr::kCl, pr::kDT, 0, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

int launch_compress(const float* p, long long rows, int V, int capacity, int32_t* ids, float* vals,
                    int32_t* lens, int32_t* ovf, cudaStream_t st) {
    pr::compress_kernel<<<(unsigned)rows, pr::kCT, 0, st>>>(p, V, capacity, ids, vals, lens, ovf);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

int launch_chain_probs(const ChainProbsArgs& c, cudaStream_t st) {
    pr::chain_probs_kernel<<<(unsigned)c.B * pr::kCl, pr::kDT, 0, st>>>(c.V, c.cand, c.target, c.draft, c.caps, c.u,
                                                        c.uf, c.prefix, c.accept, c.commit, c.bonus,
                                                        c.output, c.new_seq);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

}  // namespace dsv
