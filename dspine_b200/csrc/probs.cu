// probs.cu -- capped chain rejection from dense probabilities (sm_100a).
//
// Replaces sampling/rejection.py:12-153 (_sample_capped_chain / sample_capped_chain_from_probs):
// target p [B,16,V] and draft q [B,15,V] fp32, one CTA of 1024 threads per request.
//   1. warp 0: lane s tests draft s+1 (q in (0,1] and u_s * q < p); the first rejection is the
//      lowest set bit of a ballot, so the acceptance length needs no loop
//   2. the bonus row (residual max(p - clamp01(q), 0), or p after a fully accepted block or a
//      zero residual mass) is read once with coalesced loads; every 1024-element tile's exact
//      2^-40 fixed-point mass goes to shared memory
//   3. threshold floor(u * M) exactly; the crossing tile is found from the tile prefix sums and
//      only that tile is scanned element by element (block scan) for the first index whose
//      running mass exceeds the threshold (V-1 when none, as the reference's default)
#include <cuda_runtime.h>
#include <stdint.h>

#include "dsv_common.cuh"
#include "dsv_kernels.h"

namespace dsv {
namespace pr {

constexpr int kT = 16;
constexpr int kThreads = 1024;
constexpr int kMaxTiles = 1024;  // V <= 1M
constexpr int kMaxPackedWidth = 64;  // packed target rows (compress_probs capacity)

__device__ __forceinline__ float resid(const float* p, const float* q, int pure, int i) {
    const float pv = p[i];
    if (pure) return pv;
    const float qv = q[i];
    const float qq = (qv >= 0.0f && qv <= 1.0f) ? qv : 0.0f;
    return fmaxf(pv - qq, 0.0f);
}

__global__ void __launch_bounds__(kThreads, 1)
    chain_probs_kernel(int V, const int64_t* __restrict__ cand, const float* __restrict__ target,
                       const float* __restrict__ draft, const int32_t* __restrict__ caps,
                       const float* __restrict__ U, const float* __restrict__ UF,
                       const int32_t* __restrict__ prefix, int32_t* accept, int32_t* commit,
                       int64_t* bonus, int64_t* output, int32_t* new_seq) {
    __shared__ unsigned long long tile_mass[kMaxTiles];
    __shared__ unsigned long long wsum[kThreads / 32];
    __shared__ int s_a, s_tile, s_pure;
    __shared__ long long s_thr, s_base;
    __shared__ unsigned long long s_total;
    __shared__ int s_bonus;
    const int b = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ntiles = (V + kThreads - 1) / kThreads;
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
        if (lane == 0) {
            s_a = m ? __ffs(m) - 1 : cap - 1;
            s_pure = (s_a == cap - 1);
        }
    }
    __syncthreads();
    const int a = s_a;
    const float* prow = target + ((int64_t)b * kT + a) * V;
    const float* qrow = draft + ((int64_t)b * (kT - 1) + (a < kT - 1 ? a : 0)) * V;
    const float u = UF[b];
    int pure = s_pure;
    int64_t bo = V - 1;
    for (int attempt = 0; attempt < 2; ++attempt) {
        for (int t = tid; t < ntiles; t += kThreads) tile_mass[t] = 0;
        __syncthreads();
        // tile masses (coalesced: element t * 1024 + tid)
        for (int t = 0; t < ntiles; ++t) {
            const int i = t * kThreads + tid;
            uint64_t f = i < V ? fixv(resid(prow, qrow, pure, i)) : 0;
            f = warp_sum_u64(f);
            if (lane == 0 && f) atomicAdd(&tile_mass[t], (unsigned long long)f);
        }
        __syncthreads();
        // total and crossing tile: warp 0 scans the tile masses in order
        if (warp == 0) {
            unsigned long long run = 0;
            for (int t0 = 0; t0 < ntiles; t0 += 32) {
                const int t = t0 + lane;
                uint64_t v = t < ntiles ? tile_mass[t] : 0;
                v = warp_incl_u64(v);
                if (t < ntiles) tile_mass[t] = run + v;  // inclusive prefix
                run += __shfl_sync(0xffffffffu, v, 31);
            }
            if (lane == 0) {
                const long long thr = scale_floor(u, run);
                s_thr = thr;
                int tile = -1;
                s_bonus = (int)(V - 1);
                if (thr == -1) {
                    s_bonus = 0;  // u < 0: the first running sum already exceeds it
                } else if (thr != -2 && run != 0) {
                    // first tile whose inclusive prefix exceeds thr
                    int lo = 0, hi = ntiles - 1;
                    while (lo < hi) {
                        const int mid = (lo + hi) >> 1;
                        if ((long long)tile_mass[mid] > thr) hi = mid;
                        else lo = mid + 1;
                    }
                    tile = ((long long)tile_mass[lo] > thr) ? lo : -1;
                }
                s_tile = tile;
                s_base = tile > 0 ? (long long)tile_mass[tile - 1] : 0;
                s_total = run;
            }
        }
        __syncthreads();
        const unsigned long long total = s_total;
        if (!pure && total == 0) {  // zero residual: draw from p
            pure = 1;
            __syncthreads();
            continue;
        }
        const int tile = s_tile;
        if (tile >= 0) {
            // block inclusive scan of the crossing tile
            const int i = tile * kThreads + tid;
            uint64_t f = i < V ? fixv(resid(prow, qrow, pure, i)) : 0;
            uint64_t incl = warp_incl_u64(f);
            if (lane == 31) wsum[warp] = incl;
            __syncthreads();
            if (warp == 0) {
                uint64_t w = wsum[lane];
                uint64_t wi = warp_incl_u64(w);
                wsum[lane] = wi - w;  // exclusive
            }
            __syncthreads();
            const long long run = s_base + (long long)(wsum[warp] + incl);
            const long long prev = run - (long long)f;
            if (i < V && run > s_thr && prev <= s_thr) s_bonus = i;  // unique crossing element
            __syncthreads();
        }
        bo = s_bonus;
        break;
    }
    if (tid < kT) {
        const int64_t v = tid < a ? cand[(int64_t)b * kT + tid + 1] : (tid == a ? bo : 0);
        output[(int64_t)b * kT + tid] = v;
    }
    if (tid == 0) {
        accept[b] = a;
        commit[b] = a + 1;
        bonus[b] = bo;
        new_seq[b] = prefix[b] + a + 1;
    }
}

// ---- sparse q: sampling/sparse/accept.py:94-543 (_accept_sparse, accept_sparse) --------------

struct DrawSmem {
    unsigned long long tile_mass[kMaxTiles];
    unsigned long long wsum[kThreads / 32];
    long long thr, base;
    unsigned long long total;
    int tile, bonus;
};

// First index whose running exact fixed-point mass of w(i) (i in [0, V)) exceeds
// floor(u * M); V - 1 when none (also for u >= 1), 0 for u < 0.  Reports M.  All threads.
template <typename W>
__device__ int tile_draw(int V, float u, W w, DrawSmem* s, unsigned long long* mass_out) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ntiles = (V + kThreads - 1) / kThreads;
    for (int t = tid; t < kMaxTiles; t += kThreads) s->tile_mass[t] = 0;
    __syncthreads();
    for (int t = 0; t < ntiles; ++t) {
        const int i = t * kThreads + tid;
        uint64_t f = i < V ? fixv(w(i)) : 0;
        f = warp_sum_u64(f);
        if (lane == 0 && f) atomicAdd(&s->tile_mass[t], (unsigned long long)f);
    }
    __syncthreads();
    if (warp == 0) {
        unsigned long long run = 0;
        for (int t0 = 0; t0 < ntiles; t0 += 32) {
            const int t = t0 + lane;
            uint64_t v = t < ntiles ? s->tile_mass[t] : 0;
            v = warp_incl_u64(v);
            if (t < ntiles) s->tile_mass[t] = run + v;
            run += __shfl_sync(0xffffffffu, v, 31);
        }
        if (lane == 0) {
            const long long thr = scale_floor(u, run);
            int tile = -1, bo = V - 1;
            if (thr == -1) {
                bo = 0;
            } else if (thr != -2 && run != 0) {
                int lo = 0, hi = ntiles - 1;
                while (lo < hi) {
                    const int mid = (lo + hi) >> 1;
                    if ((long long)s->tile_mass[mid] > thr) hi = mid;
                    else lo = mid + 1;
                }
                tile = ((long long)s->tile_mass[lo] > thr) ? lo : -1;
            }
            s->thr = thr;
            s->tile = tile;
            s->bonus = bo;
            s->base = tile > 0 ? (long long)s->tile_mass[tile - 1] : 0;
            s->total = run;
        }
    }
    __syncthreads();
    *mass_out = s->total;
    const int tile = s->tile;
    if (tile >= 0) {
        const int i = tile * kThreads + tid;
        const uint64_t f = i < V ? fixv(w(i)) : 0;
        const uint64_t incl = warp_incl_u64(f);
        if (lane == 31) s->wsum[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            const uint64_t x = s->wsum[lane];
            s->wsum[lane] = warp_incl_u64(x) - x;
        }
        __syncthreads();
        const long long run = s->base + (long long)(s->wsum[warp] + incl);
        const long long prev = run - (long long)f;
        if (i < V && run > s->thr && prev <= s->thr) s->bonus = i;
    }
    __syncthreads();
    const int bo = s->bonus;
    __syncthreads();
    return bo;
}

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

__global__ void __launch_bounds__(kThreads, 1) sparse_accept_kernel(SparseAcceptArgs a) {
    __shared__ DrawSmem ds;
    __shared__ int64_t sq_id[16];
    __shared__ float sq_v[16];
    __shared__ int s_a;
    const int b = blockIdx.x;
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
        if (lane == 0) s_a = m ? __ffs(m) - 1 : cap - 1;
    }
    __syncthreads();
    const int acc = s_a;
    const bool pure0 = acc == cap - 1;
    const long long row = base + acc;
    const long long qi = (long long)b * (kT - 1) + (acc < kT - 1 ? acc : 0);
    const bool dense = packed ? (a.overflow[row] != 0) : true;
    const float uf = a.uf[b];
    long long bo = V - 1;
    if (packed && !dense) {
        // packed target row: its ids in ascending order (unused slots rank as V, the
        // reference's padding), residual against q, exact CDF (accept.py:186-204)
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
            ds.bonus = (int)bo;
        }
        __syncthreads();
        bo = ds.bonus;
    } else {
        // dense target row (or the dense fallback of an overflowed packed row)
        if (tid < 16) {
            sq_id[tid] = a.q_ids[qi * 16 + tid];
            sq_v[tid] = a.q_vals[qi * 16 + tid];
        }
        __syncthreads();
        const float* prow = a.dense ? a.dense + row * V : nullptr;
        const float den = raw ? a.denom[row] : 1.0f;
        bool pure = pure0;
        auto w = [&](int i) -> float {
            float p = prow ? prow[i] : 0.0f;
            if (raw) p = __fdiv_rn(p, den);
            if (pure) return p;
            return fmaxf(__fsub_rn(p, q_sparse(sq_id, sq_v, i, true)), 0.0f);
        };
        unsigned long long M = 0;
        int draw = tile_draw(V, uf, w, &ds, &M);
        if (!pure && M == 0) {  // zero residual: draw from p
            pure = true;
            draw = tile_draw(V, uf, w, &ds, &M);
        }
        bo = draw;
    }
    if (tid < kT) {
        const int64_t v = tid < acc ? a.cand[(int64_t)b * kT + tid + 1] : (tid == acc ? bo : 0);
        a.output[(int64_t)b * kT + tid] = v;
    }
    if (tid == 0) {
        a.accept[b] = acc;
        a.commit[b] = acc + 1;
        a.bonus[b] = bo;
        a.new_seq[b] = a.prefix[b] + acc + 1;
    }
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

int chain_probs_max_vocab() { return pr::kMaxTiles * pr::kThreads; }

int launch_sparse_accept(const SparseAcceptArgs& a, cudaStream_t st) {
    pr::sparse_accept_kernel<<<a.B, pr::kThreads, 0, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

int launch_compress(const float* p, long long rows, int V, int capacity, int32_t* ids, float* vals,
                    int32_t* lens, int32_t* ovf, cudaStream_t st) {
    pr::compress_kernel<<<(unsigned)rows, pr::kCT, 0, st>>>(p, V, capacity, ids, vals, lens, ovf);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

int launch_chain_probs(const ChainProbsArgs& c, cudaStream_t st) {
    pr::chain_probs_kernel<<<c.B, pr::kThreads, 0, st>>>(c.V, c.cand, c.target, c.draft, c.caps, c.u,
                                                        c.uf, c.prefix, c.accept, c.commit, c.bonus,
                                                        c.output, c.new_seq);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

}  // namespace dsv
