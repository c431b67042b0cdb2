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

}  // namespace pr

int chain_probs_max_vocab() { return pr::kMaxTiles * pr::kThreads; }

int launch_chain_probs(const ChainProbsArgs& c, cudaStream_t st) {
    pr::chain_probs_kernel<<<c.B, pr::kThreads, 0, st>>>(c.V, c.cand, c.target, c.draft, c.caps, c.u,
                                                        c.uf, c.prefix, c.accept, c.commit, c.bonus,
                                                        c.output, c.new_seq);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

}  // namespace dsv
