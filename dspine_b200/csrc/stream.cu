// stream.cu -- streaming verification of bf16 logit rows (sm_100a).
//
// One persistent kernel replaces the reference's build_dspine_target_probs + chain rejection
// (runtime/worker.py:440-508, sampling/rejection.py:12-153) for bf16 logits:
//
//   rows_kernel   one CTA per logit row (a target row, or the draft row of a sampled request);
//                 rows are handed out by a global counter in verify-position order (every
//                 request's position 0, then position 1, ...; the rows of the first positions
//                 as two halves on two CTAs).  The CTA streams its row through a shared-memory
//                 ring filled by cp.async.bulk copies and computes the row's descriptor: max,
//                 exact 2^-40 fixed-point softmax sum, and the kept set of the joint top-k /
//                 top-p filter as (boundary key, tie cut).  The CTA that completes a position
//                 decides that chain step; a chain stops at its first rejected step, so rows
//                 after a known rejection (or of a request whose outcome is known) are dropped
//                 when dequeued or abandoned during their first pass: they cannot change any
//                 output.  Outputs are those of processing every row, bit for bit.
//                   nucleus and keep-all rows: one pass from HBM counts every bf16 key of the
//                           row in a per-key histogram (2^-20 <= |v| < 2^12; the rare values
//                           outside it fall back to the passes below), then S and the kept-set
//                           walk come from the counts (one packed exp per key, not per element)
//                           and the tie cut in index order re-reads the row from L2
//                   other rows: bf16x2 max pass from HBM (greedy rows: and the first index of
//                           the max; they finish here), then the candidate window (top-k <= 256)
//                           or exact count walks from the top, from L2
//   chain tasks   (in the same persistent kernel) up to kCP CTAs per sampled request once its
//                 outcome is known: the residual (p - q)+ draw over target row a and draft row a
//                 of the stopping position a, the five outputs and, for the last request, the
//                 accept-compact.
//
// Arithmetic is the canonical one of dsv_common.cuh (exp2c, fix, scale_floor), so the result
// equals the CPU oracle bit for bit.  Bulk passes clamp y at -64 before the exponent trick:
// every y below -41.5 has fix(exp2(y)) = 0, so the clamp never changes a fix value; exact
// probabilities (chain, residual) use the unclamped exp2c with its y < -125 -> 0 rule.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <mutex>

#include "dsv_common.cuh"
#include "dsv_kernels.h"


namespace dsv {
namespace st {

constexpr int kBins = 24;        // level-1 bins: min(rne(-0.75 y), 23)
constexpr int kSub = 23;         // level-2 bins: rne(-16.5 y) - 22 b1 + 11, clamped to [0, 22]
constexpr int kMaxB = 1024;      // requests per launch handled by this path

enum Cat : int { kGreedy = 0, kKeepAll = 1, kWindow = 2, kBinned = 3 };

constexpr uint32_t kFill = 0xFF80FF80u;  // two bf16 -inf: slots outside the slice
constexpr float kS1 = 0.75f;             // level-1 scale (exact)
constexpr float kS2 = 16.5f;             // level-2 scale = (kSub - 1) * kS1 (exact)
constexpr float kTwo23 = 8388608.0f;

// ---------------------------------------------------------------------------------------
// optional phase profiling (builds with -DDSV_PROFILE only): thread 0 of every CTA adds the
// %globaltimer duration of each phase to u64 counters in the workspace's profiling area:
// counter [cat * 16 + phase], task count at phase 15; the chain kernel at [64 + phase]

#ifdef DSV_PROFILE
constexpr unsigned kTraceCap = 2600;   // task trace entries (5 words each)
constexpr unsigned kTraceCtas = 800;   // per-CTA start / exit entries
static_assert((260 + 5 * kTraceCap + 2 * kTraceCtas) * 8 <= kProfBytes, "trace fits the profiling area");
__device__ __forceinline__ unsigned smid() {
    unsigned r;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
    return r;
}
#define PROF_START() unsigned long long prof_t = globaltimer_ns()
#define PROF_MARK(cat_, ph)                                                              \
    do {                                                                                 \
        if (threadIdx.x == 0) {                                                          \
            const unsigned long long prof_n = globaltimer_ns();                          \
            atomicAdd(a.prof + (cat_) * 16 + (ph), \
                      prof_n - prof_t);                                                  \
            sh->prof_ph[ph] += (uint32_t)(prof_n - prof_t);                              \
            prof_t = prof_n;                                                             \
        }                                                                                \
    } while (0)
#define PROF_END(cat_, ph)                                                                  \
    do {                                                                                    \
        PROF_MARK(cat_, ph);                                                                \
        if (threadIdx.x == 0) atomicAdd(a.prof + (cat_) * 16 + 15, 1ull); \
    } while (0)
#else
#define PROF_START() \
    do {             \
    } while (0)
#define PROF_MARK(cat_, ph) \
    do {                    \
    } while (0)
#define PROF_END(cat_, ph) \
    do {                   \
    } while (0)
#endif

// ---------------------------------------------------------------------------------------
// small helpers

__device__ __forceinline__ uint32_t okey(uint32_t u16) { return Elem<__nv_bfloat16>::key(u16); }
__device__ __forceinline__ uint32_t key_bits(uint32_t k) {
    return (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu);
}
__device__ __forceinline__ float bf(uint32_t u16) { return __uint_as_float(u16 << 16); }

__device__ __forceinline__ uint32_t bf2_ge(uint32_t a, uint32_t b) {
    return __hge2_mask(*reinterpret_cast<const __nv_bfloat162*>(&a),
                       *reinterpret_cast<const __nv_bfloat162*>(&b));
}
__device__ __forceinline__ uint32_t bf2_le(uint32_t a, uint32_t b) {
    return __hle2_mask(*reinterpret_cast<const __nv_bfloat162*>(&a),
                       *reinterpret_cast<const __nv_bfloat162*>(&b));
}
__device__ __forceinline__ uint32_t bf2_eq(uint32_t a, uint32_t b) {
    return __heq2_mask(*reinterpret_cast<const __nv_bfloat162*>(&a),
                       *reinterpret_cast<const __nv_bfloat162*>(&b));
}
__device__ __forceinline__ uint32_t bf2_max(uint32_t a, uint32_t b) {
    __nv_bfloat162 r = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&a),
                               *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}

// 0xFFFF in each 16-bit half of w whose sign bit is set, else 0 (prmt sign replication:
// selector nibbles 0x9 / 0xB take bytes 1 / 3 with their top bit replicated)
__device__ __forceinline__ uint32_t prmt_sign16(uint32_t w) {
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, 0xBB99;" : "=r"(r) : "r"(w));
    return r;
}

// one-count increment of the shared-memory u32 at byte address addr (no return value)
__device__ __forceinline__ void red_shared_inc(uint32_t addr) {
    asm volatile("red.shared.add.u32 [%0], 1;" ::"r"(addr) : "memory");
}

// y of one element, clamped at -64 (bulk passes; see file header)
__device__ __forceinline__ float y_clamped(float l, float m, float c) {
    return fmaxf(__fmul_rn(__fadd_rn(l, -m), c), -64.0f);
}
__device__ __forceinline__ int bin1_of(float yc) {
    const float t = __fmaf_rn(yc, -kS1, kTwo23);
    return (int)min(__float_as_uint(t) - 0x4B000000u, (uint32_t)(kBins - 1));
}
__device__ __forceinline__ int bin2_of(float yc, int b1) {
    const float t = __fmaf_rn(yc, -kS2, kTwo23);
    const int v = (int)(__float_as_uint(t) - 0x4B000000u) - (kSub - 1) * b1 + (kSub - 1) / 2;
    return v < 0 ? 0 : (v > kSub - 1 ? kSub - 1 : v);
}
// fix(exp2(yc)) for yc in [-64, 0]: the split below, scalar form
__device__ __forceinline__ uint64_t fix_of_y(float yc) {
    const float M17 = 12582912.0f + 17.0f;
    const float t = __fadd_rn(yc, M17);
    const float f = __fsub_rn(yc, __fsub_rn(t, M17));
    float p = __uint_as_float(0x3920fddcu);
    p = __fmaf_rn(p, f, __uint_as_float(0x3aaf9f2bu));
    p = __fmaf_rn(p, f, __uint_as_float(0x3c1d96a6u));
    p = __fmaf_rn(p, f, __uint_as_float(0x3d635774u));
    p = __fmaf_rn(p, f, __uint_as_float(0x3e75fdeeu));
    p = __fmaf_rn(p, f, __uint_as_float(0x3f317218u));
    p = __fmaf_rn(p, f, 1.0f);
    const float x = __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));  // e * 2^17
    const float h = __fadd_rn(x, kTwo23);
    const float r = __fsub_rn(x, __fsub_rn(h, kTwo23));
    const float lo = __fmaf_rn(r, kTwo23, 12582912.0f);
    const uint32_t hi = __float_as_uint(h) - 0x4B000000u;
    const int32_t lv = (int32_t)(__float_as_uint(lo) - 0x4B400000u);
    return (uint64_t)((int64_t)hi * 8388608 + lv);
}


// exact probability of element value l under a row descriptor (oracle or_row_prob)
__device__ __forceinline__ float row_prob(const RowDesc& d, float l, uint32_t u16, int i) {
    if (d.flags & kDescGreedy) return i == d.argmax ? 1.0f : 0.0f;
    const uint32_t k = okey(u16);
    const bool kept = (k > d.kstar) || (k == d.kstar && i <= d.tie_cut);
    if (!kept) return 0.0f;
    return __fmul_rn(exp2c(__fmul_rn(__fadd_rn(l, -d.m), d.c)), d.inv_s);
}

// ---------------------------------------------------------------------------------------
// shared memory of the row kernel

struct TaskInfo {
    int b, s, kind, cat, cap;
    long long row;     // row index in its tensor (-1: invalid)
    float T, p, c;
    float mp;          // min-p of the request (0: no floor; always 0 in the joint mode)
    int k;
    int half;          // -1: the whole row; 0 / 1: first / second half of a split row
    int slot;          // split rows: the slot the first half publishes to
};

__device__ __forceinline__ int clamp_cap(int c) { return c < 1 ? 1 : (c > kT ? kT : c); }

__device__ int request_cat(const VerifyArgs& a, int b, float& c_out, int wink) {
    // all three loads issue before any branch (one memory round trip at kernel start)
    const float T = a.temperature[b];
    const int k = a.top_k[b];
    const float p = a.top_p[b];
    const float mp = (a.mode != kModeJoint && a.min_p) ? a.min_p[b] : 0.0f;
    const float c = log2e_over(T);
    c_out = c;
    if (is_greedy(T, k, c)) return kGreedy;
    if (p < 1.0f) return kBinned;             // nucleus (any k): per-key histogram walk
    if (k >= a.V) return mp > 0.0f ? kBinned : kKeepAll;  // min-p alone: counts from the top
    if (k <= wink) return kWindow;            // pure top-k, small k: candidate window
    return kBinned;                           // pure top-k, large k: exact counts from the top
}

// The task table of a launch, identical in every CTA.  Row tasks are ordered by verify
// position first: the position-0 rows of every request, then position 1, and so on, so that
// the rows that decide the chains (a chain stops at its first rejected step) come first and
// the later rows of a request can be dropped once its outcome is known.  Within a position:
// binned target rows, binned draft rows, keep-all/window target rows, their draft rows,
// greedy target rows.  Each class lists its requests by decreasing cap (a stable counting
// sort), so the requests with a row at position s are a prefix of the class list: n(g, s) of
// them (cap > s), and n(g, s + 1) of them have a draft row there.
struct Plan {
    uint32_t* key;   // [48]: per (class, cap) counts, then scatter bases (build only)
    uint16_t* perm;  // [B]: class 0 requests, class 1, class 2, each by decreasing cap
    uint16_t* n;     // [3][17]: requests of class g with cap > s
    uint16_t* pos;   // [17]: first row task of position s; pos[16] = row tasks
    uint16_t* gs;    // [4]: start of class g in perm
    uint8_t* req;    // [B]: cat | cap << 3
    int B;
    __device__ __forceinline__ int cnt(int g, int s) const { return n[g * 17 + s]; }
};
constexpr int kPlanFixed = 48 * 4 + (3 * 17 + 17 + 4) * 2;  // bytes besides the [B] arrays
__host__ __device__ constexpr size_t plan_bytes(int B) {
    return ((size_t)kPlanFixed + (size_t)B * 2 + (size_t)B + 15) & ~(size_t)15;
}
__device__ __forceinline__ Plan plan_at(unsigned char* base, int B) {
    Plan p;
    p.key = reinterpret_cast<uint32_t*>(base);
    p.n = reinterpret_cast<uint16_t*>(base + 48 * 4);
    p.pos = p.n + 3 * 17;
    p.gs = p.pos + 17;
    p.perm = p.gs + 4;
    p.req = reinterpret_cast<uint8_t*>(p.perm + B);
    p.B = B;
    return p;
}

template <typename Sm>
__device__ void build_plan(const VerifyArgs& a, Sm* sh, int wink) {
    const int tid = threadIdx.x, lane = tid & 31;
    const Plan& P = sh->plan;
    for (int i = tid; i < 48; i += blockDim.x) P.key[i] = 0u;
    __syncthreads();
    for (int b = tid; b < a.B; b += blockDim.x) {
        const int cap = clamp_cap(a.caps ? a.caps[b] : a.cap_all);
        float c;
        const int cat = request_cat(a, b, c, wink);
        P.req[b] = (uint8_t)(cat | (cap << 3));
        const int g = cat == kBinned ? 0 : (cat == kGreedy ? 2 : 1);
        atomicAdd(&P.key[g * 16 + cap - 1], 1u);
    }
    __syncthreads();
    if (tid < 32) {
        if (lane < 3) {
            // n(g, s) = requests of class g with cap >= s + 1
            uint32_t acc = 0;
            P.n[lane * 17 + 16] = 0;
            for (int s = 15; s >= 0; --s) {
                acc += P.key[lane * 16 + s];
                P.n[lane * 17 + s] = (uint16_t)acc;
            }
        }
        __syncwarp();
        if (lane == 0) {
            P.gs[0] = 0;
            P.gs[1] = P.n[0];
            P.gs[2] = (uint16_t)(P.n[0] + P.n[17]);
            P.gs[3] = (uint16_t)a.B;
            const int dr = a.drf != nullptr ? 1 : 0;
            uint32_t t = 0;
            for (int s = 0; s < 16; ++s) {
                P.pos[s] = (uint16_t)t;
                t += P.cnt(0, s) + dr * P.cnt(0, s + 1) + P.cnt(1, s) + dr * P.cnt(1, s + 1) + P.cnt(2, s);
            }
            P.pos[16] = (uint16_t)t;
        }
        __syncwarp();
        if (lane < 3) {
            // first slot of each (class, cap) in perm: caps above it come first
            for (int cp = 1; cp <= 16; ++cp) P.key[lane * 16 + cp - 1] = P.gs[lane] + P.n[lane * 17 + cp];
        }
        __syncwarp();
        for (int b0 = 0; b0 < a.B; b0 += 32) {
            const int b = b0 + lane;
            int k = 64 + lane;  // no class: a key of its own
            if (b < a.B) {
                const int cat = (int)(P.req[b] & 7u), cap = (int)(P.req[b] >> 3);
                k = (cat == kBinned ? 0 : (cat == kGreedy ? 2 : 1)) * 16 + cap - 1;
            }
            const unsigned peers = __match_any_sync(0xffffffffu, k);
            const int rank = __popc(peers & ((1u << lane) - 1u));
            const uint32_t base = b < a.B ? P.key[k] : 0u;
            __syncwarp();
            if (b < a.B) {
                P.perm[base + rank] = (uint16_t)b;
                if (rank == 0) P.key[k] = base + (uint32_t)__popc(peers);
            }
            __syncwarp();
        }
    }
    __syncthreads();
}

template <typename Sm>
__device__ int total_tasks(const VerifyArgs& a, const Sm* sh) {
    (void)a;
    return sh->plan.pos[16];
}

template <typename Sm>
__device__ TaskInfo decode_task(const VerifyArgs& a, const Sm* sh, int t) {
    const Plan& P = sh->plan;
    int s = 0;
    while (s < 15 && (int)P.pos[s + 1] <= t) ++s;
    int j = t - (int)P.pos[s];
    const int dr = a.drf != nullptr ? 1 : 0;
    const int seg[5] = {P.cnt(0, s), dr * P.cnt(0, s + 1), P.cnt(1, s), dr * P.cnt(1, s + 1), P.cnt(2, s)};
    int q = 0;
    while (q < 4 && j >= seg[q]) {
        j -= seg[q];
        ++q;
    }
    const int g = q >> 1;
    TaskInfo ti;
    ti.b = P.perm[P.gs[g] + j];
    ti.kind = q & 1;
    ti.s = s;
    ti.cat = (int)(P.req[ti.b] & 7u);
    ti.cap = (int)(P.req[ti.b] >> 3);
    const long long base = ti.kind == 0 ? (a.tgt_row ? a.tgt_row[ti.b] : ti.b * a.row_step)
                                        : a.drf_row[ti.b];
    const long long lim = ti.kind == 0 ? a.tgt_rows : a.drf_rows;
    const long long row = base + ti.s;
    ti.row = (row >= 0 && row < lim) ? row : -1;
    ti.T = a.temperature[ti.b];
    ti.k = a.top_k[ti.b];
    ti.p = a.top_p[ti.b];
    ti.mp = (a.mode != kModeJoint && a.min_p) ? a.min_p[ti.b] : 0.0f;
    ti.c = log2e_over(ti.T);
    ti.half = -1;
    ti.slot = -1;
    return ti;
}

// ---------------------------------------------------------------------------------------
// selection walk over groups in rank order (bins, sub-bins): first group where the count
// reaches k or the mass passes thr

struct Walk {
    int group;                 // -1: not found
    unsigned long long cnt;    // elements ranked before the group
    unsigned long long mass;   // their fixed-point mass
};

// one warp; cnt/mass arrays of n <= 32 groups
__device__ Walk walk_groups(const uint32_t* cnt, const unsigned long long* mass, int n,
                            unsigned long long cnt0, unsigned long long mass0, long long k,
                            long long thr) {
    const int lane = threadIdx.x & 31;
    unsigned long long c = lane < n ? cnt[lane] : 0ull;
    unsigned long long m = lane < n ? mass[lane] : 0ull;
    unsigned long long ci = c, mi = m;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long a = __shfl_up_sync(0xffffffffu, ci, o);
        const unsigned long long bm = __shfl_up_sync(0xffffffffu, mi, o);
        if (lane >= o) { ci += a; mi += bm; }
    }
    const unsigned long long cb = cnt0 + ci - c, mb = mass0 + mi - m;  // before the group
    const bool stop = lane < n && c > 0 &&
                      ((long long)(cb + c) >= k || (long long)(mb + m) > thr);
    const uint32_t bal = __ballot_sync(0xffffffffu, stop);
    Walk wk;
    if (bal == 0) {
        wk.group = -1;
        wk.cnt = cnt0 + __shfl_sync(0xffffffffu, ci, 31);
        wk.mass = mass0 + __shfl_sync(0xffffffffu, mi, 31);
        return wk;
    }
    const int g = __ffs(bal) - 1;
    wk.group = g;
    wk.cnt = __shfl_sync(0xffffffffu, cb, g);
    wk.mass = __shfl_sync(0xffffffffu, mb, g);
    return wk;
}

// write a row descriptor
__device__ __forceinline__ void put_desc(const VerifyArgs& a, const TaskInfo& ti, float m,
                                         uint32_t kstar, int tie, unsigned long long skept,
                                         int argmax, uint32_t flags) {
    RowDesc d;
    d.m = m;
    d.c = ti.c;
    d.inv_s = (flags & kDescGreedy) ? 1.0f : inv_from_fix(skept);
    d.kstar = kstar;
    d.tie_cut = tie;
    d.argmax = argmax;
    d.flags = flags;
    d.pad = 0;
    a.desc[(ti.b * kT + ti.s) * 2 + ti.kind] = d;
}

// exact kept-set resolution from per-key counts: walk keys hi..lo (one warp)
struct KeyStop {
    int found;
    uint32_t key;
    unsigned long long cnt;    // before the key
    unsigned long long mass;   // before the key
    uint32_t count;            // elements with this key
    unsigned long long F;      // fix value of one element with this key
};

// composite bin index of a key (level 1 and level 2); over keys of values in [-inf, m] it is
// non-increasing in the key (y is non-decreasing in the value and both bins round -0.75 y)
__device__ __forceinline__ int composite_bin(uint32_t key, float m, float c) {
    const float yc = y_clamped(bf(key_bits(key)), m, c);
    const int b1 = bin1_of(yc);
    return b1 * kSub + bin2_of(yc, b1);
}

// largest key in [kmin, kmax] whose composite bin is >= target, given bin(kmin) >= target (one
// warp, 32 probes per step; bins are non-increasing in the key, so the probes that pass form a
// prefix)
__device__ __forceinline__ int level_bin(uint32_t key, float m, float c, int lvl) {
    return lvl == 1 ? bin1_of(y_clamped(bf(key_bits(key)), m, c)) : composite_bin(key, m, c);
}

__device__ uint32_t largest_key_ge(int target, uint32_t kmin, uint32_t kmax, float m, float c,
                                   int lvl) {
    const int lane = threadIdx.x & 31;
    uint32_t lo = kmin, hi = kmax;  // invariant: bin(lo) >= target, answer in [lo, hi]
    while (lo < hi) {
        const uint32_t step = (hi - lo + 31) / 32;
        const uint32_t probe = lo + (uint32_t)(lane + 1) * step;
        const bool ok = probe <= hi && level_bin(probe, m, c, lvl) >= target;
        const int nt = __popc(__ballot_sync(0xffffffffu, ok));
        const uint32_t nlo = lo + (uint32_t)nt * step;
        const uint32_t nhi = min(hi, lo + (uint32_t)(nt + 1) * step - 1u);
        lo = nlo;
        hi = nhi;
    }
    return lo;
}

// keys in [klo, khi] within [kmin, kmax] (the keys of -inf and of the row max) are exactly
// those whose composite bin equals target (one warp)
__device__ void key_range(int target, uint32_t kmin, uint32_t kmax, float m, float c, int lvl,
                          uint32_t& klo, uint32_t& khi) {
    khi = largest_key_ge(target, kmin, kmax, m, c, lvl);
    // smallest key with bin <= target = 1 + largest key with bin >= target + 1
    if (level_bin(kmin, m, c, lvl) >= target + 1)
        klo = largest_key_ge(target + 1, kmin, kmax, m, c, lvl) + 1u;
    else
        klo = kmin;
}

// =======================================================================================
// Row kernel: ONE CTA per row, no clusters.  Each CTA streams its whole row from global
// memory with 16-byte loads: pass 1 (max; greedy rows finish here) reads HBM, pass 2 (exact
// exp, fixed-point sum and either the candidate window or the level-1 bins) and the few
// selection passes re-read the row from L2.  All selection is CTA-local (no cross-SM
// exchange); two CTAs per SM overlap a memory-bound pass with an ALU-bound one.  Rows are
// handed out by a global counter, most expensive first.

#ifndef DSV_ROWS_THREADS
#define DSV_ROWS_THREADS 256
#endif
#ifndef DSV_ROWS_MIN_CTAS
#define DSV_ROWS_MIN_CTAS 3
#endif
#ifndef DSV_RING_VECS
#define DSV_RING_VECS (2 * DSV_ROWS_THREADS)
#endif
#ifndef DSV_WATCH_PREFETCH
#define DSV_WATCH_PREFETCH 1  // the first pass's drop test reads the step word a chunk early
#endif
#ifndef DSV_SPLIT_POS
#define DSV_SPLIT_POS 3  // verification splits the rows of the first DSV_SPLIT_POS positions
#endif
constexpr int kSplitPos = DSV_SPLIT_POS;
constexpr int kRT = DSV_ROWS_THREADS;  // threads per CTA
constexpr int kRW = kRT / 32;          // warps
constexpr int kRWinK = kRT < 256 ? kRT : 256;  // top-k rows with k <= this select in a window
static_assert(kRT % 32 == 0 && kRWinK <= kRT, "row kernel launch shape");
static_assert(kRT >= 256, "the group walks give every thread one group of 32 bins (256 groups)");
constexpr int kRWinCap = 1024;     // window candidates per row
constexpr int kRKeyCap = 2048;     // keys per chunk of an exact count walk (count_walk)
constexpr int kHCap = 8192;        // per-key histogram bins (32 KB)
// one-pass histogram: fine bins for 2^-20 <= |v| < 2^12 (4096 keys per sign), the band
// |v| < 2^-20 listed element by element (at most kBandCap), -inf ignored, anything else
// (|v| >= 2^12, +inf, NaN) falls back to the max pass + adaptive histogram
constexpr uint32_t kFB = 0xB580u;     // key of +2^-20
constexpr uint32_t kFTop = 0xC57Fu;   // key of the largest bf16 below +2^12
constexpr uint32_t kFNB = 0x4A7Fu;    // key of -2^-20
constexpr uint32_t kFNLow = 0x3A80u;  // key of the smallest bf16 above -2^12
constexpr uint32_t kFPos = kFTop - kFB + 1u;  // 4096
constexpr uint32_t kNInfRaw = 0x007Fu;        // key of -inf
constexpr int kBandCap = 512;
static_assert(kFPos == 4096u && kFNB - kFNLow + 1u == 4096u && 2 * kFPos == (uint32_t)kHCap,
              "fixed histogram geometry");
#ifndef DSV_RING_SLOTS
#define DSV_RING_SLOTS 3
#endif
constexpr int kRingS = DSV_RING_SLOTS;     // streaming ring: slots
constexpr int kRingCW = DSV_RING_VECS;     // vectors (16 B) per slot (8 KB at 256 threads)
static_assert(kRingCW % kRT == 0 && kRingCW / kRT <= 2, "ring slot: one or two vectors a thread");
constexpr int kRedN = 8 * kRW > 32 ? 8 * kRW : 32;  // per-warp reduction slots (tie scan: per vector)
#ifndef DSV_BIG_VECS
#define DSV_BIG_VECS (3 * DSV_ROWS_THREADS)
#endif
constexpr int kBigCW = DSV_BIG_VECS;  // vectors per slot of the big ring
constexpr int kBigS = (kHCap * 4 + kRingS * kRingCW * 16) / (kBigCW * 16);  // big-ring slots
static_assert(kBigCW % kRT == 0 && kBigS >= 2, "big ring: whole vectors a thread, two slots");
static_assert(kBigCW / kRT * kRW <= kRedN, "tie scan: one warp sum per vector of a thread");

struct RSmem {
    // first, so that histogram byte addresses stay below 32 KB (the packed bin arithmetic of
    // the histogram pass adds the base to both 16-bit halves of a word)
    alignas(16) uint32_t hist[kHCap];       // per-key counts / window candidates / count chunks
    alignas(16) uint4 ring[kRingS][kRingCW];  // streaming ring filled by bulk copies
    Plan plan;                     // task table (after this struct in shared memory)
    int q_nchain;                  // task sources: chain tasks of the launch
    int q_sel_empty;               //               row queue exhausted
    int q_kind, q_b;               //               this task's kind and chain request
#ifdef DSV_PROFILE
    uint32_t prof_ph[16];          // profiling builds: phase durations of the current task
#endif
    int task;
    int first_min;
    int fin_claim;                 // row_finish: 1 + accepted length of a claimed request
    int exit_last;                 // this CTA is the last out of the launch
    int watch_b, watch_s;          // the row's request and position while its first pass may
                                   // be abandoned (watch_s < 0: not watched)
    int late_b, late_s;            // the same for the tie cut (late_s < 0: not watched)
    int abort_row;                 // the first pass was abandoned: the row cannot change an outcome
    int stream_end;                // chunks of the current stream that were issued
    uint32_t hbm_vecs;             // 16-byte vectors the row's first pass read from memory
    uint32_t nlist;
    uint32_t red32[kRedN];
    unsigned long long red64[kRedN];
    int sel[16];
    unsigned long long self64[8];
    uint32_t wc[kRedN];
    unsigned long long wm[kRedN];
    uint32_t nband;                // one-pass histogram: band elements listed
    uint32_t outside;              //                     a value outside the fixed range
    uint16_t band[kBandCap];       //                     the band's raw values
    uint32_t gcnt[kHCap / 32];     // histogram groups of 32 bins: counts
    unsigned long long gmass[kHCap / 32];  //                       masses
    uint32_t zcnt;                 // histogram band: elements
    unsigned long long zmass;      //                 exact mass
    alignas(8) uint64_t ring_bar[kRingS];
    uint32_t ring_cnt;                      // chunks consumed so far (slot, phase)
    // passes that need no histogram (max pass, tie cut) stream through the big ring: the
    // histogram and the ring together, kBigS slots of kBigCW vectors, own barriers
    alignas(8) uint64_t big_bar[kBigS];
    uint32_t big_cnt;
};
static_assert(offsetof(RSmem, ring) == offsetof(RSmem, hist) + sizeof(uint32_t) * kHCap,
              "the big ring spans the histogram and the ring");

// DSV_ROWS_MIN_CTAS CTAs per SM: each (this + 1 KB reserved) within the SM's 228 KB
static_assert(DSV_ROWS_MIN_CTAS * (sizeof(RSmem) + plan_bytes(64) + 1024) <= 228 * 1024,
              "row kernel shared memory (batches up to 64 at the intended occupancy)");
static_assert(2 * kRWinCap * 4 <= kHCap * 4 && kRWinCap * 8 <= kRingS * kRingCW * 16,
              "window candidates fit the histogram, the ranked list the ring");

// Per-request progress of a verification launch, two words of the workspace (zeroed by the
// last CTA out of each launch):
//   racc[2 b]      rows done: bit s = target row s, bit 16 + s = draft row s
//   racc[2 b + 1]  chain steps: bit s (s < 15) = step s accepted, bit 16 + s = step s rejected,
//                  bit 15 = the last target row (cap - 1) is done, bit 31 = outcome claimed
constexpr uint32_t kStepLast = 1u << 15;
constexpr uint32_t kClaimed = 1u << 31;

// accepted length of a request from its step word, or -1 while it is not known: the first
// rejected step r once steps 0..r-1 are all accepted, or cap - 1 once every step is accepted
// and the last target row is done
__device__ __forceinline__ int outcome_of(uint32_t w, int cap) {
    const uint32_t rej = (w >> 16) & 0x7FFFu, ok = w & 0x7FFFu;
    if (rej) {
        const int r = __ffs(rej) - 1;
        const uint32_t m = (1u << r) - 1u;
        return (ok & m) == m ? r : -1;
    }
    const uint32_t m = (1u << (cap - 1)) - 1u;
    return ((ok & m) == m && (w & kStepLast)) ? cap - 1 : -1;
}

// Whether row (b, s) can still change the outcome: not once the outcome is claimed, nor when
// a step before s is known to be rejected (the chain stops there; rows after it are never
// read).  Both only become true over time, so a row found unneeded stays unneeded.
__device__ __forceinline__ bool needed_by_word(uint32_t w, int s) {
    if (w & kClaimed) return false;
    const uint32_t rej = (w >> 16) & 0x7FFFu;
    return rej == 0u || s <= __ffs(rej) - 1;
}
__device__ __forceinline__ bool row_needed(const VerifyArgs& a, int b, int s) {
    if (a.cand == nullptr) return true;
    return needed_by_word(*(volatile const uint32_t*)&a.racc[2 * b + 1], s);
}

struct RowGeo {
    const uint16_t* rowp;
    int off, nv;   // element e is half (e + off) % 8 of vector (e + off) / 8
};

__device__ __forceinline__ RowGeo row_geo(const VerifyArgs& a, const TaskInfo& ti) {
    RowGeo g;
    const uint16_t* base = reinterpret_cast<const uint16_t*>(ti.kind == 0 ? a.tgt : a.drf);
    g.rowp = base + (ti.row < 0 ? 0 : ti.row) * a.stride;
    g.off = (int)((reinterpret_cast<uintptr_t>(g.rowp) & 15u) >> 1);
    g.nv = ti.row < 0 ? 0 : (a.V + g.off + 7) >> 3;
    return g;
}

// vector v of the row with the halves outside [0, V) set to -inf
__device__ __forceinline__ uint4 row_vec(const RowGeo& g, int V, const uint4* src, int v, uint4 x) {
    if (v == 0 || v == g.nv - 1) {
        uint32_t* u = reinterpret_cast<uint32_t*>(&x);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
            const int e = 8 * v + h - g.off;
            if (e < 0 || e >= V) {
                const uint32_t msk = (h & 1) ? 0xFFFF0000u : 0x0000FFFFu;
                u[h >> 1] = (u[h >> 1] & ~msk) | (kFill & msk);
            }
        }
    }
    return x;
}

// The slots, barriers and chunk counter of the small ring (kBig = false: kRingS slots after
// the histogram) or of the big ring (kBig = true: kBigS slots over the histogram and the ring;
// only for passes that keep nothing in the histogram).
template <bool kBig>
struct Ring {
    static constexpr int S = kBig ? kBigS : kRingS;
    static constexpr int CW = kBig ? kBigCW : kRingCW;
    uint4* buf;
    uint64_t* bar;
    uint32_t* cnt;
    __device__ __forceinline__ explicit Ring(RSmem* sh)
        : buf(kBig ? reinterpret_cast<uint4*>(sh->hist) : &sh->ring[0][0]),
          bar(kBig ? sh->big_bar : sh->ring_bar),
          cnt(kBig ? &sh->big_cnt : &sh->ring_cnt) {}
    __device__ __forceinline__ uint4* slot(uint32_t i) const { return buf + (size_t)i * CW; }
};

// Stream the row through fn(vector, v) via a ring: thread 0 keeps S chunks of CW
// vectors in flight with bulk copies (one mbarrier per slot, bounded waits); every thread
// handles vectors tid and tid + kRT of each chunk.  All threads must call it.
template <bool kBig = false, typename F>
__device__ __forceinline__ int stream_row(RSmem* sh, const VerifyArgs& a, const RowGeo& g, int V,
                                          F&& fn, int vb = 0, int ve = -1) {
    // vectors [vb, ve) of the row (default: all); fn sees row-global vector indices.  While
    // the row is watched (watch_s >= 0), thread 0 checks every 8 chunks whether it can still
    // change an outcome; if not, no further chunk is issued, the ones in flight are drained
    // unprocessed and abort_row is set.  Returns the vectors read.
    const Ring<kBig> R(sh);
    constexpr int S = Ring<kBig>::S;
    constexpr int CW = Ring<kBig>::CW;
    const int tid = threadIdx.x;
    if (ve < 0) ve = g.nv;
    const char* src = reinterpret_cast<const char*>(g.rowp - g.off) + (size_t)vb * 16;
    const int nvr = ve - vb;
    const int nch = (nvr + CW - 1) / CW;
    const uint32_t base = *R.cnt;  // uniform: read before any thread updates it
    if (tid == 0) sh->stream_end = nch;
#if DSV_WATCH_PREFETCH
    const bool watched = tid == 0 && sh->watch_s >= 0;  // thread 0's own copy
    uint32_t word = 0u;
#endif
    __syncthreads();
    if (tid == 0) {
        for (int c = 0; c < nch && c < S; ++c) {
            const uint32_t slot = (base + c) % S;
            const int nvec = min(CW, nvr - c * CW);
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&R.bar[slot], (uint32_t)nvec * 16u);
            bulk_g2s(R.slot(slot), src + (size_t)c * CW * 16, (uint32_t)nvec * 16u, &R.bar[slot]);
        }
    }
    for (int c = 0; c < nch; ++c) {
        const uint32_t k = base + c;
        const uint32_t slot = k % S;
        if (!mbar_wait_bounded(&R.bar[slot], (k / S) & 1u)) {
            if (tid == 0) atomicOr(&a.ws->err, 1u);
        }
        const int v0 = c * CW;
        const int nvec = min(CW, nvr - v0);
        if (!sh->abort_row) {
#pragma unroll
            for (int u = 0; u < CW / kRT; ++u) {
                const int i = tid + u * kRT;
                if (i < nvec) fn(row_vec(g, V, nullptr, vb + v0 + i, R.slot(slot)[i]), vb + v0 + i);
            }
        }
        __syncthreads();  // the slot is consumed
        // every thread sees the same stream_end here: thread 0 changes it only after this
        // barrier, and to a value the next iteration cannot reach
        if (c + 1 >= sh->stream_end) break;
        if (tid == 0) {
#if DSV_WATCH_PREFETCH
            // the request's step word is loaded one chunk before it is tested, so the test
            // does not wait for the load (it would delay the refill and the next barrier)
            if (watched && (c & 7) == 7 && !sh->abort_row && !needed_by_word(word, sh->watch_s)) {
#else
            if (sh->watch_s >= 0 && !sh->abort_row && (c & 7) == 7 &&
                !row_needed(a, sh->watch_b, sh->watch_s)) {
#endif
                sh->abort_row = 1;
                sh->stream_end = min(nch, c + S);  // chunks c + 1 .. c + S - 1 are in flight
            }
            if (!sh->abort_row && c + S < nch) {
                const int cn = c + S;
                const int nv2 = min(CW, nvr - cn * CW);
                fence_proxy_async_smem();
                mbar_arrive_expect_tx(&R.bar[slot], (uint32_t)nv2 * 16u);
                bulk_g2s(R.slot(slot), src + (size_t)cn * CW * 16, (uint32_t)nv2 * 16u, &R.bar[slot]);
            }
#if DSV_WATCH_PREFETCH
            if (watched && (c & 7) == 6) word = *(volatile const uint32_t*)&a.racc[2 * sh->watch_b + 1];
#endif
        }
    }
    __syncthreads();
    const int issued = sh->stream_end;
    __syncthreads();
    if (tid == 0) *R.cnt = base + (uint32_t)issued;
    __syncthreads();
    return min(nvr, issued * CW);
}

__device__ __forceinline__ unsigned long long rcta_sum_u64(unsigned long long v, RSmem* sh) {
    v = warp_sum_u64(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh->red64[threadIdx.x >> 5] = v;
    __syncthreads();
    unsigned long long s = 0;
#pragma unroll
    for (int i = 0; i < kRW; ++i) s += sh->red64[i];
    return s;
}

// CTA-wide walk over the per-key counts of keys khi, khi-1, ... (n keys, thread t owns a
// contiguous run): the first key where the count reaches k or the mass passes thr
__device__ KeyStop cta_walk_keys(RSmem* sh, const uint32_t* counts, uint32_t khi, int n, float m,
                                 float c, unsigned long long cnt0, unsigned long long mass0,
                                 long long k, long long thr) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int per = (n + kRT - 1) / kRT;
    const int i0 = min(tid * per, n), i1 = min(i0 + per, n);
    unsigned long long cs = 0, ms = 0;
    for (int i = i0; i < i1; ++i) {
        const uint32_t cc = counts[i];
        if (cc) {
            cs += cc;
            ms += (unsigned long long)cc * fix_of_y(y_clamped(bf(key_bits(khi - (uint32_t)i)), m, c));
        }
    }
    // block exclusive scan of (cs, ms)
    unsigned long long ci = cs, mi = ms;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long a = __shfl_up_sync(0xffffffffu, ci, o);
        const unsigned long long b = __shfl_up_sync(0xffffffffu, mi, o);
        if (lane >= o) { ci += a; mi += b; }
    }
    __syncthreads();
    if (lane == 31) {
        sh->wc[wid] = (uint32_t)0;
        sh->red64[wid] = ci;
        sh->wm[wid] = mi;
    }
    if (tid == 0) sh->sel[6] = 0x7fffffff;
    __syncthreads();
    unsigned long long cb = cnt0 + ci - cs, mb = mass0 + mi - ms;
    for (int w = 0; w < wid; ++w) {
        cb += sh->red64[w];
        mb += sh->wm[w];
    }
    // my first stopping key, if any
    for (int i = i0; i < i1; ++i) {
        const uint32_t cc = counts[i];
        if (!cc) continue;
        const unsigned long long F = fix_of_y(y_clamped(bf(key_bits(khi - (uint32_t)i)), m, c));
        if ((long long)(cb + cc) >= k || (long long)(mb + cc * F) > thr) {
            atomicMin(&sh->sel[6], i);
            break;
        }
        cb += cc;
        mb += cc * F;
    }
    __syncthreads();
    KeyStop ks;
    ks.found = sh->sel[6] != 0x7fffffff;
    const int istop = sh->sel[6];
    __syncthreads();
    if (ks.found && istop >= i0 && istop < i1) {
        // the owner of the stopping key recomputes its prefix and publishes the stop
        unsigned long long cb2 = cnt0 + ci - cs, mb2 = mass0 + mi - ms;
        for (int w = 0; w < wid; ++w) {
            cb2 += sh->red64[w];
            mb2 += sh->wm[w];
        }
        for (int i = i0; i < istop; ++i) {
            const uint32_t cc = counts[i];
            if (!cc) continue;
            cb2 += cc;
            mb2 += cc * fix_of_y(y_clamped(bf(key_bits(khi - (uint32_t)i)), m, c));
        }
        sh->self64[4] = cb2;
        sh->self64[5] = mb2;
        sh->self64[6] = fix_of_y(y_clamped(bf(key_bits(khi - (uint32_t)istop)), m, c));
        sh->sel[7] = (int)(khi - (uint32_t)istop);
        sh->sel[8] = (int)counts[istop];
    }
    // totals of the whole range (for a continuation into the next chunk)
    if (tid == 0) {
        unsigned long long ct = cnt0, mt = mass0;
        for (int w = 0; w < kRW; ++w) {
            ct += sh->red64[w];
            mt += sh->wm[w];
        }
        sh->self64[2] = ct;
        sh->self64[3] = mt;
    }
    __syncthreads();
    if (ks.found) {
        ks.key = (uint32_t)sh->sel[7];
        ks.count = (uint32_t)sh->sel[8];
        ks.cnt = sh->self64[4];
        ks.mass = sh->self64[5];
        ks.F = sh->self64[6];
    } else {
        ks.cnt = sh->self64[2];
        ks.mass = sh->self64[3];
    }
    __syncthreads();
    return ks;
}


// index of occurrence number `need` (1-based) of the key in index order, streaming the row
// through the ring; chunks already issued when it is found are drained, none is left in flight.
// kRev streams the row from its end and `need` counts occurrences from the end (the caller
// picks the nearer end: occurrence n of c in index order is occurrence c - n + 1 from the end).
// Returns the index, -1 if not found, or -2 if the watched row was abandoned.
template <bool kRev>
__device__ int tie_scan(RSmem* sh, const VerifyArgs& a, const RowGeo& g, int V, uint32_t key,
                        unsigned long long need_total) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const uint32_t kb = key_bits(key);
    const uint32_t kb2 = kb | (kb << 16);
    const char* src = reinterpret_cast<const char*>(g.rowp - g.off);
    const Ring<true> R(sh);  // the histogram is no longer needed
    constexpr int S = Ring<true>::S;
    constexpr int CW = Ring<true>::CW;
    constexpr int U = CW / kRT;
    const int nch = (g.nv + CW - 1) / CW;
    // the r-th chunk streamed is chunk position r (forward) or nch - 1 - r (from the end)
    auto pos_of = [&](int r) { return kRev ? nch - 1 - r : r; };
    const uint32_t base = *R.cnt;
    __syncthreads();
    if (tid == 0) {
        sh->sel[12] = -1;
        for (int r = 0; r < nch && r < S; ++r) {
            const uint32_t slot = (base + r) % S;
            const int c = pos_of(r);
            const int nvec = min(CW, g.nv - c * CW);
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&R.bar[slot], (uint32_t)nvec * 16u);
            bulk_g2s(R.slot(slot), src + (size_t)c * CW * 16, (uint32_t)nvec * 16u, &R.bar[slot]);
        }
    }
    __syncthreads();
    int issued = nch < S ? nch : S;
    unsigned long long run = 0;
    int found = -1;
    // positions outside the row read as -inf (row_vec), so unless the key is -inf itself a
    // vector's count is the number of equal halves: 16 mask bits each
    const bool packed_count = kb != (kFill & 0xFFFFu);
    auto count_in = [&](uint4 x, int v) -> uint32_t {
        x = row_vec(g, V, nullptr, v, x);
        if (packed_count)
            return (uint32_t)(__popc(bf2_eq(x.x, kb2)) + __popc(bf2_eq(x.y, kb2)) +
                              __popc(bf2_eq(x.z, kb2)) + __popc(bf2_eq(x.w, kb2))) >> 4;
        const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
        uint32_t c = 0;
#pragma unroll
        for (int h = 0; h < 8; ++h) {
            const uint32_t eq = bf2_eq(xs[h >> 1], kb2) & ((h & 1) ? 0xFFFF0000u : 0x0000FFFFu);
            const int e = 8 * v + h - g.off;
            c += (eq && e >= 0 && e < V) ? 1u : 0u;
        }
        return c;
    };
    for (int r = 0; r < issued; ++r) {
        const uint32_t k = base + r;
        const uint32_t slot = k % S;
        if (!mbar_wait_bounded(&R.bar[slot], (k / S) & 1u)) {
            if (tid == 0) atomicOr(&a.ws->err, 1u);
        }
        if (found == -1) {
            const int v0 = pos_of(r) * CW;
            const int nvec = min(CW, g.nv - v0);
            uint32_t cu[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = tid + u * kRT;
                cu[u] = i < nvec ? count_in(R.slot(slot)[i], v0 + i) : 0u;
                const uint32_t ws_ = warp_sum_u32(cu[u]);
                if (lane == 0) sh->red32[u * kRW + wid] = ws_;
            }
            __syncthreads();
            uint32_t tot[U];
            uint32_t all = 0;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                tot[u] = 0;
                for (int w = 0; w < kRW; ++w) tot[u] += sh->red32[u * kRW + w];
                all += tot[u];
            }
            if (run + all >= need_total) {
                // in this chunk, vectors are in index order u-major, then thread, then half;
                // from the end the same order is walked backwards
                uint32_t need = (uint32_t)(need_total - run);
#pragma unroll
                for (int uu = 0; uu < U; ++uu) {
                    const int u = kRev ? U - 1 - uu : uu;
                    if (need == 0u) break;
                    if (need > tot[u]) {
                        need -= tot[u];
                        continue;
                    }
                    const uint32_t incl = warp_incl_u32(cu[u]);
                    uint32_t lo;  // occurrences of this u ahead of the thread in walk order
                    if (!kRev) {
                        uint32_t wpre = 0;
                        for (int w = 0; w < wid; ++w) wpre += sh->red32[u * kRW + w];
                        lo = wpre + incl - cu[u];
                    } else {
                        uint32_t wsuf = 0;
                        for (int w = wid + 1; w < kRW; ++w) wsuf += sh->red32[u * kRW + w];
                        lo = wsuf + (sh->red32[u * kRW + wid] - incl);
                    }
                    if (cu[u] > 0 && lo < need && lo + cu[u] >= need) {
                        uint32_t k2 = need - lo;
                        const int v = v0 + tid + u * kRT;
                        const uint4 x = row_vec(g, V, nullptr, v, R.slot(slot)[tid + u * kRT]);
                        const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
                        int e_found = -1;
#pragma unroll
                        for (int hh = 0; hh < 8; ++hh) {
                            const int h = kRev ? 7 - hh : hh;
                            const uint32_t eq = bf2_eq(xs[h >> 1], kb2) & ((h & 1) ? 0xFFFF0000u : 0x0000FFFFu);
                            const int e = 8 * v + h - g.off;
                            if (e_found < 0 && eq && e >= 0 && e < V && --k2 == 0u) e_found = e;
                        }
                        sh->sel[12] = e_found;
                    }
                    need = 0u;
                }
            }
            run += all;
        }
        // a watched row that can no longer change an outcome is abandoned (checked every 8
        // chunks): -2 stops the issue of further chunks; a cut found in this same chunk may
        // win the race for sel[12], and then the row simply completes
        if (tid == 0 && (r & 7) == 7 && sh->late_s >= 0 && !row_needed(a, sh->late_b, sh->late_s) &&
            sh->sel[12] == -1)
            sh->sel[12] = -2;
        __syncthreads();  // the slot is consumed; sel[12] is visible
        found = sh->sel[12];
        const bool more = found == -1 && issued < nch;
        if (tid == 0 && more) {
            const uint32_t slot2 = (base + issued) % S;
            const int cn = pos_of(issued);
            const int nv2 = min(CW, g.nv - cn * CW);
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&R.bar[slot2], (uint32_t)nv2 * 16u);
            bulk_g2s(R.slot(slot2), src + (size_t)cn * CW * 16, (uint32_t)nv2 * 16u, &R.bar[slot2]);
        }
        if (more) ++issued;
    }
    __syncthreads();
    if (tid == 0) *R.cnt = base + (uint32_t)issued;
    __syncthreads();
    return found;
}

// Exact walk over the keys top, top-1, ..., bottom from counts gathered by streaming the row
// (kRKeyCap keys per pass, from the top): the first key where the count reaches k or the mass
// passes thr, starting from (cnt0, mass0) ranked ahead.  All threads must call it.
__device__ KeyStop count_walk(RSmem* sh, const VerifyArgs& a, const RowGeo& g, int V, uint32_t top,
                              uint32_t bottom, float m, float c, unsigned long long cnt0,
                              unsigned long long mass0, long long k, long long thr) {
    const int tid = threadIdx.x;
    KeyStop ks;
    ks.found = 0;
    ks.cnt = cnt0;
    ks.mass = mass0;
    unsigned long long cum_cnt = cnt0, cum_mass = mass0;
    for (uint32_t t = top; t >= bottom && t <= 0xFFFFu;) {
        const uint32_t bot = (t - bottom + 1u > (uint32_t)kRKeyCap) ? t - kRKeyCap + 1 : bottom;
        const int nk = (int)(t - bot + 1);
        __syncthreads();
        for (int i = tid; i < nk; i += kRT) sh->hist[i] = 0;
        __syncthreads();
        const uint32_t vlo = key_bits(bot), vhi = key_bits(t);
        const uint32_t vlo2 = vlo | (vlo << 16), vhi2 = vhi | (vhi << 16);
        stream_row(sh, a, g, V, [&](const uint4& x, int v) {
            const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t in = bf2_ge(xs[q], vlo2) & bf2_le(xs[q], vhi2);
                if (!in) continue;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int e = 8 * v + 2 * q + h - g.off;
                    if (!(in & (h ? 0xFFFF0000u : 0x0000FFFFu)) || e < 0 || e >= V) continue;
                    const uint32_t kkey = okey(h ? (xs[q] >> 16) : (xs[q] & 0xFFFFu));
                    if (kkey >= bot && kkey <= t) atomicAdd(&sh->hist[t - kkey], 1u);
                }
            }
        });
        __syncthreads();
        ks = cta_walk_keys(sh, sh->hist, t, nk, m, c, cum_cnt, cum_mass, k, thr);
        if (ks.found) break;
        cum_cnt = ks.cnt;
        cum_mass = ks.mass;
        if (bot == bottom) break;
        t = bot - 1;
    }
    return ks;
}

// Elements of the row whose key is >= kf (the min-p floor): one pass through the small ring
// (the histogram stays intact), packed bf16x2 compares.  All threads must call it.
__device__ long long count_ge_key(RSmem* sh, const VerifyArgs& a, const RowGeo& g, int V,
                                  uint32_t kf) {
    const uint32_t fb = key_bits(kf);
    const uint32_t fb2 = fb | (fb << 16);
    uint32_t cnt = 0;
    stream_row(sh, a, g, V, [&](const uint4& x, int) {
        // halves outside the row read as -inf, below every floor
        cnt += (uint32_t)(__popc(bf2_ge(x.x, fb2)) + __popc(bf2_ge(x.y, fb2)) +
                          __popc(bf2_ge(x.z, fb2)) + __popc(bf2_ge(x.w, fb2))) >> 4;
    });
    return (long long)rcta_sum_u64(cnt, sh);
}

// One row task: its descriptor (and, for greedy rows, its packed first argmax).  All threads.
// Split rows: the first half publishes its per-key counts, its maximum key, its band values
// and its out-of-range flag to the row's slot, then a flag; the second half waits for the flag
// (bounded; error bit 7) and adds them to its own.  Both halves are consecutive tasks, so the
// wait is short; the first half never waits.
__device__ void split_publish(RSmem* sh, const VerifyArgs& a, int slot, uint32_t mkey) {
    const int tid = threadIdx.x;
    uint32_t* cnt = reinterpret_cast<uint32_t*>(a.split + (size_t)slot * kSplitSlotBytes);
    uint32_t* meta = cnt + kHCap;
    uint16_t* band = reinterpret_cast<uint16_t*>(meta + 4);
    for (int i = tid; i < kHCap; i += kRT) __stcg(cnt + i, sh->hist[i]);
    const uint32_t nb = sh->nband;
    for (uint32_t i = tid; i < nb && i < (uint32_t)kBandCap; i += kRT) band[i] = sh->band[i];
    if (tid == 0) {
        meta[0] = mkey;
        meta[1] = nb;
        meta[2] = sh->outside;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) atomicExch(&a.split_flag[slot], 1u);
}

__device__ uint32_t split_merge(RSmem* sh, const VerifyArgs& a, int slot, uint32_t mkey) {
    const int tid = threadIdx.x;
    const uint32_t* cnt = reinterpret_cast<const uint32_t*>(a.split + (size_t)slot * kSplitSlotBytes);
    const uint32_t* meta = cnt + kHCap;
    const uint16_t* band = reinterpret_cast<const uint16_t*>(meta + 4);
    if (tid == 0) {
        volatile unsigned* f = a.split_flag + slot;
        if (*f == 0u) {
            const uint64_t t0 = globaltimer_ns();
            while (*f == 0u) {
                if (globaltimer_ns() - t0 > 2000000000ull) {
                    atomicOr(&a.ws->err, 128u);
                    break;
                }
                __nanosleep(128);
            }
        }
        __threadfence();
    }
    __syncthreads();
    if ((reinterpret_cast<uintptr_t>(cnt) & 15u) == 0u) {
        // every load of the slot's counts issued before any is added (16-byte vectors)
        constexpr int kV = kHCap / 4 / kRT;
        static_assert(kHCap % (4 * kRT) == 0, "whole count vectors per thread");
        const uint4* c4 = reinterpret_cast<const uint4*>(cnt);
        uint4* h4 = reinterpret_cast<uint4*>(sh->hist);
        uint4 v[kV];
#pragma unroll
        for (int u = 0; u < kV; ++u) v[u] = __ldcg(c4 + tid + u * kRT);
#pragma unroll
        for (int u = 0; u < kV; ++u) {
            uint4 x = h4[tid + u * kRT];
            x.x += v[u].x;
            x.y += v[u].y;
            x.z += v[u].z;
            x.w += v[u].w;
            h4[tid + u * kRT] = x;
        }
    } else {
        for (int i = tid; i < kHCap; i += kRT) sh->hist[i] += __ldcg(cnt + i);
    }
    const uint32_t mk1 = __ldcg(meta + 0), nb1 = __ldcg(meta + 1), out1 = __ldcg(meta + 2);
    const uint32_t nb0 = sh->nband;
    for (uint32_t i = tid; i < nb1 && nb0 + i < (uint32_t)kBandCap; i += kRT) sh->band[nb0 + i] = band[i];
    __syncthreads();
    if (tid == 0) {
        sh->nband = nb0 + nb1;
        sh->outside |= out1;
        a.split_flag[slot] = 0u;  // for the next launch
    }
    __syncthreads();
    return mk1 > mkey ? mk1 : mkey;
}

// Nucleus and keep-all rows start with the fixed-range histogram (one pass, no max pass) and
// are the ones split in halves; sequential-mode nucleus rows with a top-k take the max pass
__device__ __forceinline__ bool row_onepass(const VerifyArgs& a, const TaskInfo& ti) {
    const bool seq_k = a.mode == kModeSeq && ti.k < a.V && ti.p < 1.0f;
    return ti.cat == kKeepAll || (ti.cat == kBinned && ti.p < 1.0f && !seq_k);
}

__device__ void process_row_body(RSmem* sh, const VerifyArgs& a, const TaskInfo& ti) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int V = a.V;
    PROF_START();
    if (ti.row < 0 && tid == 0) atomicOr(&a.ws->err, 2u);
    const RowGeo g = row_geo(a, ti);
    const bool greedy = ti.cat == kGreedy;

    // Nucleus and keep-all rows start with the fixed-range histogram (one pass, no max
    // pass); the other rows, and rows with values outside that range, start with the max.
    // sequential-mode nucleus rows with a top-k need the top-k's mass before the histogram
    // walk (counts from the top, which reuse the histogram's storage): they take the max pass
    const bool seq_k = a.mode == kModeSeq && ti.k < V && ti.p < 1.0f;
    const bool onepass = row_onepass(a, ti);
    if (ti.half == 0 && !onepass) return;  // only one-pass rows are split: the second half does all
    const int half = onepass ? ti.half : -1;
    uint32_t tkey = 0, mkey = 0;
    bool fixed_hist = false;
    if (onepass) {
        // a split row's halves: vectors [0, nv / 2) and [nv / 2, nv)
        const int hb = half < 0 ? 0 : (half == 0 ? 0 : g.nv / 2);
        const int he = half < 0 ? g.nv : (half == 0 ? g.nv / 2 : g.nv);
        __syncthreads();
        for (int i = tid; i < kHCap; i += kRT) sh->hist[i] = 0u;
        if (tid == 0) {
            sh->nband = 0u;
            sh->outside = 0u;
        }
        __syncthreads();
        uint32_t vmax2 = 0xFF80FF80u;  // running bf16x2 maximum (-inf, -inf)
        // Bins of a word whose two halves are both fine, packed: sgn = 0xFFFF in each negative
        // half, y = bits (negative) or 0xFFFF - bits (positive), bin = y + (sgn & 0x1500) -
        // 0xBA80, i.e. 0x457F - bits for positive v (descending key) and bits - 0xA580 for
        // negative v (4096 + descending key of the negative part).  The histogram's word
        // address / 4 is added to both halves and the result scaled by 4, so each half is the
        // shared byte address of its bin: every half stays in [0, 0x4000) on the way (the
        // histogram starts below 32 KB), so no carry or borrow crosses the halves.
        const uint32_t hbase = smem_u32(sh->hist);
        const uint32_t hq = hbase >> 2;
        const uint32_t koff = ((hq << 16) | hq) - 0xBA80BA80u;
        if (hbase + 4u * 0x2000u > 0x10000u && tid == 0) atomicOr(&a.ws->err, 32u);  // layout
        auto hist_fn = [&](const uint4& x, int) {
            const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
            vmax2 = bf2_max(vmax2, bf2_max(bf2_max(xs[0], xs[1]), bf2_max(xs[2], xs[3])));
            // fine iff 2^-20 <= |v| < 2^12, i.e. 0x3580 <= |bits| <= 0x457F: bit 15 of
            // |bits| + 0x4A80 says ">= 0x3580", of |bits| + 0x3A80 says ">= 0x4580"
            uint32_t f[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t a2 = xs[q] & 0x7FFF7FFFu;
                f[q] = (a2 + 0x4A804A80u) & ~(a2 + 0x3A803A80u);
            }
            uint32_t rare = 0;  // bit q: word q has an element outside the fine bins
            if ((f[0] & f[1] & f[2] & f[3] & 0x80008000u) == 0x80008000u) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t w = xs[q];
                    const uint32_t sgn = prmt_sign16(w);
                    const uint32_t b2 = ((w ^ ~sgn) + (sgn & 0x15001500u) + koff) << 2;
                    red_shared_inc(b2 & 0xFFFFu);
                    red_shared_inc(b2 >> 16);
                }
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    if ((f[q] & 0x80008000u) == 0x80008000u) {
                        const uint32_t w = xs[q];
                        const uint32_t sgn = prmt_sign16(w);
                        const uint32_t b2 = ((w ^ ~sgn) + (sgn & 0x15001500u) + koff) << 2;
                        red_shared_inc(b2 & 0xFFFFu);
                        red_shared_inc(b2 >> 16);
                    } else {
                        rare |= 1u << q;
                    }
                }
            }
            if (rare) {
#pragma unroll 1
                for (int h = 0; h < 8; ++h) {
                    if (!(rare & (1u << (h >> 1)))) continue;
                    const uint32_t u16 = (h & 1) ? (xs[h >> 1] >> 16) : (xs[h >> 1] & 0xFFFFu);
                    const uint32_t ab = u16 & 0x7FFFu;
                    if (ab >= 0x3580u && ab <= 0x457Fu) {          // a fine element
                        atomicAdd(&sh->hist[(u16 & 0x8000u) ? ab - 0x2580u : 0x457Fu - u16], 1u);
                        continue;
                    }
                    if (u16 == 0xFF80u) continue;                   // -inf (and the row's fill)
                    if (ab < 0x3580u) {                             // the band |v| < 2^-20
                        const uint32_t p = atomicAdd(&sh->nband, 1u);
                        if (p < (uint32_t)kBandCap) sh->band[p] = (uint16_t)u16;
                    } else {
                        sh->outside = 1u;                           // |v| >= 2^12, inf, NaN
                    }
                }
            }
        };
        const int nread = stream_row(sh, a, g, V, hist_fn, hb, he);
        if (tid == 0) {
            sh->hbm_vecs = (uint32_t)nread;
            sh->watch_s = -1;  // later passes run from L2 and are short: not abandoned
        }
        if (sh->abort_row) return;  // the row can no longer change an outcome
        {
            const uint32_t k0 = okey(vmax2 & 0xFFFFu), k1 = okey(vmax2 >> 16);
            tkey = k0 > k1 ? k0 : k1;
        }
        PROF_MARK(ti.cat, 2);
        const uint32_t wk0 = __reduce_max_sync(0xffffffffu, tkey);
        if (lane == 0) sh->red32[wid] = wk0;
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kRW; ++i) mkey = max(mkey, sh->red32[i]);
        if (half == 0) {
            split_publish(sh, a, ti.slot, mkey);
            return;
        }
        if (half == 1) mkey = split_merge(sh, a, ti.slot, mkey);
        fixed_hist = sh->outside == 0u && sh->nband <= (uint32_t)kBandCap && mkey > kNInfRaw &&
                     mkey <= kFTop;
        __syncthreads();
    }
    if (!fixed_hist) {
        // ---- pass 1: max (greedy rows: and the first index of the max) ---------------
        tkey = 0;
        int tfirst = 0x7fffffff;
        auto max_fn = [&](const uint4& x, int v) {
            uint32_t mx = bf2_max(bf2_max(x.x, x.y), bf2_max(x.z, x.w));
            const uint32_t k0 = okey(mx & 0xFFFFu), k1 = okey(mx >> 16);
            const uint32_t vk = k0 > k1 ? k0 : k1;
            if (vk > tkey) {
                tkey = vk;
                if (greedy) {
                    // first half of this vector with the new maximum (vectors arrive in order)
                    const uint32_t b = key_bits(vk);
                    const uint32_t b2 = b | (b << 16);
                    const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
                    int f = 0x7fffffff;
#pragma unroll
                    for (int h = 7; h >= 0; --h) {
                        const uint32_t eq = bf2_eq(xs[h >> 1], b2) & ((h & 1) ? 0xFFFF0000u : 0x0000FFFFu);
                        const int e = 8 * v + h - g.off;
                        if (eq && e >= 0 && e < V) f = e;
                    }
                    tfirst = f;
                }
            }
        };
        const int nread = stream_row<true>(sh, a, g, V, max_fn);
        if (tid == 0) {
            if (!onepass) sh->hbm_vecs = (uint32_t)nread;
            sh->watch_s = -1;
        }
        if (sh->abort_row) return;
        PROF_MARK(ti.cat, 0);
        const uint32_t wk = __reduce_max_sync(0xffffffffu, tkey);
        if (lane == 0) sh->red32[wid] = wk;
        if (tid == 0) sh->first_min = 0x7fffffff;
        __syncthreads();
        mkey = 0;
#pragma unroll
        for (int i = 0; i < kRW; ++i) mkey = max(mkey, sh->red32[i]);
        if (greedy) {
            if (tkey == mkey && tfirst != 0x7fffffff) atomicMin(&sh->first_min, tfirst);
            __syncthreads();
            if (tid == 0) {
                const int f = sh->first_min;
                // always written (0: no finite maximum), so no value of an earlier launch is read
                a.gmax[ti.b * kT + ti.s] =
                    f == 0x7fffffff ? 0ull : (((unsigned long long)mkey << 32) | (0xFFFFFFFFull - (unsigned)f));
                put_desc(a, ti, bf(key_bits(mkey)), mkey, f, 1ull << kFixBits, f == 0x7fffffff ? 0 : f,
                         kDescGreedy);
            }
            PROF_END(ti.cat, 1);
            return;
        }
    }
    const float m = bf(key_bits(mkey));
    const long long k_top = ti.k < V ? (long long)ti.k : (long long)V;
    long long kk = k_top;
    if (ti.mp > 0.0f) {
        // min-p: the kept set is also a prefix of the elements at or above the floor key
        if (tid == 0) sh->sel[13] = (int)key16_floor(minp_floor32(m, ti.c, ti.mp));
        __syncthreads();
        const uint32_t kf = (uint32_t)sh->sel[13];
        const long long cm = kf > 0xFFFFu ? 0ll : count_ge_key(sh, a, g, V, kf);
        if (cm < kk) kk = cm;
        if (kk < 1) kk = 1;
    }
    const int cat = ti.cat;
    const bool nucleus = ti.p < 1.0f;
    const uint32_t kninf = okey(0xFF80u);  // key of -inf
    KeyStop ks;
    ks.found = 0;
    unsigned long long S = 0;
    long long thr = 0x7fffffffffffffffll;
    // sequential mode: top-p is taken against the mass of the top-k elements (k before the
    // min-p floor), found by counting from the top
    unsigned long long s_top = 0;
    bool have_s_top = false;
    if (seq_k) {
        const KeyStop k1 = count_walk(sh, a, g, V, mkey, kninf, m, ti.c, 0ull, 0ull, k_top, thr);
        if (k1.found) {
            s_top = k1.mass + (unsigned long long)(k_top - (long long)k1.cnt) * k1.F;
            have_s_top = true;
        }
    }

    if (cat == kWindow) {
        // ---- pure top-k, k <= 256: candidates >= tau, ranked exactly -------------------
        // tau = the largest value with at least k thread maxima >= tau (each such thread
        // holds an element >= tau)
        uint32_t tau = 0;
        for (int bit = 15; bit >= 0; --bit) {
            const uint32_t cand = tau | (1u << bit);
            if (__syncthreads_count(tkey >= cand) >= kk) tau = cand;
        }
        if (tau < kninf) tau = kninf;  // fewer than k threads hold data (tiny vocabularies)
        if (tid == 0) sh->nlist = 0;
        __syncthreads();
        const uint32_t taub = key_bits(tau);
        const uint32_t tau2 = taub | (taub << 16);
        stream_row(sh, a, g, V, [&](const uint4& x, int v) {
            const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t ge = bf2_ge(xs[q], tau2);
                if (!ge) continue;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int e = 8 * v + 2 * q + h - g.off;
                    if ((ge & (h ? 0xFFFF0000u : 0x0000FFFFu)) && e >= 0 && e < V) {
                        const uint32_t pos = atomicAdd(&sh->nlist, 1u);
                        if (pos < kRWinCap) {
                            sh->hist[pos] = okey(h ? (xs[q] >> 16) : (xs[q] & 0xFFFFu));
                            sh->hist[kRWinCap + pos] = (uint32_t)e;
                        }
                    }
                }
            }
        });
        PROF_MARK(ti.cat, 2);
        const int n = (int)sh->nlist;
        if (n >= 1 && n <= kRWinCap) {
            // rank the candidates by (key desc, index asc); the first k are kept
            // candidates: keys hist[0, n), indices hist[kRWinCap, kRWinCap + n); the ranked
            // list goes to the ring (idle after the pass)
            const uint32_t* wkey = sh->hist;
            const uint32_t* widx = sh->hist + kRWinCap;
            uint2* srt = reinterpret_cast<uint2*>(&sh->ring[0][0]);
            for (int i = tid; i < n; i += kRT) {
                const uint32_t ki = wkey[i], xi = widx[i];
                int r = 0;
                for (int j = 0; j < n; ++j) {
                    const uint32_t kj = wkey[j];
                    r += (kj > ki) || (kj == ki && widx[j] < xi);
                }
                srt[r] = make_uint2(ki, xi);
            }
            __syncthreads();
            if (tid < 32) {
                const int nsel = n < kk ? n : (int)kk;
                unsigned long long sk = 0;
                for (int r = lane; r < nsel; r += 32)
                    sk += fix_of_y(y_clamped(bf(key_bits(srt[r].x)), m, ti.c));
                sk = warp_sum_u64(sk);
                if (lane == 0) put_desc(a, ti, m, srt[nsel - 1].x, (int)srt[nsel - 1].y, sk, 0, 0u);
            }
            PROF_END(ti.cat, 3);
            return;
        }
        // the window overflowed (many equal values): exact counts from the top instead
        ks = count_walk(sh, a, g, V, mkey, kninf, m, ti.c, 0ull, 0ull, kk, thr);
    } else if (cat == kKeepAll || nucleus) {
        // ---- exact per-key histogram of every element with nonzero fixed-point mass -----
        // key < klo: y < -42 so fix(exp2(y)) = 0; such elements are never in a nucleus
        // (their mass ranked ahead is S > floor(top_p S)) and add nothing to S.
        const float vlo = m - 42.5f / ti.c;
        uint32_t klo = kninf + 1u;
        if (vlo > -INFINITY) {
            const uint32_t vb = __float_as_uint(vlo) >> 16;  // truncated toward zero
            const uint32_t kt = okey(vb);
            klo = kt > kninf + 1u ? kt - 1u : kninf + 1u;      // one bf16 step below vlo
        }
        if (klo > mkey) klo = mkey;
        uint32_t kB = 0x8000u, kNB = 0x7FFFu, npos = 0, nneg = 0, negtop = 0, topkey = 0;
        if (fixed_hist) {
            // the one-pass histogram: fixed bins, the band's elements listed
            kB = kFB;
            kNB = kFNB;
            npos = kFPos;
            nneg = kFPos;
            negtop = kFNB;
            topkey = kFTop;
            if (tid == 0) {
                sh->zcnt = 0u;
                sh->zmass = 0ull;
            }
            __syncthreads();
            const uint32_t nb = sh->nband;
            for (uint32_t i = tid; i < nb; i += kRT) {
                const uint32_t u16 = sh->band[i];
                const uint32_t key = okey(u16);
                if (key < klo || key > mkey) continue;
                atomicAdd(&sh->zcnt, 1u);
                const unsigned long long F = fix_of_y(y_clamped(bf(u16), m, ti.c));
                if (F) atomicAdd(&sh->zmass, F);
            }
            __syncthreads();
        } else {
            // the band |v| < 2^zb is left out of the histogram (exact per element, usually
            // empty): the smallest band for which the rest fits kHCap bins
            for (int zb = -126; zb <= 127; ++zb) {
                const uint32_t bits = (uint32_t)(127 + zb) << 7;
                kB = 0x8000u | bits;          // key of +2^zb
                kNB = 0x7FFFu - bits;         // key of -2^zb
                npos = mkey >= kB ? mkey - kB + 1u : 0u;
                const uint32_t ntop = kNB < mkey ? kNB : mkey;
                nneg = ntop >= klo ? ntop - klo + 1u : 0u;
                if (npos + nneg <= (uint32_t)kHCap - 64u) break;  // ceil/32 of both parts <= 256
            }
            negtop = kNB < mkey ? kNB : mkey;
            topkey = mkey;
            __syncthreads();
            for (uint32_t i = tid; i < npos + nneg; i += kRT) sh->hist[i] = 0u;
            if (tid == 0) {
                sh->zcnt = 0u;
                sh->zmass = 0ull;
            }
            __syncthreads();
            const float mz = m, cz = ti.c;
            const uint32_t nposv = npos, negv = npos + negtop, mk = mkey, kl = klo, kb = kB, knb = kNB;
            stream_row(sh, a, g, V, [&](const uint4& x, int) {
                const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
                uint32_t band = 0;  // bit h: element h of this vector is in the band
#pragma unroll
                for (int h = 0; h < 8; ++h) {
                    const uint32_t u16 = (h & 1) ? (xs[h >> 1] >> 16) : (xs[h >> 1] & 0xFFFFu);
                    // ordered key (-0 joins +0 inside the band, which is handled exactly below)
                    const uint32_t key = u16 ^ ((u16 & 0x8000u) ? 0xFFFFu : 0x8000u);
                    const bool pos = key >= kb;
                    const uint32_t idx = pos ? mk - key : negv - key;
                    const bool fine = key >= kl && key <= mk && (pos || key <= knb);
                    if (fine) atomicAdd(&sh->hist[idx], 1u);
                    band |= (key >= kl && key <= mk && !pos && key > knb) ? (1u << h) : 0u;
                }
                if (band) {
#pragma unroll 1
                    for (int h = 0; h < 8; ++h) {
                        if (!(band & (1u << h))) continue;
                        const uint32_t u16 = (h & 1) ? (xs[h >> 1] >> 16) : (xs[h >> 1] & 0xFFFFu);
                        const unsigned long long F = fix_of_y(y_clamped(bf(u16), mz, cz));
                        atomicAdd(&sh->zcnt, 1u);
                        if (F) atomicAdd(&sh->zmass, F);
                    }
                }
            });
            (void)nposv;
        }
        PROF_MARK(ti.cat, 2);
        // ---- S and the walk over groups of 32 bins: positive groups, the band, negative
        // groups (rank order).  Thread g sums group g (its 32 bins in a skewed order, so the
        // lanes of a warp read distinct banks; one fix(exp2c) per nonzero bin), thread g
        // scans group g, and the warp of the stopping group finds the bin.
        const uint32_t ngp = (npos + 31u) >> 5, ngn = (nneg + 31u) >> 5, ng = ngp + ngn;
        for (uint32_t gi = (uint32_t)tid; gi < ng; gi += kRT) {
            const bool neg = gi >= ngp;
            const uint32_t b0 = (neg ? gi - ngp : gi) << 5;   // first bin within its part
            const uint32_t lim = neg ? nneg : npos;
            const uint32_t* hp = sh->hist + (neg ? npos : 0u);
            const uint32_t top = neg ? negtop : topkey;
            uint32_t gc = 0;
            unsigned long long gm = 0;
            // branchless, two bins per packed exp: keys below klo (and empty bins) give
            // fix = 0 or count 0, so every bin can be evaluated
            const float2 nm2 = make_float2(-m, -m), c2 = make_float2(ti.c, ti.c);
#pragma unroll 4
            for (uint32_t jp = 0; jp < 16u; ++jp) {
                const uint32_t i0 = b0 + ((2u * jp + 2u * (uint32_t)tid) & 31u);
                // (scalar loads: the negative part's base, hist + npos, may be odd)
                const uint2 cc = make_uint2(i0 < lim ? hp[i0] : 0u, i0 + 1u < lim ? hp[i0 + 1u] : 0u);
                const uint32_t w = key_bits(top - i0) | (key_bits(top - i0 - 1u) << 16);
                const Pair pr = exp_pair(w, nm2, c2);
                const unsigned long long F0 =
                    (unsigned long long)((long long)(pr.h0 - 0x4B000000u) * 8388608 + (int32_t)(pr.l0 - 0x4B400000u));
                const unsigned long long F1 =
                    (unsigned long long)((long long)(pr.h1 - 0x4B000000u) * 8388608 + (int32_t)(pr.l1 - 0x4B400000u));
                gc += cc.x + cc.y;
                gm += (unsigned long long)cc.x * F0 + (unsigned long long)cc.y * F1;
            }
            sh->gcnt[gi] = gc;
            sh->gmass[gi] = gm;
        }
        __syncthreads();
        const unsigned long long zc = sh->zcnt, zm = sh->zmass;
        const uint32_t gme = (uint32_t)tid;
        const unsigned long long ct = gme < ng ? sh->gcnt[gme] : 0ull;
        const unsigned long long mt = gme < ng ? sh->gmass[gme] : 0ull;
        unsigned long long ci = ct, mi = mt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long x1 = __shfl_up_sync(0xffffffffu, ci, o);
            const unsigned long long x2 = __shfl_up_sync(0xffffffffu, mi, o);
            if (lane >= o) {
                ci += x1;
                mi += x2;
            }
        }
        if (lane == 31) {
            sh->red64[wid] = ci;
            sh->wm[wid] = mi;
        }
        if (tid == 0) sh->sel[6] = 0x7fffffff;
        __syncthreads();
        unsigned long long cb = ci - ct, mb = mi - mt, Sall = 0;
        for (int w = 0; w < kRW; ++w) {
            if (w < wid) {
                cb += sh->red64[w];
                mb += sh->wm[w];
            }
            Sall += sh->wm[w];
        }
        if (gme >= ngp) {
            cb += zc;
            mb += zm;
        }
        S = Sall + zm;
        if (cat == kKeepAll || !nucleus) {
            if (tid == 0) put_desc(a, ti, m, 0u, 0x7fffffff, S, 0, 0u);
            PROF_END(ti.cat, 3);
            return;
        }
        thr = scale_floor(ti.p, have_s_top ? s_top : S);
        PROF_MARK(ti.cat, 4);
        if (gme < ng && ct > 0 && ((long long)(cb + ct) >= kk || (long long)(mb + mt) > thr))
            atomicMin(&sh->sel[6], tid);
        if (gme + 1u == ngp || (ngp == 0u && tid == 0)) {
            // the band, between the positive and the negative groups
            const unsigned long long c0 = ngp ? cb + ct : 0ull, m0 = ngp ? mb + mt : 0ull;
            const bool bstop = zc > 0 && ((long long)(c0 + zc) >= kk || (long long)(m0 + zm) > thr);
            sh->sel[9] = bstop ? 1 : 0;
            sh->self64[7] = c0;
            sh->self64[6] = m0;
        }
        __syncthreads();
        const int owner = sh->sel[6];
        const bool band_stop = sh->sel[9] != 0 && (owner == 0x7fffffff || (uint32_t)owner >= ngp);
        if (tid == 0) sh->sel[10] = owner;
        if (owner != 0x7fffffff && !band_stop) {
            // the owner group's prefix, then the first bin of it that stops
            if (tid == owner) {
                sh->self64[4] = cb;
                sh->self64[5] = mb;
            }
            __syncthreads();
            const uint32_t go = (uint32_t)owner;
            if (wid == 0) {
                const bool neg = go >= ngp;
                const uint32_t j = neg ? go - ngp : go;
                const uint32_t i = (j << 5) + lane;
                const uint32_t lim = neg ? nneg : npos;
                uint32_t cnt = 0;
                unsigned long long F = 0;
                uint32_t key = 0;
                if (i < lim) {
                    cnt = sh->hist[(neg ? npos : 0u) + i];
                    key = (neg ? negtop : topkey) - i;
                    if (cnt && key >= klo) F = fix_of_y(y_clamped(bf(key_bits(key)), m, ti.c));
                }
                const unsigned long long c0 = sh->self64[4], m0 = sh->self64[5];
                const unsigned long long mm = (unsigned long long)cnt * F;
                const unsigned long long cin = warp_incl_u64(cnt), min_ = warp_incl_u64(mm);
                const unsigned long long cbl = c0 + cin - cnt, mbl = m0 + min_ - mm;
                const bool stop = cnt > 0 && ((long long)(cbl + cnt) >= kk || (long long)(mbl + mm) > thr);
                const uint32_t bal = __ballot_sync(0xffffffffu, stop);
                const int sl = bal ? __ffs(bal) - 1 : 0;
                if (lane == sl) {
                    sh->sel[7] = (int)key;
                    sh->sel[8] = (int)cnt;
                    sh->self64[4] = cbl;
                    sh->self64[5] = mbl;
                    sh->self64[3] = F;
                    sh->sel[11] = bal ? 1 : 0;
                }
            }
            __syncthreads();
            ks.found = sh->sel[11];
            ks.key = (uint32_t)sh->sel[7];
            ks.count = (uint32_t)sh->sel[8];
            ks.cnt = sh->self64[4];
            ks.mass = sh->self64[5];
            ks.F = sh->self64[3];
            __syncthreads();
        } else if (band_stop) {
            const unsigned long long c0 = sh->self64[7], m0 = sh->self64[6];
            __syncthreads();
            const uint32_t btop = (kB - 1u) < mkey ? kB - 1u : mkey;
            const uint32_t bbot = (kNB + 1u) > klo ? kNB + 1u : klo;
            ks = count_walk(sh, a, g, V, btop, bbot, m, ti.c, c0, m0, kk, thr);
        }
    } else {
        // ---- pure top-k with k > 256: exact counts from the top ------------------------
        ks = count_walk(sh, a, g, V, mkey, kninf, m, ti.c, 0ull, 0ull, kk, thr);
    }
    if (!ks.found) {
        if (tid == 0) {
            atomicOr(&a.ws->err, 8u);
            put_desc(a, ti, m, 0u, 0x7fffffff, S, 0, 0u);
        }
        return;
    }
    PROF_MARK(ti.cat, 6);
    unsigned long long ntie = ks.count;
    if ((long long)(ks.cnt + ntie) > kk) ntie = (unsigned long long)(kk - (long long)ks.cnt);
    if (ks.F > 0 && (long long)ks.mass <= thr) {
        const unsigned long long pb_ = (unsigned long long)(thr - (long long)ks.mass) / ks.F + 1ull;
        if (pb_ < ntie) ntie = pb_;
    }
    if (ntie < 1) ntie = 1;
    const unsigned long long skept = ks.mass + ntie * ks.F;
    if (ntie >= ks.count) {
        if (tid == 0) put_desc(a, ti, m, ks.key, 0x7fffffff, skept, 0, 0u);
        PROF_END(ti.cat, 7);
        return;
    }

    // ---- tie cut: occurrence number ntie of the boundary key in index order ------------
    {
        // from the nearer end: occurrence ntie of count in index order is occurrence
        // count - ntie + 1 from the end.  Only for a normal nonzero key, where equal values are
        // equal bits, so the scan's matches are exactly the key's counted elements.
        const uint32_t kexp = (key_bits(ks.key) >> 7) & 0xFFu;
        const bool normal_key = kexp != 0u && kexp != 0xFFu;
        // a row that can no longer change an outcome stops here (no descriptor: nothing reads it)
        if (tid == 0 && sh->late_s >= 0 && !row_needed(a, sh->late_b, sh->late_s)) sh->abort_row = 1;
        __syncthreads();
        if (sh->abort_row) return;
        const int tie = (!normal_key || 2 * ntie <= (unsigned long long)ks.count + 1ull)
                            ? tie_scan<false>(sh, a, g, V, ks.key, ntie)
                            : tie_scan<true>(sh, a, g, V, ks.key, (unsigned long long)ks.count - ntie + 1ull);
        if (tie == -2) {
            if (tid == 0) sh->abort_row = 1;
            __syncthreads();
            return;
        }
        if (tid == 0) {
            if (tie < 0) atomicOr(&a.ws->err, 16u);
            put_desc(a, ti, m, ks.key, tie, skept, 0, 0u);
        }
    }
    PROF_END(ti.cat, 8);
}

// One row task (all threads); returns the bytes its first pass read from memory (the later
// passes re-read the row from L2).  abort_row is set if the row was abandoned.
__device__ unsigned long long process_row(RSmem* sh, const VerifyArgs& a, const TaskInfo& ti) {
    process_row_body(sh, a, ti);
    __syncthreads();
    return (unsigned long long)sh->hbm_vecs * 16ull;
}

// a row descriptor written by another CTA of this launch (L2, not a stale L1 line)
__device__ __forceinline__ RowDesc load_desc_cg(const RowDesc* p) {
    static_assert(sizeof(RowDesc) == 32, "row descriptor: two 16-byte words");
    const uint4 w0 = __ldcg(reinterpret_cast<const uint4*>(p));
    const uint4 w1 = __ldcg(reinterpret_cast<const uint4*>(p) + 1);
    RowDesc d;
    d.m = __uint_as_float(w0.x);
    d.c = __uint_as_float(w0.y);
    d.inv_s = __uint_as_float(w0.z);
    d.kstar = w0.w;
    d.tie_cut = (int32_t)w1.x;
    d.argmax = (int32_t)w1.y;
    d.flags = w1.z;
    d.pad = w1.w;
    return d;
}


__device__ __forceinline__ uint64_t fix_w(float w) {
    if (!(w > 0.0f)) return 0;
    return fix01(fminf(w, 1.0f));
}

// the five outputs of request b (sampling/rejection.py:66-98 output convention)
__device__ void write_request(const VerifyArgs& a, int b, int acc, long long bonus) {
    a.accept[b] = acc;
    a.commit[b] = acc + 1;
    a.bonus[b] = bonus;
    for (int i = 0; i < kT; ++i) {
        long long v = 0;
        if (i < acc) v = a.cand[b * kT + i + 1];
        else if (i == acc) v = bonus;
        a.output[b * kT + i] = v;
    }
    a.new_seq[b] = a.prefix[b] + acc + 1;
}

// ---------------------------------------------------------------------------------------
// chain + bonus + outputs: up to kCP CTAs per request (chain_slices), no cluster
//
// Every CTA of a request decides the chain (warp 0, one lane per step), then takes one slice
// of the bonus row: the slice's exact residual mass goes to the request's task-result area in
// the workspace (unused by this path otherwise).  The last CTA of the request (a done
// counter) forms the threshold from the slice totals, rescans only the crossing slice tile by
// tile (block scans) and writes the five outputs; the last request packs tokens and KV slots.
// p is evaluated only for kept elements and q only where p > 0 (the residual is 0 elsewhere).

constexpr int kCP = 32;                   // CTAs (slices) per request
constexpr int kCT = 256;                  // threads per CTA (4 CTAs per SM: one wave)
constexpr int kCTW = kCT / 32;
static_assert(kCP * 1 <= 2 * kT, "slice masses live in the request's task-result area (32 u64)");
static_assert(kCP <= 32 && kCTW <= 8, "per-warp slice masses: [B][32][8] in the workspace");

struct ChainSmem {
    uint2 queue[kCTW][256];        // per warp: kept elements of one vector per lane
    unsigned long long wsum[kCTW];
    uint32_t red_a[kRW > kCTW ? kRW : kCTW], red_b[kRW > kCTW ? kRW : kCTW];  // per warp of the CTA
    unsigned long long slice[kCP];
    long long thr, base;
    int acc, bonus, flag, last, cross;
    unsigned long long total;
};

template <int NT>
__device__ void compact_all_nt(const VerifyArgs& a, uint32_t* red_a, uint32_t* red_b) {
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    int run_c = 0, run_f = 0;
    if (tid == 0) {
        a.offsets[0] = 0;
        a.free_offsets[0] = 0;
    }
    for (int b0 = 0; b0 < a.B; b0 += NT) {
        const int b = b0 + tid;
        int cm = 0, fr = 0;
        if (b < a.B) {
            const int cap = clamp_cap(a.caps[b]);
            cm = __ldcg(&a.commit[b]);
            fr = cap - cm;
            if (fr < 0) fr = 0;
        }
        const uint32_t ic = warp_incl_u32((uint32_t)cm);
        const uint32_t iff = warp_incl_u32((uint32_t)fr);
        if (lane == 31) {
            red_a[w] = ic;
            red_b[w] = iff;
        }
        __syncthreads();
        int wc = 0, wf = 0, tc = 0, tf = 0;
        for (int q = 0; q < NW; ++q) {
            if (q < w) {
                wc += (int)red_a[q];
                wf += (int)red_b[q];
            }
            tc += (int)red_a[q];
            tf += (int)red_b[q];
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

// the bonus row of one request: p row (target), q (draft row, one-hot or none)
struct BonusRow {
    RowDesc dt, dd;
    bool has_dq;
    const uint16_t* prow;
    const uint16_t* qrow;
    long long onehot;
    int poff;     // misalignment of prow in elements
    int nvp;      // 16-byte vectors covering the p row
    bool qvec;    // q row has the same alignment: load q vectors alongside
};

constexpr int kCTileV = 4 * kCT;           // vectors per tile: 4 consecutive per thread
constexpr int kCMaxTiles = 1;              // tiles per slice (kCP x kCMaxTiles <= 32): V <= kMaxV
static_assert(kCMaxTiles == 1, "the crossing search takes the slice as its tile");
constexpr int kMaxV = 8 * (kCP * kCMaxTiles * kCTileV - kCP) - 16;  // vectors of every slice fit

// Slices (chain tasks) per sampled request for rows of V elements: as few as keep every slice
// within one tile (a row at any alignment spans at most (V + 14) / 8 vectors), at most kCP.
// Fewer, fuller slices: the per-task costs (descriptor loads, block sums, the dequeue) are paid
// fewer times (V = 151936: 19 slices instead of 32).
__device__ __forceinline__ int chain_slices(int V) {
    const int nvp = (V + 14) >> 3;
    const int n = (nvp + kCTileV - 1) / kCTileV;
    return n < 1 ? 1 : (n > kCP ? kCP : n);
}

__device__ __forceinline__ bool kept_in(const RowDesc& d, uint32_t u16, int i) {
    const uint32_t k = okey(u16);
    return (k > d.kstar) || (k == d.kstar && i <= d.tie_cut);
}

// residual fixed-point weight of one kept p element (p bits pb, q bits qb, index i)
__device__ __forceinline__ unsigned long long resid_kept(const BonusRow& r, bool pure, uint32_t pb,
                                                         uint32_t qb, int i) {
    const float p = __fmul_rn(exp2c(__fmul_rn(__fadd_rn(bf(pb), -r.dt.m), r.dt.c)), r.dt.inv_s);
    if (!(p > 0.0f)) return 0ull;
    float w = p;
    if (!pure) {
        float q;
        if (r.has_dq) q = row_prob(r.dd, bf(qb), qb, i);
        else q = (i == r.onehot) ? 1.0f : 0.0f;
        const float qq = (q >= 0.0f && q <= 1.0f) ? q : 0.0f;
        w = fmaxf(__fsub_rn(p, qq), 0.0f);
    }
    return fix_w(w);
}

// p and q bits of the 8 elements of p-row vector v
__device__ __forceinline__ void load8(const BonusRow& r, int v, bool pure, uint4& x, uint4& y) {
    x = __ldg(reinterpret_cast<const uint4*>(r.prow - r.poff) + v);
    y = make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u);
    if (!pure && r.has_dq && r.qvec) y = __ldg(reinterpret_cast<const uint4*>(r.qrow - r.poff) + v);
}

__device__ __forceinline__ uint32_t half16(const uint4& x, int h) {
    const uint32_t w = h < 2 ? x.x : (h < 4 ? x.y : (h < 6 ? x.z : x.w));
    return (h & 1) ? (w >> 16) : (w & 0xFFFFu);
}

// Residual mass of tile [tv0, tv1) (vectors; thread t owns 4 consecutive vectors).  Kept p
// elements are queued per warp (shared memory) and evaluated 32 at a time, so the exps are
// not serialised by lanes whose elements are outside the kept set.  Returns this thread's sum.
__device__ unsigned long long tile_mass(const BonusRow& r, int V, int tv0, int tv1, bool pure,
                                        uint2* queue) {
    const int tid = threadIdx.x, lane = tid & 31;
    unsigned long long mine = 0;
    if (tid >= kCT) return 0ull;  // a tile is kCT threads' work (whole warps return here)
    // the thread's 4 vectors (p and q) are loaded before any is used
    uint4 xa[4], ya[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int v = tv0 + 4 * tid + u;
        xa[u] = make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u);
        ya[u] = xa[u];
        if (v < tv1) load8(r, v, pure, xa[u], ya[u]);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        const int v = tv0 + 4 * tid + u;
        const uint4 x = xa[u], y = ya[u];
        uint32_t keep = 0;
#pragma unroll
        for (int h = 0; h < 8; ++h) {
            const int i = 8 * v + h - r.poff;
            if (v < tv1 && i >= 0 && i < V && kept_in(r.dt, half16(x, h), i)) keep |= 1u << h;
        }
        const uint32_t n = __popc(keep);
        const uint32_t incl = warp_incl_u32(n);
        const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
        uint32_t slot = incl - n;
        while (keep) {
            const int h = __ffs(keep) - 1;
            keep &= keep - 1;
            const int i = 8 * v + h - r.poff;
            uint32_t qb = half16(y, h);
            if (!pure && r.has_dq && !r.qvec) qb = r.qrow ? (uint32_t)__ldg(r.qrow + i) : 0xFF80u;
            queue[slot++] = make_uint2(half16(x, h) | (qb << 16), (uint32_t)i);
        }
        __syncwarp();
        for (uint32_t e = lane; e < total; e += 32) {
            const uint2 q = queue[e];
            mine += resid_kept(r, pure, q.x & 0xFFFFu, q.x >> 16, (int)q.y);
        }
        __syncwarp();
    }
    return mine;
}

__device__ __forceinline__ unsigned long long block_sum_u64(unsigned long long v,
                                                            unsigned long long* wsum) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    v = warp_sum_u64(v);
    __syncthreads();
    if (lane == 0 && wid < kCTW) wsum[wid] = v;  // warps beyond kCTW hold no tile work
    __syncthreads();
    unsigned long long t = 0;
#pragma unroll
    for (int w = 0; w < kCTW; ++w) t += wsum[w];
    __syncthreads();
    return t;
}

// One chain task: slice `rank` of sampled request b (its accepted length was decided by the row
// pass).  Each task sums the exact residual mass of its slice of the rejected position's rows
// and records per-warp masses; the task that completes the request's slices finds the bonus
// token and writes the request's outputs (returns true).
__device__ bool chain_task(const VerifyArgs& a, ChainSmem* sh, int b, int rank) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int cap = clamp_cap(a.caps[b]);
    const uint16_t* tgt = reinterpret_cast<const uint16_t*>(a.tgt);
    const uint16_t* drf = reinterpret_cast<const uint16_t*>(a.drf);
    const bool onehot_q = a.drf == nullptr;
    bool finished = false;
    (void)lane;
    // the accepted length, decided by the row kernel when the request's rows completed
    if (tid == 0) sh->acc = outcome_of(__ldcg(&a.racc[2 * b + 1]), cap);  // claimed: known
    __syncthreads();
    const int acc = sh->acc;
    const bool pure0 = acc == cap - 1;
    const int V = a.V;
    BonusRow r;
    r.dt = load_desc_cg(&a.desc[(b * kT + acc) * 2 + 0]);
    const long long tr = a.tgt_row[b] + acc;
    r.prow = (tr >= 0 && tr < a.tgt_rows) ? tgt + tr * a.stride : nullptr;
    r.has_dq = false;
    r.qrow = nullptr;
    r.onehot = -1;
    if (!pure0) {
        if (onehot_q) {
            r.onehot = a.cand[b * kT + acc + 1];
        } else {
            r.dd = load_desc_cg(&a.desc[(b * kT + acc) * 2 + 1]);
            r.has_dq = true;
            const long long dr = a.drf_row[b] + acc;
            if (dr >= 0 && dr < a.drf_rows) r.qrow = drf + dr * a.stride;
        }
    }
    r.poff = r.prow ? (int)((reinterpret_cast<uintptr_t>(r.prow) & 15u) >> 1) : 0;
    r.nvp = r.prow ? (V + r.poff + 7) >> 3 : 0;
    r.qvec = r.qrow && (int)((reinterpret_cast<uintptr_t>(r.qrow) & 15u) >> 1) == r.poff;
    // this CTA's slice of vectors, in tiles of kCTileV; tile masses go to the request's
    // task-result area (kCP x kCMaxTiles u64)
    const int ncp = chain_slices(V);
    const int per = (r.nvp + ncp - 1) / ncp;
    const int v0 = min(rank * per, r.nvp), v1 = min(v0 + per, r.nvp);
    unsigned long long* tmass = reinterpret_cast<unsigned long long*>(a.res) + (size_t)b * kT * 2;
    auto slice_tiles = [&](int q, bool pure_) -> unsigned long long {
        const int u0 = min(q * per, r.nvp), u1 = min(u0 + per, r.nvp);
        unsigned long long tot = 0;
        if (tid == 0 && u0 >= u1) tmass[q * kCMaxTiles] = 0ull;  // an empty slice
        for (int t = 0; u0 + t * kCTileV < u1 && t < kCMaxTiles; ++t) {
            const int tv0 = u0 + t * kCTileV, tv1 = min(tv0 + kCTileV, u1);
            const unsigned long long m =
                block_sum_u64(tile_mass(r, V, tv0, tv1, pure_, sh->queue[wid < kCTW ? wid : 0]), sh->wsum);
            if (tid == 0) tmass[q * kCMaxTiles + t] = m;
            // per-warp masses (still in shared memory) for the crossing search
            if (tid < kCTW) a.wmass[((size_t)b * kCP + q) * kCTW + tid] = sh->wsum[tid];
            tot += m;
        }
        return tot;
    };
    const unsigned long long mine = slice_tiles(rank, pure0);
    (void)v0;
    (void)v1;
    (void)mine;
    if (tid == 0) {
        __threadfence();
        const unsigned old = atomicAdd(&a.done[b], 1u);
        sh->last = old == (unsigned)(ncp - 1);
    }
    __syncthreads();
    if (sh->last) {
        __threadfence();
        bool pure = pure0;
        if (tid < ncp) sh->slice[tid] = __ldcg(&tmass[tid * kCMaxTiles]);  // one tile per slice
        __syncthreads();
        unsigned long long M = 0;
#pragma unroll
        for (int q = 0; q < ncp; ++q) M += sh->slice[q];
        if (!pure && M == 0) {
            // zero residual mass: draw from p (this CTA recomputes every slice)
            pure = true;
            M = 0;
            for (int q = 0; q < ncp; ++q) {
                const unsigned long long t = slice_tiles(q, true);
                if (tid == 0) sh->slice[q] = t;
                M += t;
            }
            __syncthreads();
        }
        const long long thr = scale_floor(a.uf[b], M);
        long long bonus = (long long)V - 1;
        if (thr == -1) {
            bonus = 0;  // u < 0: the first running sum already exceeds it
        } else if (thr != -2 && M != 0) {
            // the crossing slice and tile from the totals, then the tile element by element
            long long base = 0;
            int qs = -1, tq = -1;
            for (int q = 0; q < ncp && qs < 0; ++q) {
                const long long t = (long long)sh->slice[q];
                if (base + t > thr) {
                    qs = q;
                    tq = 0;  // one tile per slice (kCMaxTiles == 1)
                } else {
                    base += t;
                }
            }
            if (qs >= 0 && tq >= 0) {
                const int u0 = min(qs * per, r.nvp), u1 = min(u0 + per, r.nvp);
                const int tv0 = u0 + tq * kCTileV, tv1 = min(tv0 + kCTileV, u1);
                // the crossing warp from the slice's per-warp masses (warp w owns vectors
                // tv0 + 128 w ..., so warp order is index order), then that warp alone:
                // lane masses (4 consecutive vectors per lane), a warp scan, and the lane
                // holding the crossing walks its 32 elements
                const unsigned long long* wm = a.wmass + ((size_t)b * kCP + qs) * kCTW;
                unsigned long long wv[kCTW];
#pragma unroll
                for (int w = 0; w < kCTW; ++w) wv[w] = __ldcg(&wm[w]);  // independent loads
                int ws_ = kCTW - 1;
#pragma unroll
                for (int w = 0; w < kCTW; ++w) {
                    const long long m_ = (long long)wv[w];
                    if (base + m_ > thr) {
                        ws_ = w;
                        break;
                    }
                    base += m_;
                }
                if (tid == 0) sh->bonus = -1;
                __syncthreads();
                {
                    // the crossing warp's 128 vectors (1024 elements) by the whole CTA:
                    // thread t takes elements [4 t, 4 t + 4) of the region (half of
                    // vector t / 2), a block scan of the thread masses finds the thread,
                    // and it walks its four elements
                    // (threads beyond kCT take no element: the region is kCT threads' work)
                    const bool mine_t = tid < kCT;
                    const int v = tv0 + 128 * ws_ + (tid >> 1);
                    uint4 xa = make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u);
                    uint4 ya = xa;
                    if (mine_t && v < tv1) load8(r, v, pure, xa, ya);
                    unsigned long long f4[4];
                    unsigned long long own = 0;
#pragma unroll
                    for (int hh = 0; hh < 4; ++hh) {
                        const int h = 4 * (tid & 1) + hh;
                        const int i = 8 * v + h - r.poff;
                        unsigned long long f = 0;
                        if (mine_t && v < tv1 && i >= 0 && i < V && kept_in(r.dt, half16(xa, h), i)) {
                            uint32_t qb = half16(ya, h);
                            if (!pure && r.has_dq && !r.qvec)
                                qb = r.qrow ? (uint32_t)__ldg(r.qrow + i) : 0xFF80u;
                            f = resid_kept(r, pure, half16(xa, h), qb, i);
                        }
                        f4[hh] = f;
                        own += f;
                    }
                    const unsigned long long incl = warp_incl_u64(own);
                    if (lane == 31 && mine_t) sh->wsum[wid] = incl;
                    __syncthreads();
                    unsigned long long wpre = 0;
                    for (int w = 0; w < wid && mine_t; ++w) wpre += sh->wsum[w];
                    long long run = base + (long long)(wpre + incl - own);
                    if (mine_t && run <= thr && run + (long long)own > thr) {
#pragma unroll
                        for (int hh = 0; hh < 4; ++hh) {
                            run += (long long)f4[hh];
                            if (run > thr) {
                                sh->bonus = 8 * v + 4 * (tid & 1) + hh - r.poff;
                                break;
                            }
                        }
                    }
                }
                __syncthreads();
                if (sh->bonus >= 0) bonus = sh->bonus;
            }
        }
#ifdef DSV_PROFILE
        if (tid == 0) atomicAdd(a.prof + 64 + 15, 1ull);
        if (tid == 0 && b < 128) a.prof[128 + b] = globaltimer_ns();
#endif
        if (tid == 0) {
            write_request(a, b, acc, bonus);
            a.done[b] = 0u;
        }
        finished = true;
    }
    return finished;
}

// Step s of request b (s < cap - 1): draft token s + 1 against target row s, both rows done
// (sampling/rejection.py:66-98: u * q < p with q in (0, 1]).  Greedy requests: one-hot p at
// the row's first argmax (packed by the row pass), one-hot q at the drafted token.
__device__ bool step_accepted(const VerifyArgs& a, int b, int s, bool greedy) {
    const long long tok = a.cand[b * kT + s + 1];
    const bool valid = tok >= 0 && tok < a.V;
    float p = 0.0f, q = 0.0f;
    if (greedy) {
        const unsigned long long g = __ldcg(&a.gmax[b * kT + s]);
        const long long am = g ? (long long)(0xFFFFFFFFull - (g & 0xFFFFFFFFull)) : 0ll;
        p = (valid && tok == am) ? 1.0f : 0.0f;
        q = valid ? 1.0f : 0.0f;
    } else if (valid) {
        const uint16_t* tgt = reinterpret_cast<const uint16_t*>(a.tgt);
        const uint16_t* drf = reinterpret_cast<const uint16_t*>(a.drf);
        const RowDesc dt = load_desc_cg(&a.desc[(b * kT + s) * 2 + 0]);
        const long long tr = a.tgt_row[b] + s;
        if (tr >= 0 && tr < a.tgt_rows) {
            const uint32_t pb = tgt[tr * a.stride + tok];
            p = row_prob(dt, bf(pb), pb, (int)tok);
        }
        if (a.drf == nullptr) {
            q = 1.0f;
        } else {
            const RowDesc dd = load_desc_cg(&a.desc[(b * kT + s) * 2 + 1]);
            const long long dr = a.drf_row[b] + s;
            if (dr >= 0 && dr < a.drf_rows) {
                const uint32_t qb = drf[dr * a.stride + tok];
                q = row_prob(dd, bf(qb), qb, (int)tok);
            }
        }
    }
    return q > 0.0f && q <= 1.0f && __fmul_rn(a.u[b * (kT - 1) + s], q) < p;
}

// After this CTA wrote the outputs of a request: the CTA that finishes the last request packs
// tokens and KV slots (all threads of the CTA call it).
__device__ void finalize_request(const VerifyArgs& a, ChainSmem* sh) {
    const int tid = threadIdx.x;
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned old = atomicAdd(&a.ws->finalized, 1u);
        sh->flag = old == (unsigned)(a.B - 1);
    }
    __syncthreads();
    if (sh->flag) {
        __threadfence();
        if (a.tok_out != nullptr) compact_all_nt<kRT>(a, sh->red_a, sh->red_b);
        __syncthreads();
        if (tid == 0) a.ws->finalized = 0;
    }
    __syncthreads();
}

// After a whole row of request b (verification only; all threads): marks the row done.  The
// CTA whose row completes verify position s (its target row and, where the chain has one,
// its draft row) decides step s, or for s = cap - 1 records the last target row.  The CTA
// whose decision makes the outcome known claims the request: a greedy request is finished
// right there (returns true: this CTA wrote its outputs); a sampled one joins the ready list,
// from which its chain tasks (the bonus draw) are taken.
__device__ bool row_finish(RSmem* sh, const VerifyArgs& a, const TaskInfo& ti) {
    const int tid = threadIdx.x;
    if (a.cand == nullptr) return false;
    const int b = ti.b, s = ti.s, cap = ti.cap;
    const bool greedy = ti.cat == kGreedy;
    const bool has_d = !greedy && a.drf != nullptr && s < cap - 1;
    __syncthreads();
    if (tid == 0) {
        __threadfence();  // this row's descriptor and packed argmax before its mark
        const uint32_t bit = ti.kind == 0 ? (1u << s) : (1u << (16 + s));
        const uint32_t need = (1u << s) | (has_d ? (1u << (16 + s)) : 0u);
        const uint32_t old = atomicOr(&a.racc[2 * b], bit);
        int claim = 0;
        if (((old | bit) & need) == need && (old & need) != need) {
            __threadfence();
            const uint32_t dbit = s < cap - 1 ? (step_accepted(a, b, s, greedy) ? 1u << s : 1u << (16 + s))
                                              : kStepLast;
            const uint32_t w = atomicOr(&a.racc[2 * b + 1], dbit) | dbit;
            const int acc = outcome_of(w, cap);
            if (acc >= 0 && !(atomicOr(&a.racc[2 * b + 1], kClaimed) & kClaimed)) claim = acc + 1;
        }
        sh->fin_claim = claim;
    }
    __syncthreads();
    const int claim = sh->fin_claim;
    if (!claim || tid != 0) return claim != 0 && greedy;
    const int acc = claim - 1;
    if (greedy) {
        // the residual against a one-hot q is the same one-hot or empty (then the fallback to
        // p): the draw is the argmax of row acc unless u is outside [0, 1)
        const unsigned long long g = __ldcg(&a.gmax[b * kT + acc]);
        const long long ga = g ? (long long)(0xFFFFFFFFull - (g & 0xFFFFFFFFull)) : 0ll;
        const long long thr = scale_floor(a.uf[b], 1ull << kFixBits);
        write_request(a, b, acc, thr == -2 ? (long long)a.V - 1 : (thr < 0 ? 0ll : ga));
        return true;
    }
    __threadfence();
    const unsigned pos = atomicAdd(&a.ws->ready_tail, 1u);
    a.order[pos] = (unsigned)b + 1u;  // nonzero: published
    return false;
}

// Request index of ready-list entry qi (thread 0; waits, bounded, for the entry to be
// published), or -1 after the time limit (error bit 6).
__device__ int wait_ready(const VerifyArgs& a, int qi) {
    volatile unsigned* e = a.order + qi;
    unsigned v = *e;
    if (v == 0u) {
        const uint64_t t0 = globaltimer_ns();
        while ((v = *e) == 0u) {
            if (globaltimer_ns() - t0 > 2000000000ull) {
                atomicOr(&a.ws->err, 64u);
                return -1;
            }
            __nanosleep(256);
        }
    }
    __threadfence();
    return (int)v - 1;
}

__global__ void __launch_bounds__(kRT, DSV_ROWS_MIN_CTAS) rows_kernel(VerifyArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    RSmem* sh = reinterpret_cast<RSmem*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < kRingS; ++i) mbar_init(&sh->ring_bar[i], 1);
        for (int i = 0; i < kBigS; ++i) mbar_init(&sh->big_bar[i], 1);
        fence_mbar_init();
        sh->ring_cnt = 0;
        sh->big_cnt = 0;
#ifdef DSV_PROFILE
        for (int q = 0; q < 16; ++q) sh->prof_ph[q] = 0u;
#endif
        sh->plan = plan_at(smem_raw + sizeof(RSmem), a.B);
    }
#ifdef DSV_PROFILE
    const unsigned long long trace_t0 = globaltimer_ns();
#endif
    __syncthreads();
    build_plan(a, sh, kRWinK);
    // Task sources.  Row tasks come in plan order (positions first, see Plan).  Some rows are
    // split in two halves, up to the workspace's slot count: in verification, the rows of the
    // first kSplitPos positions (the rows most likely to decide a chain: two CTAs halve the
    // latency of their histogram pass; positions 0-2 measured 1.5% faster than 0-1 on config
    // 1), as tasks 2 r and 2 r + 1 of row r < nfront; for target
    // probabilities, the rows beyond the first wave (index >= grid), whose halves shorten the
    // tail: row task x maps to row x below the grid, to row G + (x - G) / 2, half (x - G) % 2
    // for the next 2 * nsplit tasks, and to row x - nsplit after.  After its first row a CTA
    // takes, in order: (1) a chain task of a request whose outcome is known (ncp bonus slices
    // per sampled request, from the ready list), (2) the next row task that can still change
    // an outcome (rows after a known rejection, or of a request already claimed, are dropped
    // at dequeue or abandoned during their first pass), (3) a chain task whose request is not
    // ready yet (every row has been taken by then, so it will be; the wait is bounded).
    const int nrows = total_tasks(a, sh);
    const int ncp = chain_slices(a.V);  // chain tasks per sampled request
    const int G = (int)gridDim.x;
    const bool verifying = a.cand != nullptr;
    const int nfront = (verifying && kSplitPos > 0 && a.split_cap > 0)
                           ? min((int)sh->plan.pos[kSplitPos], a.split_cap) : 0;
    const int nsplit = (!verifying && a.split_cap > 0 && nrows > G) ? min(nrows - G, a.split_cap) : 0;
    const int nrt = nrows + nfront + nsplit;
    auto row_of = [&](int x, int& half) {
        half = -1;
        if (nfront > 0) {
            if (x < 2 * nfront) {
                half = x & 1;
                return x >> 1;
            }
            return x - nfront;
        }
        if (x >= G + 2 * nsplit) return x - nsplit;
        if (x >= G) {
            half = (x - G) & 1;
            return G + (x - G) / 2;
        }
        return x;
    };
    auto slot_of = [&](int x) { return nfront > 0 ? x >> 1 : (x - G) / 2; };
    if (tid < 32) {
        int ns = 0;
        for (int b0 = 0; b0 < a.B; b0 += 32) {
            const int b = b0 + lane;
            ns += __popc(__ballot_sync(0xffffffffu, b < a.B && (sh->plan.req[b] & 7u) != (unsigned)kGreedy));
        }
        if (lane == 0) {
            sh->q_nchain = a.cand != nullptr ? ns * ncp : 0;
            sh->q_sel_empty = 0;
        }
    }
    static_assert(sizeof(ChainSmem) <= sizeof(uint32_t) * kHCap && alignof(ChainSmem) <= 16,
                  "chain tasks use the histogram area");
    ChainSmem* csh = reinterpret_cast<ChainSmem*>(sh->hist);  // idle between tasks
    bool first_task = true;
    for (;;) {
        __syncthreads();
        if (tid == 0) {
            const int nchain = sh->q_nchain;
            int kind = 0, t = -1;
            auto try_chain = [&]() {
                // a chain task of a published request, claimed only below the published count
                for (int tries = 0; tries < 4; ++tries) {
                    const unsigned ready = *(volatile unsigned*)&a.ws->ready_tail * (unsigned)ncp;
                    const unsigned cn = *(volatile unsigned*)&a.ws->chain_next;
                    if (cn >= ready || cn >= (unsigned)nchain) return false;
                    if (atomicCAS(&a.ws->chain_next, cn, cn + 1u) == cn) {
                        kind = 2;
                        t = (int)cn;
                        return true;
                    }
                }
                return false;
            };
            for (;;) {
                if (nchain > 0 && try_chain()) break;
                if (sh->q_sel_empty) break;
                int x;
                if (first_task && (int)blockIdx.x < nrt) {
                    x = (int)blockIdx.x;  // the first task of CTA i is row task i
                    first_task = false;
                } else {
                    x = (int)(gridDim.x + atomicAdd(&a.ws->next, 1u));
                }
                if (x >= nrt) {
                    sh->q_sel_empty = 1;
                    break;
                }
                // the first half of a split row is always taken: its second half may have been
                // dequeued (and found needed) before this check, and it waits for the first
                int half;
                const TaskInfo ti = decode_task(a, sh, row_of(x, half));
                if (half == 0 || row_needed(a, ti.b, ti.s)) {
                    kind = 1;
                    t = x;
                    break;
                }
            }
            if (!kind) {
                // every row taken: a chain task whose request is not published yet
                if (nchain > 0) {
                    const int j = (int)atomicAdd(&a.ws->chain_next, 1u);
                    if (j < nchain) {
                        kind = 2;
                        t = j;
                    }
                }
            }
            if (kind == 2) {
                const int b = wait_ready(a, t / ncp);
                if (b < 0) kind = 3;  // gave up: the request stays unfinished (error bit 6)
                sh->q_b = b;
            }
            if (kind == 1) {
                int half;
                const TaskInfo ti = decode_task(a, sh, row_of(t, half));
                const bool watch = a.cand != nullptr && half < 0;
                sh->watch_b = watch ? ti.b : -1;
                sh->watch_s = watch ? ti.s : -1;
                sh->late_b = sh->watch_b;
                sh->late_s = sh->watch_s;
            }
            sh->abort_row = 0;
            sh->hbm_vecs = 0u;
            sh->task = t;
            sh->q_kind = kind;
        }
        __syncthreads();
        const int t = sh->task, kind = sh->q_kind;
        if (kind == 0) break;
        if (kind == 3) continue;
#ifdef DSV_PROFILE
        const unsigned long long trace_r0 = globaltimer_ns();
        int trace_cat = 8;
#endif
        bool finished;
        if (kind == 1) {
            int half;
            const int r = row_of(t, half);
            TaskInfo ti = decode_task(a, sh, r);
            ti.half = half;
            ti.slot = half >= 0 ? slot_of(t) : -1;
#ifdef DSV_PROFILE
            trace_cat = ti.cat;
#endif
            const unsigned long long nbytes = process_row(sh, a, ti);
            if (tid == 0 && nbytes) atomicAdd(&a.ws->bytes_read, nbytes);
            // an abandoned row is not done (nothing waits for it); a first half is not a row
            finished = (sh->abort_row || half == 0) ? false : row_finish(sh, a, ti);
        } else {
            finished = chain_task(a, csh, sh->q_b, t % ncp);
        }
        if (finished) finalize_request(a, csh);
#ifdef DSV_PROFILE
        // task trace: [256] entries used, [260 + 5 i] start, end, task | cat << 16 | sm << 24,
        // phases 2 | 4 << 32, phases 6 | 8 << 32 (ns; cat 8: a chain task)
        if (tid == 0) {
            const unsigned long long now = globaltimer_ns();
            const unsigned long long i = atomicAdd(a.prof + 256, 1ull);
            if (i < kTraceCap) {
                unsigned long long* e = a.prof + 260 + 5 * i;
                e[0] = trace_r0;
                e[1] = now;
                e[2] = (unsigned long long)t | ((unsigned long long)trace_cat << 16) |
                       ((unsigned long long)smid() << 24) | ((unsigned long long)blockIdx.x << 40);
                e[3] = (unsigned long long)sh->prof_ph[2] | ((unsigned long long)sh->prof_ph[4] << 32);
                e[4] = (unsigned long long)sh->prof_ph[6] | ((unsigned long long)(sh->prof_ph[7] + sh->prof_ph[8]) << 32);
            }
            for (int q = 0; q < 16; ++q) sh->prof_ph[q] = 0u;
        }
#endif
    }
#ifdef DSV_PROFILE
    if (tid == 0 && blockIdx.x < kTraceCtas) {  // per CTA: start and exit
        unsigned long long* e = a.prof + 260 + 5 * kTraceCap + 2 * blockIdx.x;
        e[0] = trace_t0;
        e[1] = globaltimer_ns();
    }
#endif
    // the last CTA out resets the counters, the ready list, the per-request progress words and
    // the split flags for the next launch
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        sh->exit_last = atomicAdd(&a.ws->exited, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (sh->exit_last) {
        __threadfence();
        const unsigned nready = *(volatile unsigned*)&a.ws->ready_tail;
        for (unsigned i = tid; i < nready && i < (unsigned)a.B; i += kRT) a.order[i] = 0u;
        if (a.cand != nullptr)
            for (int i = tid; i < 2 * a.B; i += kRT) a.racc[i] = 0u;
        for (int i = tid; i < nsplit + nfront; i += kRT) a.split_flag[i] = 0u;
        __syncthreads();
        if (tid == 0) {
            a.ws->next = 0;
            a.ws->ready_tail = 0;
            a.ws->chain_next = 0;
            a.ws->exited = 0;
        }
        __threadfence();
    }
}

int launch_rows_cta(VerifyArgs a, cudaStream_t stream) {
    // fixed state + the batch's task table; the grid fills every SM at the occupancy this size
    // allows (cached per device and size)
    const size_t smem = sizeof(RSmem) + plan_bytes(a.B);
    constexpr int kMaxDev = 64;
    struct Cache {
        bool attr;
        size_t smem;
        int blocks;
    };
    static Cache cache[kMaxDev] = {};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return kLaunchFailed;
    int blocks = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        Cache& c = cache[dev];
        if (!c.attr) {
            if (cudaFuncSetAttribute(rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)(sizeof(RSmem) + plan_bytes(kMaxB))) != cudaSuccess)
                return kLaunchFailed;
            c.attr = true;
        }
        if (c.smem != smem) {
            int per_sm = 0, sms = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rows_kernel, kRT, smem) != cudaSuccess ||
                per_sm < 1)
                return kLaunchFailed;
            if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
                return kLaunchFailed;
            c.smem = smem;
            c.blocks = per_sm * sms;
        }
        blocks = c.blocks;
    }
    rows_kernel<<<blocks, kRT, smem, stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}


// ---------------------------------------------------------------------------------------
// dense target probabilities from the row descriptors (runtime/worker.py:440-508 output)

constexpr int kPW = 256;  // threads per CTA of the writer
constexpr int kPWChunk = 8192;  // elements per CTA
static_assert(kPWChunk % (8 * kPW) == 0, "whole 8-element vectors per thread");

// CTA (x, r) writes elements [8192 x, 8192 (x + 1)) of row r.  vec: the logit row and the output
// row are 16-byte aligned and V is a multiple of 8, so each thread loads its four 8-element
// vectors (16 bytes each, all four in flight) before writing any of their 32 probabilities.
__global__ void __launch_bounds__(kPW) probs_write_kernel(VerifyArgs a, float* out, bool vec) {
    const long long r = blockIdx.y;                 // row within the launch's requests
    const int b = (int)(r / a.cap_all), s = (int)(r % a.cap_all);
    const RowDesc d = a.desc[(b * kT + s) * 2 + 0];
    const long long row = b * a.row_step + s;
    const uint16_t* lr = reinterpret_cast<const uint16_t*>(a.tgt) + row * a.stride;
    float* o = out + r * (long long)a.V;
    const int i0 = blockIdx.x * kPWChunk;
    const int i1 = min(i0 + kPWChunk, a.V);
    if (vec) {
        constexpr int kVec = kPWChunk / (8 * kPW);
        uint4 x[kVec];
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
            const int i = i0 + (threadIdx.x + j * kPW) * 8;
            if (i < i1) x[j] = __ldcs(reinterpret_cast<const uint4*>(lr + i));
        }
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
            const int i = i0 + (threadIdx.x + j * kPW) * 8;
            if (i >= i1) continue;
            float pv[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const uint32_t u = half16(x[j], e);
                pv[e] = row_prob(d, bf(u), u, i + e);
            }
            float4* o4 = reinterpret_cast<float4*>(o + i);
            o4[0] = make_float4(pv[0], pv[1], pv[2], pv[3]);
            o4[1] = make_float4(pv[4], pv[5], pv[6], pv[7]);
        }
    } else {
        for (int i = i0 + threadIdx.x; i < i1; i += kPW) {
            const uint32_t u = lr[i];
            o[i] = row_prob(d, bf(u), u, i);
        }
    }
    // greedy rows packed their first argmax for the chain step; clear it for the next launch
    if (blockIdx.x == 0 && threadIdx.x == 0 && (d.flags & kDescGreedy)) a.gmax[b * kT + s] = 0ull;
}

int launch_target_probs(VerifyArgs a, float* out, cudaStream_t stream) {
    const int st_ = launch_rows_cta(a, stream);
    if (st_ != kOk) return st_;
    const dim3 grid((unsigned)((a.V + kPWChunk - 1) / kPWChunk), (unsigned)(a.B * a.cap_all));
    const bool vec = (a.V % 8 == 0) && (a.stride % 8 == 0) &&
                     ((reinterpret_cast<uintptr_t>(a.tgt) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0;
    probs_write_kernel<<<grid, kPW, 0, stream>>>(a, out, vec);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

}  // namespace st

bool stream_supported(const VerifyArgs& a, int dtype) {
    if (dtype != 0) return false;
    if (a.B > st::kMaxB || a.desc == nullptr || a.gmax == nullptr) return false;
    if ((reinterpret_cast<uintptr_t>(a.tgt) & 1u) || (a.drf && (reinterpret_cast<uintptr_t>(a.drf) & 1u)))
        return false;
    return a.V <= st::kMaxV;
}

int launch_target_probs(VerifyArgs a, float* out, cudaStream_t stream) {
    return st::launch_target_probs(a, out, stream);
}

int launch_stream(VerifyArgs a, cudaStream_t stream) {
    return st::launch_rows_cta(a, stream);  // rows and chain tasks in one persistent launch
}

}  // namespace dsv
