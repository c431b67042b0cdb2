/*
 * dsv_oracle.c -- CPU restatement of the DSpine draft-block verification path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA product (see dsv_oracle.h).  Compiled
 * with -ffp-contract=off so every fp32 operation below rounds exactly once, as written.
 *
 * The arithmetic rules that make results independent of reduction order:
 *   fix(x)   = round-half-even(min(x,1) * 2^40) for x > 0, else 0          (exact integer)
 *   exp2(y)  = or_exp2 (Cody-Waite split y = n + f, |f| <= 1/2, Horner degree 6)
 *   e_i      = exp2((l_i - m) * (log2(e) / T))                              (fp32 ops)
 *   sums     = integer sums of fix(.) ; comparisons against u * S are exact (128-bit)
 */
#include "dsv_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint32_t bits_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* log2(e) rounded to fp32 */
#define LOG2E_BITS 0x3FB8AA3Bu
/* 2^f ~ 1 + f*(C1 + f*(C2 + ... + f*C6)) on |f| <= 1/2: weighted least-squares fit iterated
 * toward equal ripple of the relative error (fit done for this project; < 1 ulp in fp32
 * Horner form). */
#define C1_BITS 0x3f317218u
#define C2_BITS 0x3e75fdeeu
#define C3_BITS 0x3d635774u
#define C4_BITS 0x3c1d96a6u
#define C5_BITS 0x3aaf9f2bu
#define C6_BITS 0x3920fddcu

float or_exp2(float y) {
    if (!(y >= -125.0f)) return 0.0f;
    const float magic = 12582912.0f; /* 1.5 * 2^23 */
    float t = y + magic;
    int32_t n = (int32_t)(bits_of(t) - 0x4B400000u);
    float f = y - (t - magic);
    float p = from_bits(C6_BITS);
    p = fmaf(p, f, from_bits(C5_BITS));
    p = fmaf(p, f, from_bits(C4_BITS));
    p = fmaf(p, f, from_bits(C3_BITS));
    p = fmaf(p, f, from_bits(C2_BITS));
    p = fmaf(p, f, from_bits(C1_BITS));
    p = fmaf(p, f, 1.0f);
    return from_bits(bits_of(p) + ((uint32_t)n << 23));
}

uint64_t or_fix(float x) {
    if (!(x > 0.0f)) return 0;
    if (x > 1.0f) x = 1.0f;
    return (uint64_t)nearbyint((double)x * 1099511627776.0 /* 2^40 */);
}

uint32_t or_key_f32(float v) {
    uint32_t u = bits_of(v);
    if (u == 0x80000000u) u = 0; /* -0 ranks with +0 */
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

int64_t or_scale_floor(float u, uint64_t m) {
    if (u != u || u >= 1.0f) return -2;
    if (u < 0.0f) return -1;
    uint32_t b = bits_of(u);
    uint32_t e = (b >> 23) & 0xFFu;
    uint64_t mant = (b & 0x7FFFFFu) | (e ? 0x800000u : 0u);
    int shift = e ? (150 - (int)e) : 149; /* u = mant * 2^-shift */
    if (shift >= 128) return 0;
    unsigned __int128 prod = (unsigned __int128)mant * m;
    return (int64_t)(prod >> shift);
}

/* ---- row processing ------------------------------------------------------------------ */

/* LSD radix sort of 64-bit keys, ascending, 16-bit digits */
static void radix_sort_u64(uint64_t* a, uint64_t* tmp, int64_t n) {
    uint32_t* cnt = (uint32_t*)malloc(65536 * sizeof(uint32_t));
    for (int pass = 0; pass < 4; ++pass) {
        int sh = pass * 16;
        memset(cnt, 0, 65536 * sizeof(uint32_t));
        for (int64_t i = 0; i < n; ++i) cnt[(a[i] >> sh) & 0xFFFF]++;
        uint32_t sum = 0;
        for (int d = 0; d < 65536; ++d) { uint32_t c = cnt[d]; cnt[d] = sum; sum += c; }
        for (int64_t i = 0; i < n; ++i) tmp[cnt[(a[i] >> sh) & 0xFFFF]++] = a[i];
        memcpy(a, tmp, (size_t)n * sizeof(uint64_t));
    }
    free(cnt);
}

static int row_is_greedy(float T, int32_t top_k, float* c_out) {
    float c = from_bits(LOG2E_BITS) / T;
    *c_out = c;
    return (top_k <= 1) || !(T > 0.0f) || !(c < INFINITY);
}

/* min-p key floor (runtime/worker.py:485-491 "p >= min_p * max p"; tests/ref_utils.py:95-105):
 * the max element has e = exp2(0) = 1, so the test is e >= min_p.  exp2 is monotone only up to
 * one-ulp ripples, so the floor is defined as the result of a bisection over the 32-bit ordered
 * keys between -inf (e = 0) and the max (e = 1): the smallest key hi with e(val(hi)) >= min_p
 * that the bisection reaches.  Every element whose key is >= the floor passes.  min_p > 1
 * passes nothing (the caller keeps at least one element). */
uint32_t or_minp_floor(float m, float c, float min_p) {
    uint32_t lo = or_key_f32(-INFINITY), hi = or_key_f32(m);
    if (!(min_p <= 1.0f)) return hi + 1u;
    while (hi - lo > 1u) {
        uint32_t mid = lo + (hi - lo) / 2u;
        uint32_t u = (mid & 0x80000000u) ? (mid & 0x7FFFFFFFu) : ~mid;
        float e = or_exp2((from_bits(u) - m) * c);
        if (e >= min_p) hi = mid; else lo = mid;
    }
    return hi;
}

int64_t or_scale_floor_exact(float u, uint64_t m, int* exact) {
    int64_t f = or_scale_floor(u, m);
    *exact = 0;
    if (f >= 0) {
        uint32_t b = bits_of(u);
        uint32_t e = (b >> 23) & 0xFFu;
        uint64_t mant = (b & 0x7FFFFFu) | (e ? 0x800000u : 0u);
        int shift = e ? (150 - (int)e) : 149;
        unsigned __int128 prod = (unsigned __int128)mant * m;
        *exact = shift >= 128 ? prod == 0 : ((prod & ((((unsigned __int128)1) << shift) - 1)) == 0);
    }
    return f;
}

/* The kept set of one row (runtime/worker.py:440-508 build_dspine_target_probs +
 * filter_target_probs; tests/ref_utils.py:79-108 ref_target_row), as a prefix of the rank order
 * (key desc, index asc) of length n:
 *   OR_JOINT  (flashinfer, min-p off for the batch): n = min(top_k, n_p), n_p = ranks whose
 *             mass ranked ahead is <= floor(top_p * S), S the whole row's mass;
 *   OR_SEQ    (flashinfer, min-p on for the batch; worker.py:485-491): top-k, then top-p
 *             against the top-k's own mass S_k (floor(top_p * S_k)), then the min-p floor;
 *   OR_TORCH  (pytorch backend, worker.py:52-67 _torch_backend_filtered_probs): the joint
 *             top-k / top-p set, then the min-p floor.
 * min_p <= 0 switches the floor off.  At least one element is kept. */
void or_process_row_ex(const float* l, int32_t V, float T, int32_t top_k, float top_p,
                       float min_p, int32_t mode, or_row_desc* d) {
    memset(d, 0, sizeof(*d));
    int32_t g = 0;
    float m = l[0];
    for (int32_t i = 1; i < V; ++i)
        if (l[i] > m) { m = l[i]; g = i; }
    d->argmax = g;
    d->m = m;
    float c;
    d->greedy = row_is_greedy(T, top_k, &c);
    d->c = c;
    if (d->greedy) {
        d->kstar = or_key_f32(m);
        d->tie_cut = g;
        d->n_kept = 1;
        d->s_total = d->s_kept = (uint64_t)1 << OR_FIX_BITS;
        d->inv_s = 1.0f;
        return;
    }
    uint64_t* F = (uint64_t*)malloc((size_t)V * sizeof(uint64_t));
    uint64_t* ck = (uint64_t*)malloc((size_t)V * sizeof(uint64_t));
    uint64_t* tmp = (uint64_t*)malloc((size_t)V * sizeof(uint64_t));
    uint64_t S = 0;
    for (int32_t i = 0; i < V; ++i) {
        float y = (l[i] - m) * c;
        F[i] = or_fix(or_exp2(y));
        S += F[i];
        /* ascending sort of ~composite = descending by (key, -index) */
        uint64_t comp = ((uint64_t)or_key_f32(l[i]) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)i);
        ck[i] = ~comp;
    }
    radix_sort_u64(ck, tmp, V);
#define RANK_IDX(r) ((int32_t)(0xFFFFFFFFu - (uint32_t)(~ck[r] & 0xFFFFFFFFu)))
#define RANK_KEY(r) ((uint32_t)(~ck[r] >> 32))
    int32_t n = (top_k >= V) ? V : top_k;
    if (top_p < 1.0f) {
        uint64_t base = S;
        if (mode == OR_SEQ && n >= 1 && n < V) {
            base = 0;
            for (int32_t r = 0; r < n; ++r) base += F[RANK_IDX(r)];
        }
        int64_t thr = or_scale_floor(top_p, base);
        uint64_t A = 0;
        int32_t np = 0;
        for (int32_t r = 0; r < V; ++r) {
            if ((int64_t)A <= thr) np = r + 1; else break;
            A += F[RANK_IDX(r)];
        }
        if (np < n) n = np;
    }
    if (mode != OR_JOINT && min_p > 0.0f) {
        uint32_t kf = or_minp_floor(m, c, min_p);
        int32_t nm = 0;
        while (nm < V && RANK_KEY(nm) >= kf) ++nm;
        if (nm < n) n = nm;
    }
    if (n < 1) n = 1;
    uint64_t SK = 0;
    int32_t last = 0;
    for (int32_t r = 0; r < n; ++r) {
        int32_t idx = RANK_IDX(r);
        SK += F[idx];
        last = idx;
    }
#undef RANK_IDX
#undef RANK_KEY
    d->kstar = or_key_f32(l[last]);
    d->tie_cut = last;
    d->n_kept = n;
    d->s_total = S;
    d->s_kept = SK;
    if (SK == 0) {
        d->inv_s = 0.0f;
    } else {
        float sf = (float)(int64_t)SK * 9.094947017729282e-13f; /* 2^-40 */
        d->inv_s = 1.0f / sf;
    }
    free(F);
    free(ck);
    free(tmp);
}

void or_process_row(const float* l, int32_t V, float T, int32_t top_k, float top_p,
                    or_row_desc* d) {
    or_process_row_ex(l, V, T, top_k, top_p, 0.0f, OR_JOINT, d);
}

float or_row_prob(const float* l, const or_row_desc* d, int32_t i) {
    if (d->greedy) return i == d->argmax ? 1.0f : 0.0f;
    uint32_t k = or_key_f32(l[i]);
    int kept = (k > d->kstar) || (k == d->kstar && i <= d->tie_cut);
    if (!kept) return 0.0f;
    float e = or_exp2((l[i] - d->m) * d->c);
    return e * d->inv_s;
}

void or_target_probs_ex(const float* logits, int64_t rows, int32_t V, int32_t rpr,
                        const float* temperature, const int32_t* top_k, const float* top_p,
                        const float* min_p, int32_t mode, float* out, int32_t nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int64_t r = 0; r < rows; ++r) {
        int64_t b = r / rpr;
        const float* l = logits + r * (int64_t)V;
        or_row_desc d;
        or_process_row_ex(l, V, temperature[b], top_k[b], top_p[b], min_p ? min_p[b] : 0.0f,
                          mode, &d);
        for (int32_t i = 0; i < V; ++i) out[r * (int64_t)V + i] = or_row_prob(l, &d, i);
    }
}

void or_target_probs(const float* logits, int64_t rows, int32_t V, int32_t rpr,
                     const float* temperature, const int32_t* top_k, const float* top_p,
                     float* out, int32_t nthreads) {
    or_target_probs_ex(logits, rows, V, rpr, temperature, top_k, top_p, NULL, OR_JOINT, out,
                       nthreads);
}

/* ---- small-support joint target (build_sparse_target) ---------------------------------- */

/* build_sparse_target (sampling/sparse/target.py:95-178; its CPU branch :156-178 is the
 * definition, _pack_joint :23-53 and _overflow_dense :56-76 the CUDA branch), one row at a
 * time over rows of logits:
 *   threshold = the k-th largest p (k = top_k, ties kept: every p >= threshold passes);
 *   nucleus   = the mass of strictly larger p is < top_p (or top_p >= 1);
 *   kept      = p > 0 and both tests.  count > capacity: overflow, and the dense row holds
 *               p >= threshold renormalised (no nucleus test is needed there: a (capacity+1)-th
 *               kept element ties the k-th, so every p >= threshold is in the nucleus);
 *               otherwise the kept ids ascending with p / (kept mass).
 * Canonical arithmetic: p ~ e_i = exp2((l_i - m) c); "strictly larger p" = larger key; masses
 * are exact fixed-point sums; "mass < top_p" is H < top_p * S exactly.  A row with temperature
 * <= 0 is one-hot at its first argmax (the reference gates greedy batches away).
 * Outputs per row r: ids [r, capacity] i32 (-1 padded), values f32 (0 padded), lengths
 * (min(count, capacity)), overflow (0/1); dense[r, :] is written for overflow rows only. */
void or_sparse_target(const float* logits, int64_t rows, int32_t V, const float* temperature,
                      const int32_t* top_k, const float* top_p, int32_t capacity, int32_t* ids,
                      float* values, int32_t* lengths, int32_t* overflow, float* dense,
                      int32_t nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int64_t r = 0; r < rows; ++r) {
        const float* l = logits + r * (int64_t)V;
        int32_t* rid = ids + r * (int64_t)capacity;
        float* rval = values + r * (int64_t)capacity;
        for (int32_t j = 0; j < capacity; ++j) { rid[j] = -1; rval[j] = 0.0f; }
        int32_t g = 0;
        float m = l[0];
        for (int32_t i = 1; i < V; ++i)
            if (l[i] > m) { m = l[i]; g = i; }
        float c = from_bits(LOG2E_BITS) / temperature[r];
        if (!(temperature[r] > 0.0f) || !(c < INFINITY)) {
            rid[0] = g;
            rval[0] = 1.0f;
            lengths[r] = 1;
            overflow[r] = 0;
            continue;
        }
        uint64_t* F = (uint64_t*)malloc((size_t)V * sizeof(uint64_t));
        float* e = (float*)malloc((size_t)V * sizeof(float));
        uint64_t* ck = (uint64_t*)malloc((size_t)V * sizeof(uint64_t));
        uint64_t* tmp = (uint64_t*)malloc((size_t)V * sizeof(uint64_t));
        uint64_t S = 0;
        for (int32_t i = 0; i < V; ++i) {
            e[i] = or_exp2((l[i] - m) * c);
            F[i] = or_fix(e[i]);
            S += F[i];
            uint64_t comp = ((uint64_t)or_key_f32(l[i]) << 32) | (uint64_t)(0xFFFFFFFFu - (uint32_t)i);
            ck[i] = ~comp;
        }
        radix_sort_u64(ck, tmp, V);
        int32_t k = top_k[r] < 1 ? 1 : (top_k[r] > V ? V : top_k[r]);
        uint32_t thr_key = (uint32_t)(~ck[k - 1] >> 32);
        int exact = 0;
        int64_t pf = or_scale_floor_exact(top_p[r], S, &exact);
        /* H < top_p * S  <=>  H <= floor - (exact ? 1 : 0);  pf == -2: top_p >= 1 (or NaN) */
        int use_p = !(top_p[r] >= 1.0f);
        int64_t hmax = pf >= 0 ? pf - (exact ? 1 : 0) : -1;
        uint64_t H = 0, Sk = 0, Sthr = 0;
        int32_t count = 0;
        uint32_t prev_key = 0xFFFFFFFFu;
        uint64_t run = 0; /* mass of keys strictly above the current key */
        for (int32_t rk = 0; rk < V; ++rk) {
            uint32_t key = (uint32_t)(~ck[rk] >> 32);
            int32_t idx = (int32_t)(0xFFFFFFFFu - (uint32_t)(~ck[rk] & 0xFFFFFFFFu));
            if (key < thr_key) break;
            if (key != prev_key) { H = run; prev_key = key; }
            run += F[idx];
            Sthr += F[idx];
            int nucleus = !use_p || (pf != -2 && (int64_t)H <= hmax);
            if (e[idx] > 0.0f && nucleus) { ++count; Sk += F[idx]; }
        }
        overflow[r] = count > capacity;
        lengths[r] = count < capacity ? count : capacity;
        if (count > capacity) {
            float inv = Sthr ? 1.0f / ((float)(int64_t)Sthr * 9.094947017729282e-13f) : 0.0f;
            float* d = dense + r * (int64_t)V;
            for (int32_t i = 0; i < V; ++i)
                d[i] = or_key_f32(l[i]) >= thr_key ? e[i] * inv : 0.0f;
        } else if (count > 0) {
            float inv = Sk ? 1.0f / ((float)(int64_t)Sk * 9.094947017729282e-13f) : 0.0f;
            /* kept ids ascending: every kept element has key >= thr_key, and its key's mass
             * ranked above passes the nucleus test */
            int32_t n = 0;
            for (int32_t i = 0; i < V && n < count; ++i) {
                uint32_t key = or_key_f32(l[i]);
                if (key < thr_key || !(e[i] > 0.0f)) continue;
                uint64_t Hk = 0;
                if (use_p) {
                    for (int32_t j = 0; j < V; ++j)
                        if (or_key_f32(l[j]) > key) Hk += F[j];
                    if (!(pf != -2 && (int64_t)Hk <= hmax)) continue;
                }
                rid[n] = i;
                rval[n] = e[i] * inv;
                ++n;
            }
        }
        free(F);
        free(e);
        free(ck);
        free(tmp);
    }
}

/* ---- residual draw --------------------------------------------------------------------- */

/* first index whose running sum of fix(w) exceeds floor(u * total); V-1 if none.
 * w(i) is produced by the callback; the caller has already decided pure/residual. */
typedef float (*wfun)(const void* ctx, int32_t i);

static int64_t draw_from(const void* ctx, wfun w, int32_t V, float u, uint64_t* mass_out) {
    uint64_t M = 0;
    for (int32_t i = 0; i < V; ++i) M += or_fix(w(ctx, i));
    *mass_out = M;
    int64_t thr = or_scale_floor(u, M);
    if (thr == -2) return V - 1;
    uint64_t C = 0;
    for (int32_t i = 0; i < V; ++i) {
        C += or_fix(w(ctx, i));
        if ((int64_t)C > thr) return i;
    }
    return V - 1;
}

typedef struct {
    const float* p;
    const float* q;
    int pure;
} dense_ctx;

static float dense_w(const void* vctx, int32_t i) {
    const dense_ctx* c = (const dense_ctx*)vctx;
    float p = c->p[i];
    if (c->pure) return p;
    float q = c->q[i];
    float qq = (q >= 0.0f && q <= 1.0f) ? q : 0.0f;
    return fmaxf(p - qq, 0.0f);
}

/* the bonus of one request: pure draw from p, or residual (p - q)+ with fallback to p */
static int64_t bonus_dense(const float* p, const float* q, int pure, int32_t V, float u) {
    dense_ctx ctx = {p, q, pure};
    uint64_t M;
    int64_t bonus = draw_from(&ctx, dense_w, V, u, &M);
    if (!pure && M == 0) {
        ctx.pure = 1;
        bonus = draw_from(&ctx, dense_w, V, u, &M);
    }
    return bonus;
}

static void write_outputs(int32_t b, int32_t a, int64_t bonus, const int64_t* cand,
                          const int32_t* prefix, int32_t* accept, int32_t* commit,
                          int64_t* bonus_out, int64_t* output, int32_t* new_seq) {
    accept[b] = a;
    commit[b] = a + 1;
    bonus_out[b] = bonus;
    for (int i = 0; i < 16; ++i) {
        int64_t v = 0;
        if (i < a) v = cand[b * 16 + i + 1];
        else if (i == a) v = bonus;
        output[b * 16 + i] = v;
    }
    new_seq[b] = prefix[b] + a + 1;
}

static inline int32_t clamp_cap(int32_t c) { return c < 1 ? 1 : (c > 16 ? 16 : c); }

void or_chain_from_probs(int32_t B, int32_t V, const int64_t* cand, const float* target,
                         const float* draft, const int32_t* caps, const float* U,
                         const float* UF, const int32_t* prefix, int32_t* accept,
                         int32_t* commit, int64_t* bonus, int64_t* output, int32_t* new_seq) {
    for (int32_t b = 0; b < B; ++b) {
        int32_t cap = clamp_cap(caps[b]);
        int32_t a = 0;
        for (int32_t s = 0; s < cap - 1; ++s) {
            int64_t tok = cand[b * 16 + s + 1];
            float p = 0.0f, q = 0.0f;
            if (tok >= 0 && tok < V) {
                p = target[((int64_t)b * 16 + s) * V + tok];
                q = draft[((int64_t)b * 15 + s) * V + tok];
            }
            if (q > 0.0f && q <= 1.0f && U[b * 15 + s] * q < p) ++a; else break;
        }
        int pure = (a == cap - 1);
        const float* prow = target + ((int64_t)b * 16 + a) * V;
        const float* qrow = pure ? NULL : draft + ((int64_t)b * 15 + a) * V;
        int64_t bo = bonus_dense(prow, qrow, pure, V, UF[b]);
        write_outputs(b, a, bo, cand, prefix, accept, commit, bonus, output, new_seq);
    }
}

/* ---- fused verification from logits ---------------------------------------------------- */

typedef struct {
    const float* lp;
    const or_row_desc* dp;
    const float* lq;       /* NULL: one-hot q */
    const or_row_desc* dq;
    int64_t onehot;        /* drafted token when lq == NULL */
    int pure;
} logit_ctx;

static float logit_w(const void* vctx, int32_t i) {
    const logit_ctx* c = (const logit_ctx*)vctx;
    float p = or_row_prob(c->lp, c->dp, i);
    if (c->pure) return p;
    float q = c->lq ? or_row_prob(c->lq, c->dq, i) : (i == c->onehot ? 1.0f : 0.0f);
    float qq = (q >= 0.0f && q <= 1.0f) ? q : 0.0f;
    return fmaxf(p - qq, 0.0f);
}

void or_verify_logits_ex(int32_t B, int32_t V, const int64_t* cand, const float* target,
                         const int64_t* tgt_row, const float* draft, const int64_t* drf_row,
                         int64_t stride, const float* temperature, const int32_t* top_k,
                         const float* top_p, const float* min_p, int32_t mode,
                         const int32_t* caps, const float* U, const float* UF,
                         const int32_t* prefix, int32_t* accept, int32_t* commit,
                         int64_t* bonus, int64_t* output, int32_t* new_seq, int32_t nthreads) {
    /* phase 1: every row descriptor a request may consult */
    or_row_desc* dt = (or_row_desc*)calloc((size_t)B * 16, sizeof(or_row_desc));
    or_row_desc* dq = (or_row_desc*)calloc((size_t)B * 16, sizeof(or_row_desc));
    int32_t ntask = B * 32;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int32_t t = 0; t < ntask; ++t) {
        int32_t b = t % B, s = (t / B) % 16, kind = t / (B * 16);
        int32_t cap = clamp_cap(caps[b]);
        float c;
        int greedy = row_is_greedy(temperature[b], top_k[b], &c);
        if (kind == 0) {
            if (s >= cap) continue;
            or_process_row_ex(target + (tgt_row[b] + s) * stride, V, temperature[b], top_k[b],
                              top_p[b], min_p ? min_p[b] : 0.0f, mode, &dt[b * 16 + s]);
        } else {
            if (s >= cap - 1 || greedy || draft == NULL) continue;
            or_process_row_ex(draft + (drf_row[b] + s) * stride, V, temperature[b], top_k[b],
                              top_p[b], min_p ? min_p[b] : 0.0f, mode, &dq[b * 16 + s]);
        }
    }
    /* phase 2: chain + bonus per request */
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1)
#endif
    for (int32_t b = 0; b < B; ++b) {
        int32_t cap = clamp_cap(caps[b]);
        float c;
        int onehot_q = row_is_greedy(temperature[b], top_k[b], &c) || draft == NULL;
        int32_t a = 0;
        for (int32_t s = 0; s < cap - 1; ++s) {
            int64_t tok = cand[b * 16 + s + 1];
            float p = 0.0f, q = 0.0f;
            if (tok >= 0 && tok < V) {
                const float* lp = target + (tgt_row[b] + s) * stride;
                p = or_row_prob(lp, &dt[b * 16 + s], (int32_t)tok);
                if (onehot_q) q = 1.0f;
                else q = or_row_prob(draft + (drf_row[b] + s) * stride, &dq[b * 16 + s], (int32_t)tok);
            }
            if (q > 0.0f && q <= 1.0f && U[b * 15 + s] * q < p) ++a; else break;
        }
        int pure = (a == cap - 1);
        logit_ctx ctx;
        ctx.lp = target + (tgt_row[b] + a) * stride;
        ctx.dp = &dt[b * 16 + a];
        ctx.lq = NULL;
        ctx.dq = NULL;
        ctx.onehot = -1;
        ctx.pure = pure;
        if (!pure) {
            if (onehot_q) {
                ctx.onehot = cand[b * 16 + a + 1];
            } else {
                ctx.lq = draft + (drf_row[b] + a) * stride;
                ctx.dq = &dq[b * 16 + a];
            }
        }
        uint64_t M;
        int64_t bo = draw_from(&ctx, logit_w, V, UF[b], &M);
        if (!pure && M == 0) {
            ctx.pure = 1;
            bo = draw_from(&ctx, logit_w, V, UF[b], &M);
        }
        write_outputs(b, a, bo, cand, prefix, accept, commit, bonus, output, new_seq);
    }
    free(dt);
    free(dq);
}

void or_verify_logits(int32_t B, int32_t V, const int64_t* cand, const float* target,
                      const int64_t* tgt_row, const float* draft, const int64_t* drf_row,
                      int64_t stride, const float* temperature, const int32_t* top_k,
                      const float* top_p, const int32_t* caps, const float* U, const float* UF,
                      const int32_t* prefix, int32_t* accept, int32_t* commit, int64_t* bonus,
                      int64_t* output, int32_t* new_seq, int32_t nthreads) {
    or_verify_logits_ex(B, V, cand, target, tgt_row, draft, drf_row, stride, temperature, top_k,
                        top_p, NULL, OR_JOINT, caps, U, UF, prefix, accept, commit, bonus, output,
                        new_seq, nthreads);
}

/* ---- sparse q (accept_sparse) ---------------------------------------------------------- */

static float q_at(const int64_t* qid, const float* qv, int64_t token, int clamp) {
    float s = 0.0f;
    for (int k = 0; k < 16; ++k) {
        if (qid[k] != token) continue;
        float v = qv[k];
        if (clamp) v = (v >= 0.0f && v <= 1.0f) ? v : 0.0f;
        s = s + v;
    }
    return s;
}

static float packed_p_at(const int32_t* ids, const float* vals, int32_t len, int32_t width,
                         int64_t token) {
    float s = 0.0f;
    for (int32_t l = 0; l < width && l < len; ++l)
        if ((int64_t)ids[l] == token) s = s + vals[l];
    return s;
}

typedef struct {
    const float* prow;     /* dense row */
    float den;
    int raw;
    const int64_t* qid;
    const float* qv;
    int pure;
} sparse_ctx;

static float sparse_dense_w(const void* vctx, int32_t i) {
    const sparse_ctx* c = (const sparse_ctx*)vctx;
    float p = c->prow ? c->prow[i] : 0.0f;
    if (c->raw) p = p / c->den;
    if (c->pure) return p;
    float q = q_at(c->qid, c->qv, i, 1);
    return fmaxf(p - q, 0.0f);
}

static int64_t packed_bonus(const int32_t* ids, const float* vals, int32_t len, int32_t width,
                            const int64_t* qid, const float* qv, int pure, int32_t V, float u) {
    int32_t n = width;
    int64_t* ord = (int64_t*)malloc((size_t)n * sizeof(int64_t));
    float* p = (float*)malloc((size_t)n * sizeof(float));
    float* r = (float*)malloc((size_t)n * sizeof(float));
    for (int32_t l = 0; l < n; ++l) ord[l] = (l < len) ? (int64_t)ids[l] : (int64_t)V;
    /* insertion sort ascending (small width) */
    for (int32_t i = 1; i < n; ++i) {
        int64_t x = ord[i];
        int32_t j = i - 1;
        while (j >= 0 && ord[j] > x) { ord[j + 1] = ord[j]; --j; }
        ord[j + 1] = x;
    }
    for (int32_t j = 0; j < n; ++j) {
        p[j] = (ord[j] < V) ? packed_p_at(ids, vals, len, width, ord[j]) : 0.0f;
        r[j] = pure ? p[j] : fmaxf(p[j] - q_at(qid, qv, ord[j], 1), 0.0f);
    }
    uint64_t M = 0;
    for (int32_t j = 0; j < n; ++j) M += or_fix(r[j]);
    if (!pure && M == 0) {
        for (int32_t j = 0; j < n; ++j) r[j] = p[j];
        for (int32_t j = 0; j < n; ++j) M += or_fix(r[j]);
    }
    int64_t res = V - 1;
    int64_t thr = or_scale_floor(u, M);
    if (thr != -2) {
        uint64_t C = 0;
        for (int32_t j = 0; j < n; ++j) {
            C += or_fix(r[j]);
            if ((int64_t)C > thr) { if (ord[j] < V) res = ord[j]; break; }
        }
    }
    free(ord);
    free(p);
    free(r);
    return res;
}

void or_accept_sparse(int32_t B, int32_t V, const int64_t* cand, const float* dense_p,
                      const int32_t* p_ids, const float* p_vals, const int32_t* p_len,
                      const int32_t* overflow, int32_t width, const int64_t* q_ids,
                      const float* q_vals, const int32_t* caps, const float* U, const float* UF,
                      const int32_t* prefix, const int64_t* row_offsets, const float* denom,
                      int32_t* accept, int32_t* commit, int64_t* bonus, int64_t* output,
                      int32_t* new_seq) {
    int packed = (p_ids != NULL);
    int raw = (denom != NULL);
    for (int32_t b = 0; b < B; ++b) {
        int64_t base = row_offsets ? row_offsets[b] : (int64_t)b * 16;
        int32_t cap = clamp_cap(caps[b]);
        int32_t a = 0;
        for (int32_t step = 1; step < cap; ++step) {
            int64_t row = base + step - 1;
            int64_t qi = (int64_t)b * 15 + step - 1;
            int64_t tok = cand[b * 16 + step];
            int dense = packed ? (overflow[row] != 0) : 1;
            float p = 0.0f;
            if (tok >= 0 && tok < V) {
                if (dense) {
                    p = dense_p ? dense_p[row * V + tok] : 0.0f;
                    if (raw) p = p / denom[row];
                } else {
                    p = packed_p_at(p_ids + row * width, p_vals + row * width, p_len[row], width, tok);
                }
            }
            float q = q_at(q_ids + qi * 16, q_vals + qi * 16, tok, 0);
            if (q > 0.0f && q <= 1.0f && U[qi] * q < p) ++a; else break;
        }
        int pure = (a == cap - 1);
        int64_t row = base + a;
        int64_t qi = (int64_t)b * 15 + a;
        int dense = packed ? (overflow[row] != 0) : 1;
        int64_t bo;
        if (packed && !dense) {
            bo = packed_bonus(p_ids + row * width, p_vals + row * width, p_len[row], width,
                              q_ids + qi * 16, q_vals + qi * 16, pure, V, UF[b]);
        } else {
            sparse_ctx ctx;
            ctx.prow = dense_p ? dense_p + row * V : NULL;
            ctx.den = raw ? denom[row] : 1.0f;
            ctx.raw = raw;
            ctx.qid = q_ids + qi * 16;
            ctx.qv = q_vals + qi * 16;
            ctx.pure = pure;
            uint64_t M;
            bo = draw_from(&ctx, sparse_dense_w, V, UF[b], &M);
            if (!pure && M == 0) {
                ctx.pure = 1;
                bo = draw_from(&ctx, sparse_dense_w, V, UF[b], &M);
            }
        }
        write_outputs(b, a, bo, cand, prefix, accept, commit, bonus, output, new_seq);
    }
}

/* ---- compress_probs -------------------------------------------------------------------- */

void or_compress_probs(const float* p, int64_t rows, int32_t V, int32_t capacity, int32_t* ids,
                       float* values, int32_t* lengths, int32_t* overflow) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* x = p + r * V;
        int32_t* oi = ids + r * capacity;
        float* ov = values + r * capacity;
        for (int32_t l = 0; l < capacity; ++l) { oi[l] = -1; ov[l] = 0.0f; }
        int64_t count = 0, bad = 0;
        for (int32_t i = 0; i < V; ++i) {
            float v = x[i];
            if (v < 0.0f || v != v || fabsf(v) == INFINITY) ++bad;
            if (v > 0.0f) {
                if (count < capacity) { oi[count] = i; ov[count] = v; }
                ++count;
            }
        }
        lengths[r] = (int32_t)(count < capacity ? count : capacity);
        overflow[r] = (count > capacity) || (bad > 0);
    }
}

/* ---- greedy ---------------------------------------------------------------------------- */

void or_accept_greedy(int32_t B, const int64_t* cand, const int64_t* top1, const int32_t* caps,
                      const int32_t* prefix, int32_t* accept, int32_t* commit, int64_t* bonus,
                      int64_t* output, int32_t* new_seq) {
    for (int32_t b = 0; b < B; ++b) {
        int32_t cap = clamp_cap(caps[b]);
        int32_t a = cap - 1;
        for (int32_t i = 0; i < 16; ++i) {
            int64_t proposed = (i < 15) ? cand[b * 16 + i + 1] : 0;
            int matched = (i < cap - 1) && (proposed == top1[b * 16 + i]);
            if (!matched) { if (i < a) a = i; break; }
        }
        int64_t bo = top1[b * 16 + a];
        accept[b] = a;
        commit[b] = a + 1;
        bonus[b] = bo;
        for (int32_t i = 0; i < 16; ++i) {
            int64_t proposed = (i < 15) ? cand[b * 16 + i + 1] : 0;
            output[b * 16 + i] = (i == a) ? bo : proposed;
        }
        new_seq[b] = prefix[b] + a + 1;
    }
}

void or_argmax_rows(const float* x, int64_t rows, int32_t V, int64_t stride, int64_t* out) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* l = x + r * stride;
        int32_t g = 0;
        float m = l[0];
        for (int32_t i = 1; i < V; ++i)
            if (l[i] > m) { m = l[i]; g = i; }
        out[r] = g;
    }
}

/* ---- top-k ----------------------------------------------------------------------------- */

/* precedes: a before b in (value desc, id asc) */
static inline int precedes(float va, int64_t ia, float vb, int64_t ib) {
    return (va > vb) || (va == vb && ia < ib);
}

void or_topk_sorted(const float* x, int64_t rows, int32_t V, int64_t stride, int32_t k,
                    float* vals, int64_t* ids) {
    for (int64_t r = 0; r < rows; ++r) {
        const float* l = x + r * stride;
        float* ov = vals + r * k;
        int64_t* oi = ids + r * k;
        int32_t n = 0;
        for (int32_t i = 0; i < V; ++i) {
            float v = l[i];
            if (v != v) continue;
            if (n == k && !precedes(v, i, ov[k - 1], oi[k - 1])) continue;
            int32_t j = (n < k) ? n++ : k - 1;
            while (j > 0 && precedes(v, i, ov[j - 1], oi[j - 1])) {
                ov[j] = ov[j - 1];
                oi[j] = oi[j - 1];
                --j;
            }
            ov[j] = v;
            oi[j] = i;
        }
        for (; n < k; ++n) { ov[n] = -INFINITY; oi[n] = -1; }
    }
}

static int cmp_i64(const void* a, const void* b) {
    int64_t x = *(const int64_t*)a, y = *(const int64_t*)b;
    return (x > y) - (x < y);
}

void or_topk_ids(const float* x, int64_t rows, int32_t V, int64_t stride, int32_t k, int64_t* out) {
    float* vals = (float*)malloc((size_t)k * sizeof(float));
    for (int64_t r = 0; r < rows; ++r) {
        or_topk_sorted(x + r * stride, 1, V, stride, k, vals, out + r * k);
        qsort(out + r * k, (size_t)k, sizeof(int64_t), cmp_i64);
    }
    free(vals);
}

/* ---- seeded uniforms ------------------------------------------------------------------- */

static inline uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

void or_uniforms(const int64_t* seeds, const int64_t* positions, int32_t n, int32_t width,
                 int32_t stream, float* out) {
    for (int32_t r = 0; r < n; ++r) {
        uint64_t s = (uint64_t)seeds[r];
        for (int32_t col = 0; col < width; ++col) {
            uint32_t blocks[4];
            blocks[0] = (uint32_t)(s & 0xFFFFFFFFu);
            blocks[1] = (uint32_t)(s >> 32);
            blocks[2] = (uint32_t)((uint64_t)positions[r] & 0xFFFFFFFFu);
            blocks[3] = (uint32_t)col + ((uint32_t)stream << 16);
            uint32_t h = 0;
            for (int j = 0; j < 4; ++j) {
                uint32_t k = blocks[j] * 0xCC9E2D51u;
                k = rotl32(k, 15);
                h ^= k * 0x1B873593u;
                h = rotl32(h, 13);
                h = h * 5u + 0xE6546B64u;
            }
            h ^= 16u;
            h ^= h >> 16;
            h *= 0x85EBCA6Bu;
            h ^= h >> 13;
            h *= 0xC2B2AE35u;
            h ^= h >> 16;
            out[(int64_t)r * width + col] = (float)(h >> 8) * 5.9604644775390625e-08f;
        }
    }
}

/* ---- SPS ------------------------------------------------------------------------------- */

typedef struct { float s; int32_t idx; } surv_t;

static int cmp_surv(const void* a, const void* b) {
    const surv_t* x = (const surv_t*)a;
    const surv_t* y = (const surv_t*)b;
    if (x->s > y->s) return -1;
    if (x->s < y->s) return 1;
    return (x->idx > y->idx) - (x->idx < y->idx);
}

void or_sps_lens(int32_t B, const float* raw, const float* table, int32_t nbins,
                 const float* boundaries, int32_t nbound, int32_t budget, int32_t* lens) {
    const int32_t G = 15;
    surv_t* sv = (surv_t*)malloc((size_t)B * G * sizeof(surv_t));
    for (int32_t b = 0; b < B; ++b) {
        /* torch.cumprod of fp32 on the host accumulates in fp64 and rounds each prefix */
        double run = 1.0;
        float mn = INFINITY;
        for (int32_t d = 0; d < G; ++d) {
            float x = raw[b * G + d];
            int64_t bin;
            if (boundaries) {
                bin = 0;
                while (bin < nbound && boundaries[bin] < x) ++bin;
            } else {
                float sc = x * (float)nbins;
                bin = (sc != sc) ? 0 : (int64_t)sc;
                if (bin < 0) bin = 0;
                if (bin > nbins - 1) bin = nbins - 1;
            }
            float cond = table[d * nbins + bin];
            run = (d == 0) ? (double)cond : run * (double)cond;
            float pre = (float)run;
            mn = (d == 0 || pre < mn) ? pre : mn;
            sv[d * B + b].s = mn;
            sv[d * B + b].idx = d * B + b;
        }
    }
    qsort(sv, (size_t)B * G, sizeof(surv_t), cmp_surv);
    for (int32_t b = 0; b < B; ++b) lens[b] = 1;
    for (int32_t j = 0; j < budget - B; ++j) lens[sv[j].idx % B] += 1;
    free(sv);
}

void or_sps_index(int32_t B, const int32_t* lens, int32_t T, int64_t* qo, int64_t* index) {
    qo[0] = 0;
    for (int32_t b = 0; b < B; ++b) qo[b + 1] = qo[b] + lens[b];
    for (int32_t b = 0; b < B; ++b)
        for (int32_t t = 0; t < lens[b]; ++t) index[qo[b] + t] = (int64_t)b * T + t;
}

/* ---- accept-compact -------------------------------------------------------------------- */

void or_accept_compact(int32_t B, const int32_t* commit, const int32_t* lens,
                       const int64_t* output, const int32_t* slots, const int64_t* slot_row,
                       int64_t* tok_out, int32_t* slot_out, int32_t* offsets, int32_t* free_out,
                       int32_t* free_offsets) {
    offsets[0] = 0;
    free_offsets[0] = 0;
    for (int32_t b = 0; b < B; ++b) {
        int32_t c = commit[b];
        int32_t f = lens[b] - c;
        if (f < 0) f = 0;
        offsets[b + 1] = offsets[b] + c;
        free_offsets[b + 1] = free_offsets[b] + f;
    }
    for (int32_t b = 0; b < B; ++b) {
        int32_t c = commit[b];
        for (int32_t i = 0; i < c; ++i) {
            tok_out[offsets[b] + i] = output[b * 16 + i];
            slot_out[offsets[b] + i] = slots[slot_row[b] + i];
        }
        int32_t f = free_offsets[b + 1] - free_offsets[b];
        for (int32_t j = 0; j < f; ++j) free_out[free_offsets[b] + j] = slots[slot_row[b] + c + j];
    }
}

/* ---- TP merge -------------------------------------------------------------------------- */

typedef struct { float v; int64_t id; int32_t pos; } cand_t;

static int cmp_cand(const void* a, const void* b) {
    const cand_t* x = (const cand_t*)a;
    const cand_t* y = (const cand_t*)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    if (x->id != y->id) return (x->id > y->id) - (x->id < y->id);
    return (x->pos > y->pos) - (x->pos < y->pos);
}

void or_merge_topk(int64_t n, int32_t m, const float* values, const int64_t* ids, int32_t k,
                   float* out_vals, int64_t* out_ids) {
    cand_t* c = (cand_t*)malloc((size_t)m * sizeof(cand_t));
    for (int64_t r = 0; r < n; ++r) {
        for (int32_t j = 0; j < m; ++j) {
            c[j].v = values[r * m + j];
            c[j].id = ids[r * m + j];
            c[j].pos = j;
        }
        qsort(c, (size_t)m, sizeof(cand_t), cmp_cand);
        for (int32_t j = 0; j < k; ++j) {
            out_vals[r * k + j] = c[j].v;
            out_ids[r * k + j] = c[j].id;
        }
    }
    free(c);
}
