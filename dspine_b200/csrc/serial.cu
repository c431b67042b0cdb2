// serial.cu -- the draft side of a block: the serial last-write refinement tables and chains
// that produce the draft tokens, their q rows and their confidences (sm_100a).
//
//   sample_chain_kernel  sampled chain over a K x K table (kernels/dspine.py:616-772
//                        _serial_sample_chain / serial_sample_chain): per request, row by row,
//                        softmax(table[n, sender] * inv_temp), joint top-k / top-p / min-p
//                        filter, inverse-CDF draw with u[n]; writes the token, the filtered q
//                        row that verification consumes, the pre-filter confidence
//   table_kernel         greedy refinement table (kernels/dspine.py:210-287 _serial_table /
//                        serial_table): s[j, c] = base[c] + rms * sum_r m[j, r] TG[id_c, r],
//                        best lane per sender lane j, confidence 1 / sum exp((s - best) / rms)
//   chain_kernel         greedy walk of that table (kernels/dspine.py:290-324 _serial_chain)
//
// All three are per-request or per-row work on K <= 64 candidates: the cost is launch latency
// and, for the table, reading K weight rows per drafted position.  Arithmetic is fp32 as in
// the reference (exp through expf, sigmoid as 1 / (1 + exp(-x)), IEEE division).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "dsv_common.cuh"
#include "dsv_kernels.h"

namespace dsv {
namespace ser {

constexpr int kMaxK = 64;
constexpr int kChainWarps = 4;  // requests per CTA of the sampled chain

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---- sampled chain -----------------------------------------------------------------------
//
// One warp per request; lane l holds candidates l and l + 32.  Per drafted row n:
//   p      = softmax(table[n, sender, :] * inv_temp)      (max-shifted expf, butterfly sum, IEEE /)
//   rank_c = #{d : p_d > p_c or (p_d == p_c and d < c)}   (ties to the lower lane)
//   before = exclusive prefix sum of p in rank order       (warp scan, see below)
//   keep   = rank < top_k and before <= top_p and p >= min_p * max p
//   q      = keep ? p / sum(kept p) : 0                    (butterfly sum)
//   cdf    = inclusive prefix sum of q in lane order        (warp scan)
//   choice = min(#{c : cdf_c <= u * cdf_{K-1}}, last kept lane)
// The token is cand[n, choice] (greedy requests: greedy_tok[n] with a one-hot q on the
// matching candidates); the next row's sender lane is choice in both cases.
// Summation orders (fixed, so results do not depend on timing): butterfly sums add lane
// l + 32 to lane l, then xor-shuffles 16, 8, 4, 2, 1; prefix sums are Kogge-Stone scans
// (shifts 1, 2, 4, 8, 16) over positions 0..31 and 32..63, the second half plus the total
// of the first.  The K x K block of the next row is copied to shared memory (cp.async)
// while the current row is processed, so no row waits on a dependent global load.

__device__ __forceinline__ float warp_scan(float x, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x = x + y;
    }
    return x;
}

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

size_t chain_smem_bytes(int k) { return (size_t)kChainWarps * 2 * k * k * sizeof(float); }

__global__ void __launch_bounds__(kChainWarps * 32)
    sample_chain_kernel(SampleChainArgs a) {
    extern __shared__ __align__(16) float s_tab[];   // [warp][2][K * K] table blocks
    __shared__ float s_p[kChainWarps][kMaxK];        // p by lane
    __shared__ float s_r[kChainWarps][kMaxK];        // p by rank, then its prefix sums
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x * kChainWarps + warp;
    if (b >= a.bs) return;
    const int K = a.k, KK = K * K;
    float* tb = s_tab + (size_t)warp * 2 * KK;
    float* P = s_p[warp];
    float* R = s_r[warp];
    const int64_t n0 = (int64_t)b * a.tm1;
    auto prefetch = [&](int row) {
        const float* src = a.table + (n0 + row) * KK;
        float* dst = tb + (row & 1) * KK;
        for (int i = lane; i < KK; i += 32) cp_async4(dst + i, src + i);
        cp_async_commit();
    };
    prefetch(0);
    const float inv_t = a.inv_temp[b];
    const int top_k = a.top_k[b];
    const float top_p = a.top_p[b], min_p = a.min_p[b];
    const bool greedy = a.greedy[b] != 0;
    const bool v0 = lane < K, v1 = lane + 32 < K;
    int sender = 0;
    for (int row = 0; row < a.tm1; ++row) {
        const int64_t n = n0 + row;
        // loads that do not depend on the previous draw go first
        const float un = a.u[n];
        const int64_t gtok = a.greedy_tok[n];
        const int64_t* cand = a.cand + n * K;
        const int64_t cd0 = v0 ? cand[lane] : 0, cd1 = v1 ? cand[lane + 32] : 0;
        cp_async_wait_all();
        __syncwarp();  // this row's block is visible; every lane is done with the other buffer
        if (row + 1 < a.tm1) prefetch(row + 1);
        const float* tab = tb + (row & 1) * KK + sender * K;
        const float s0 = v0 ? tab[lane] * inv_t : -INFINITY;
        const float s1 = v1 ? tab[lane + 32] * inv_t : -INFINITY;
        const float mx = warp_max(fmaxf(s0, s1));
        const float m0 = v0 ? expf(s0 - mx) : 0.0f;
        const float m1 = v1 ? expf(s1 - mx) : 0.0f;
        const float total = warp_sum(m0 + m1);
        const float p0 = m0 / total, p1 = m1 / total;
        const float pmax = warp_max(fmaxf(v0 ? p0 : -INFINITY, v1 ? p1 : -INFINITY));
        if (a.confidence && !greedy && lane == 0) a.confidence[n] = pmax;
        P[lane] = v0 ? p0 : 0.0f;
        P[lane + 32] = v1 ? p1 : 0.0f;
        __syncwarp();
        int r0 = 0, r1 = 0;
        for (int d = 0; d < K; ++d) {
            const float pd = P[d];
            r0 += (pd > p0) || (pd == p0 && d < lane);
            r1 += (pd > p1) || (pd == p1 && d < lane + 32);
        }
        // positions K..63 hold zeros; a lane's rank is < K (it never counts itself)
        R[lane] = 0.0f;
        R[lane + 32] = 0.0f;
        __syncwarp();
        if (v0) R[r0 & (kMaxK - 1)] = p0;
        if (v1) R[r1 & (kMaxK - 1)] = p1;
        __syncwarp();
        const float x0 = warp_scan(R[lane], lane);
        const float x1 = warp_scan(R[lane + 32], lane) + __shfl_sync(0xffffffffu, x0, 31);
        __syncwarp();
        R[lane] = x0;
        R[lane + 32] = x1;
        __syncwarp();
        const float b0 = r0 > 0 ? R[(r0 - 1) & (kMaxK - 1)] : 0.0f;  // mass ranked ahead
        const float b1 = r1 > 0 ? R[(r1 - 1) & (kMaxK - 1)] : 0.0f;
        const float floor_p = min_p * pmax;
        const bool k0 = v0 && r0 < top_k && b0 <= top_p && p0 >= floor_p;
        const bool k1 = v1 && r1 < top_k && b1 <= top_p && p1 >= floor_p;
        const float w0 = k0 ? p0 : 0.0f, w1 = k1 ? p1 : 0.0f;
        const float wsum = warp_sum(w0 + w1);
        const float q0 = w0 / wsum, q1 = w1 / wsum;
        const float c0 = warp_scan(v0 ? q0 : 0.0f, lane);
        const float c1 = warp_scan(v1 ? q1 : 0.0f, lane) + __shfl_sync(0xffffffffu, c0, 31);
        const float ctot = __shfl_sync(0xffffffffu, K > 32 ? c1 : c0, (K - 1) & 31);
        const float thr = un * ctot;
        const unsigned under0 = __ballot_sync(0xffffffffu, v0 && c0 <= thr);
        const unsigned under1 = __ballot_sync(0xffffffffu, v1 && c1 <= thr);
        int choice = __popc(under0) + __popc(under1);
        const unsigned kb0 = __ballot_sync(0xffffffffu, k0);
        const unsigned kb1 = __ballot_sync(0xffffffffu, k1);
        const int last = kb1 ? 32 + 31 - __clz(kb1) : (kb0 ? 31 - __clz(kb0) : 0);
        choice = min(choice, last);
        const int64_t picked = __shfl_sync(0xffffffffu, choice < 32 ? cd0 : cd1, choice & 31);
        float* qo = a.out_q + n * K;
        if (v0) qo[lane] = greedy ? (cd0 == gtok ? 1.0f : 0.0f) : q0;
        if (v1) qo[lane + 32] = greedy ? (cd1 == gtok ? 1.0f : 0.0f) : q1;
        if (lane == 0) a.out_tok[n] = greedy ? gtok : picked;
        sender = choice;
    }
    cp_async_wait_all();
}

// ---- greedy refinement table ---------------------------------------------------------------
//
// One CTA per drafted row n (request b = n / (T-1), block row r = n % (T-1), state row
// b * T + 1 + r).  Candidate lanes c < K with ids id_c = cand[n, c]; sender lanes j carry the
// anchor token on block row 0 and the previous row's candidates after it.
//   u[h]    = raw[row, h] * norm_w[h]                                  (fp32)
//   base[c] = sum_h W[id_c, h] u[h]      (W = lm_head rows by id, or candidate_head[n, c])
//   m[j, r] = sigmoid(query[row, r] + TSV[sid_j, r] + gate_b[r]) * TSV[sid_j, RK + r]
//   s[j, c] = base[c] + rms[row] * sum_r m[j, r] TG[id_c, r]
//   idx[n, j] = first c of max_c s[j, c];  conf[n, j] = 1 / sum_c exp((s[j, c] - max) / max(rms, 1e-6))
// The r sum runs in chunks of 128 columns staged in shared memory (row pitch 129 floats so the
// K candidate rows of one column sit in distinct banks); each thread owns up to 16 (j, c) pairs.
constexpr int kTabThreads = 256;
constexpr int kRChunk = 128;
constexpr int kRPitch = kRChunk + 1;
constexpr int kMaxPairs = kMaxK * kMaxK / kTabThreads;  // 16

__device__ __forceinline__ float bf(const __nv_bfloat16 x) { return __bfloat162float(x); }

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

size_t table_smem_bytes(int h, int k) {
    return (size_t)h * 4 + (size_t)2 * k * kRPitch * 4 + (size_t)k * 4 + (size_t)2 * k * 8 + 16;
}

// kP: (candidate, candidate) pairs per thread, ceil(K^2 / kTabThreads) rounded up to a power
// of two (the refinement sums stay in registers; a small K keeps the register count, and so
// the resident CTAs per SM, of a small K)
template <int kP>
__global__ void __launch_bounds__(kTabThreads, kP <= 2 ? 3 : 2)
    table_kernel(TableArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int K = a.k, H = a.h, RK = a.rk;
    float* u = reinterpret_cast<float*>(smem);               // [H]
    float* mch = u + H;                                      // [K][kRPitch]
    float* gch = mch + K * kRPitch;                          // [K][kRPitch]
    float* base = gch + K * kRPitch;                         // [K]
    int64_t* ids = reinterpret_cast<int64_t*>(base + K + (K & 1));  // [K]
    int64_t* sid = ids + K;                                  // [K]
    __shared__ int s_bad;

    const int n = blockIdx.x;
    const int tm1 = a.t - 1;
    const int b = n / tm1, r = n % tm1;
    const int64_t row = (int64_t)b * a.t + 1 + r;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) s_bad = 0;
    __syncthreads();
    if (tid < K) {
        const int64_t id = a.cand[(int64_t)n * K + tid];
        const int64_t s = r == 0 ? a.input_ids[(int64_t)b * a.t] : a.cand[(int64_t)(n - 1) * K + tid];
        ids[tid] = id;
        sid[tid] = s;
        if (id < 0 || id >= a.vocab || s < 0 || s >= a.vocab) atomicOr(&s_bad, 1);
    }
    const __nv_bfloat16* xr = a.raw + row * a.raw_stride;
    for (int h = tid; h < H; h += kTabThreads) u[h] = bf(xr[h]) * bf(a.norm_w[h]);
    __syncthreads();
    if (s_bad) {  // a candidate or sender id outside the tables: no reads, flagged outputs
        if (tid < K) {
            a.idx[(int64_t)n * K + tid] = -1;
            if (a.confidence) a.confidence[(int64_t)n * K + tid] = NAN;
        }
        return;
    }
    // base[c]: each warp takes two candidate rows at a time; every lane keeps four 16-byte
    // loads of each row in flight (the rows are gathered by id, so latency, not bandwidth,
    // bounds a row), two partial sums per row
    constexpr int kTW = kTabThreads / 32;
    for (int c0 = warp; c0 < K; c0 += 2 * kTW) {
        const int c1 = c0 + kTW;
        const __nv_bfloat16* w0 = a.head_candidates ? a.lm_w + ((int64_t)n * K + c0) * a.w_stride
                                                    : a.lm_w + ids[c0] * a.w_stride;
        const __nv_bfloat16* w1 = c1 >= K ? w0
                                  : (a.head_candidates ? a.lm_w + ((int64_t)n * K + c1) * a.w_stride
                                                       : a.lm_w + ids[c1] * a.w_stride);
        float acc0 = 0.0f, acc1 = 0.0f;
        for (int hb = lane * 8; hb < H; hb += 4 * 256) {
            uint4 x0[4], x1[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int h = hb + j * 256;
                if (h < H) {
                    x0[j] = *reinterpret_cast<const uint4*>(w0 + h);
                    x1[j] = *reinterpret_cast<const uint4*>(w1 + h);
                }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int h = hb + j * 256;
                if (h < H) {
                    const float4 ua = *reinterpret_cast<const float4*>(u + h);
                    const float4 ub = *reinterpret_cast<const float4*>(u + h + 4);
                    const float uu[8] = {ua.x, ua.y, ua.z, ua.w, ub.x, ub.y, ub.z, ub.w};
                    const __nv_bfloat162* p0 = reinterpret_cast<const __nv_bfloat162*>(&x0[j]);
                    const __nv_bfloat162* p1 = reinterpret_cast<const __nv_bfloat162*>(&x1[j]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f0 = __bfloat1622float2(p0[e]);
                        const float2 f1 = __bfloat1622float2(p1[e]);
                        acc0 = fmaf(f0.x, uu[2 * e], acc0);
                        acc0 = fmaf(f0.y, uu[2 * e + 1], acc0);
                        acc1 = fmaf(f1.x, uu[2 * e], acc1);
                        acc1 = fmaf(f1.y, uu[2 * e + 1], acc1);
                    }
                }
            }
        }
        acc0 = warp_sum(acc0);
        acc1 = warp_sum(acc1);
        if (lane == 0) {
            base[c0] = acc0;
            if (c1 < K) base[c1] = acc1;
        }
    }
    const int pairs = K * K;
    float acc[kP];
#pragma unroll
    for (int i = 0; i < kP; ++i) acc[i] = 0.0f;
    const __nv_bfloat16* q = a.query + row * a.q_stride;
    for (int r0 = 0; r0 < RK; r0 += kRChunk) {
        __syncthreads();  // previous chunk consumed
        // two columns per thread and step (4-byte loads), several steps in flight
#pragma unroll 4
        for (int e = tid; e < K * (kRChunk / 2); e += kTabThreads) {
            const int j = e / (kRChunk / 2), rr = 2 * (e % (kRChunk / 2)), col = r0 + rr;
            const __nv_bfloat16* t = a.tsv + sid[j] * (int64_t)(2 * RK);
            const float2 q2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(q + col));
            const float2 t2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(t + col));
            const float2 b2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(a.gate_b + col));
            const float2 v2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(t + RK + col));
            const float2 g2 = __bfloat1622float2(
                *reinterpret_cast<const __nv_bfloat162*>(a.tg + ids[j] * (int64_t)RK + col));
            mch[j * kRPitch + rr] = sigmoidf_((q2.x + t2.x) + b2.x) * v2.x;
            mch[j * kRPitch + rr + 1] = sigmoidf_((q2.y + t2.y) + b2.y) * v2.y;
            gch[j * kRPitch + rr] = g2.x;
            gch[j * kRPitch + rr + 1] = g2.y;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kP; ++i) {
            const int pidx = tid + i * kTabThreads;
            if (pidx < pairs) {
                const int j = pidx / K, c = pidx % K;
                const float* mr = mch + j * kRPitch;
                const float* gr = gch + c * kRPitch;
                float s = acc[i];
                for (int rr = 0; rr < kRChunk; ++rr) s = fmaf(mr[rr], gr[rr], s);
                acc[i] = s;
            }
        }
    }
    __syncthreads();
    // s[j][c] into the m area (pitch K + 1), then one warp per sender lane j
    float* sv = mch;
    const float rms = a.rms[row];
#pragma unroll
    for (int i = 0; i < kP; ++i) {
        const int pidx = tid + i * kTabThreads;
        if (pidx < pairs) {
            const int j = pidx / K, c = pidx % K;
            sv[j * (K + 1) + c] = base[c] + rms * acc[i];
        }
    }
    __syncthreads();
    const float scale = fmaxf(rms, 1e-6f);
    for (int j = warp; j < K; j += kTabThreads / 32) {
        const float* sr = sv + j * (K + 1);
        const float x0 = lane < K ? sr[lane] : -INFINITY;
        const float x1 = lane + 32 < K ? sr[lane + 32] : -INFINITY;
        const float best = warp_max(fmaxf(x0, x1));
        const unsigned at0 = __ballot_sync(0xffffffffu, lane < K && x0 == best);
        const unsigned at1 = __ballot_sync(0xffffffffu, lane + 32 < K && x1 == best);
        const int arg = at0 ? __ffs(at0) - 1 : (at1 ? 32 + __ffs(at1) - 1 : 0);
        if (lane == 0) a.idx[(int64_t)n * K + j] = arg;
        if (a.confidence) {
            const float e0 = lane < K ? expf((x0 - best) / scale) : 0.0f;
            const float e1 = lane + 32 < K ? expf((x1 - best) / scale) : 0.0f;
            const float mass = warp_sum(e0 + e1);
            if (lane == 0) a.confidence[(int64_t)n * K + j] = 1.0f / mass;
        }
    }
}

// ---- greedy chain ---------------------------------------------------------------------------
// One warp per request: the request's (T-1) x K lane table is copied to shared memory, lane 0
// walks it (j = idx[first row, lane 0], then idx[next row, j]), and the lanes gather the
// candidates (and confidences) of the walked lanes in parallel.  A lane outside [0, K)
// selects nothing (value 0), as the reference's masked selection does.
constexpr int kWalkWarps = 4;

size_t walk_smem_bytes(int tm1, int k) {
    return (size_t)kWalkWarps * ((size_t)tm1 * k * sizeof(int64_t) + (size_t)tm1 * 2 * sizeof(int32_t));
}

__global__ void __launch_bounds__(kWalkWarps * 32)
    chain_kernel(int bs, int tm1, int K, const int64_t* __restrict__ idx,
                 const int64_t* __restrict__ cand, int64_t* out,
                 const float* __restrict__ conf, float* conf_out) {
    extern __shared__ __align__(16) unsigned char s_walk[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x * kWalkWarps + warp;
    if (b >= bs) return;
    const size_t per = (size_t)tm1 * K * sizeof(int64_t) + (size_t)tm1 * 2 * sizeof(int32_t);
    int64_t* tab = reinterpret_cast<int64_t*>(s_walk + warp * per);
    int32_t* js = reinterpret_cast<int32_t*>(tab + (size_t)tm1 * K);  // walked lane per row
    int32_t* ps = js + tm1;                                           // previous lane per row
    const int64_t n0 = (int64_t)b * tm1;
    const int64_t* src = idx + n0 * K;
    for (int i = lane; i < tm1 * K; i += 32) tab[i] = src[i];
    __syncwarp();
    if (lane == 0) {
        int64_t j = tab[0], prev = 0;
        for (int r = 0; r < tm1; ++r) {
            const bool in = j >= 0 && j < K;
            js[r] = in ? (int32_t)j : -1;
            ps[r] = (prev >= 0 && prev < K) ? (int32_t)prev : -1;
            prev = j;
            j = (r + 1 < tm1 && in) ? tab[(size_t)(r + 1) * K + j] : 0;
        }
    }
    __syncwarp();
    for (int r = lane; r < tm1; r += 32) {
        const int64_t n = n0 + r;
        out[n] = js[r] >= 0 ? cand[n * K + js[r]] : 0;
        if (conf) conf_out[n] = ps[r] >= 0 ? conf[n * K + ps[r]] : 0.0f;
    }
}

}  // namespace ser

int launch_sample_chain(const SampleChainArgs& a, cudaStream_t st) {
    const unsigned blocks = (unsigned)((a.bs + ser::kChainWarps - 1) / ser::kChainWarps);
    const size_t smem = ser::chain_smem_bytes(a.k);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(ser::sample_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return kLaunchFailed;
    ser::sample_chain_kernel<<<blocks, ser::kChainWarps * 32, smem, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

int serial_max_k() { return ser::kMaxK; }

size_t serial_table_smem(int h, int k) { return ser::table_smem_bytes(h, k); }

namespace {
template <int kP>
int launch_table_p(const TableArgs& a, size_t smem, cudaStream_t st) {
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(ser::table_kernel<kP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return kLaunchFailed;
    ser::table_kernel<kP><<<(unsigned)a.n, ser::kTabThreads, smem, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}
}  // namespace

int launch_serial_table(const TableArgs& a, cudaStream_t st) {
    const size_t smem = ser::table_smem_bytes(a.h, a.k);
    const int pairs = a.k * a.k;
    static_assert(ser::kMaxPairs == 16, "pair classes 1, 2, 4, 8, 16");
    if (pairs <= ser::kTabThreads) return launch_table_p<1>(a, smem, st);
    if (pairs <= 2 * ser::kTabThreads) return launch_table_p<2>(a, smem, st);
    if (pairs <= 4 * ser::kTabThreads) return launch_table_p<4>(a, smem, st);
    if (pairs <= 8 * ser::kTabThreads) return launch_table_p<8>(a, smem, st);
    return launch_table_p<16>(a, smem, st);
}

size_t serial_chain_smem(int tm1, int k) { return ser::walk_smem_bytes(tm1, k); }

int launch_serial_chain(int bs, int tm1, int k, const int64_t* idx, const int64_t* cand,
                        int64_t* out, const float* conf, float* conf_out, cudaStream_t st) {
    const size_t smem = ser::walk_smem_bytes(tm1, k);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(ser::chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return kLaunchFailed;
    const unsigned blocks = (unsigned)((bs + ser::kWalkWarps - 1) / ser::kWalkWarps);
    ser::chain_kernel<<<blocks, ser::kWalkWarps * 32, smem, st>>>(bs, tm1, k, idx, cand, out, conf,
                                                                 conf_out);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

}  // namespace dsv
