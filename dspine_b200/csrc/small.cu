// small.cu -- the per-request (not per-logit) steps around verification (sm_100a).
//
//   greedy_kernel    capped greedy accept from target top-1 ids
//                    (verification/caps.py:32-59 _accept_capped, verification/ragged.py:51-76)
//   uniforms_kernel  request-seeded uniforms: MurmurHash3 (x86_32) mixing of the seed's two
//                    32-bit halves, the position and (column + stream << 16), finalised with
//                    fmix32(h ^ 16), value = (bits >> 8) * 2^-24
//                    (sampling/random.py:22-91 seeded_uniforms / _cpu_uniforms)
//   sps_kernel       SPS verify lengths: conditional acceptance per (request, depth) from a bin
//                    table, survival = cumulative product then running minimum, stable
//                    descending rank of all B x 15 survivals, lens = 1 + selected per request,
//                    plus qo_indptr and the token index (verification/sps.py:27-58)
//   compact_kernel   accept-compact of tokens and KV slots by the exclusive scan of commit
//                    (SGLang's _commit_accept, wrapped at runtime/worker.py:745-777)
//   adjust_kernel    in-place logit adjustments: penalties, grammar bitmask, logit bias
//                    (sampling/compact.py:14-79 adjust_logits), one pass over the rows
//
// Every kernel is small (B requests, at most a few thousand entries); the cost is launch
// latency, so each is one launch with no host synchronisation.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "dsv_common.cuh"
#include "dsv_kernels.h"

namespace dsv {
namespace sm {

constexpr int kT = 16;  // draft block: anchor + 15 drafts

__device__ __forceinline__ int clamp_cap(int c) { return c < 1 ? 1 : (c > kT ? kT : c); }

__global__ void greedy_kernel(int B, const int64_t* __restrict__ cand, const int64_t* __restrict__ top1,
                              long long top1_stride, const int32_t* __restrict__ caps,
                              const int32_t* __restrict__ prefix, int32_t* accept, int32_t* commit,
                              int64_t* bonus, int64_t* output, int32_t* new_seq) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    const int cap = clamp_cap(caps[b]);
    const int64_t* c = cand + (int64_t)b * kT;
    const int64_t* t = top1 + (int64_t)b * kT * top1_stride;
    int a = cap - 1;
    for (int i = 0; i < cap - 1; ++i)
        if (c[i + 1] != t[i * top1_stride]) {
            a = i;
            break;
        }
    const int64_t bo = t[a * top1_stride];
    accept[b] = a;
    commit[b] = a + 1;
    bonus[b] = bo;
    for (int i = 0; i < kT; ++i) output[(int64_t)b * kT + i] = (i == a) ? bo : (i < kT - 1 ? c[i + 1] : 0);
    new_seq[b] = prefix[b] + a + 1;
}

__device__ __forceinline__ uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

__device__ __forceinline__ uint32_t murmur_block(uint32_t h, uint32_t k) {
    k *= 0xCC9E2D51u;
    k = rotl32(k, 15);
    k *= 0x1B873593u;
    h ^= k;
    h = rotl32(h, 13);
    return h * 5u + 0xE6546B64u;
}

__device__ __forceinline__ uint32_t fmix32(uint32_t h) {
    h ^= h >> 16;
    h *= 0x85EBCA6Bu;
    h ^= h >> 13;
    h *= 0xC2B2AE35u;
    h ^= h >> 16;
    return h;
}

template <typename PosT>
__global__ void uniforms_kernel(int n, int width, const int64_t* __restrict__ seeds,
                                const PosT* __restrict__ positions, uint32_t stream, float* out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)n * width) return;
    const int r = (int)(i / width), col = (int)(i % width);
    const uint64_t s = (uint64_t)seeds[r];
    uint32_t h = 0;
    h = murmur_block(h, (uint32_t)(s & 0xFFFFFFFFu));
    h = murmur_block(h, (uint32_t)(s >> 32));
    h = murmur_block(h, (uint32_t)((uint64_t)(int64_t)positions[r] & 0xFFFFFFFFu));
    h = murmur_block(h, (uint32_t)col + (stream << 16));
    const uint32_t bits = fmix32(h ^ 16u);
    out[i] = (float)(bits >> 8) * 5.9604644775390625e-08f;  // 2^-24
}

constexpr int kSpsThreads = 1024;
constexpr int kSpsMaxB = 1024;
constexpr int kSpsG = kT - 1;                  // drafted depths per request
constexpr int kSpsSort = 16384;                // >= kSpsMaxB * kSpsG, power of two

// one CTA: survivals -> stable descending order -> lens, qo_indptr, index
__global__ void __launch_bounds__(kSpsThreads, 1)
    sps_kernel(int B, const float* __restrict__ raw, const float* __restrict__ table, int nbins,
               const float* __restrict__ bounds, int nbound, int budget, int32_t* lens,
               int64_t* qo, int64_t* index) {
    extern __shared__ uint64_t keys[];         // [kSpsSort]: (~survival bits) << 32 | d * B + b
    __shared__ int32_t cnt[kSpsMaxB];
    __shared__ int64_t scan[kSpsThreads];
    const int tid = threadIdx.x;
    const int n = B * kSpsG;
    int sort_n = 1;
    while (sort_n < n) sort_n <<= 1;
    for (int b = tid; b < B; b += kSpsThreads) {
        // survival of request b at every depth, position-major index d * B + b
        double run = 1.0;
        float mn = INFINITY;
        for (int d = 0; d < kSpsG; ++d) {
            const float x = raw[b * kSpsG + d];
            int bin;
            if (bounds) {
                bin = 0;
                while (bin < nbound && bounds[bin] < x) ++bin;
            } else {
                const float sc = x * (float)nbins;
                long long t = (sc != sc) ? 0 : (long long)sc;
                if (sc != sc) t = 0;
                t = t < 0 ? 0 : (t > nbins - 1 ? nbins - 1 : t);
                bin = (int)t;
            }
            const float cond = table[d * nbins + bin];
            run = (d == 0) ? (double)cond : run * (double)cond;
            const float pre = (float)run;
            mn = (d == 0 || pre < mn) ? pre : mn;
            // survival is >= 0: its float bits order like the value; descending -> complement
            const uint32_t okey = 0xFFFFFFFFu - __float_as_uint(mn);
            keys[d * B + b] = ((uint64_t)okey << 32) | (uint32_t)(d * B + b);
        }
        cnt[b] = 1;
    }
    for (int i = n + tid; i < sort_n; i += kSpsThreads) keys[i] = ~0ull;
    __syncthreads();
    // bitonic sort, ascending
    for (int size = 2; size <= sort_n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < sort_n; i += kSpsThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool up = (i & size) == 0;
                    const uint64_t a = keys[i], c = keys[j];
                    if ((a > c) == up) {
                        keys[i] = c;
                        keys[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int j = tid; j < budget - B; j += kSpsThreads) {
        const uint32_t idx = (uint32_t)keys[j];
        atomicAdd(&cnt[idx % B], 1);
    }
    __syncthreads();
    // exclusive scan of lens -> qo (B <= 1024: one entry per thread)
    const int64_t my = tid < B ? cnt[tid] : 0;
    scan[tid] = my;
    __syncthreads();
    for (int o = 1; o < kSpsThreads; o <<= 1) {
        const int64_t v = tid >= o ? scan[tid - o] : 0;
        __syncthreads();
        scan[tid] += v;
        __syncthreads();
    }
    if (tid < B) {
        lens[tid] = (int32_t)my;
        const int64_t start = scan[tid] - my;
        qo[tid + 1] = scan[tid];
        for (int t = 0; t < my; ++t) index[start + t] = (int64_t)tid * kT + t;
    }
    if (tid == 0) qo[0] = 0;
}

constexpr int kCompactThreads = 1024;

// one CTA: exclusive scans of commit and of the freed counts, then the packed copies
__global__ void __launch_bounds__(kCompactThreads, 1)
    compact_kernel(int B, const int32_t* __restrict__ commit, const int32_t* __restrict__ lens,
                   const int64_t* __restrict__ output, const int32_t* __restrict__ slots,
                   long long slots_len, const int64_t* __restrict__ slot_row, int64_t* tok_out,
                   int32_t* slot_out, int32_t* offsets, int32_t* free_out, int32_t* free_offsets,
                   unsigned int* err) {
    __shared__ int32_t sc[kCompactThreads], sf[kCompactThreads];
    __shared__ int32_t carry_c, carry_f;
    const int tid = threadIdx.x;
    if (tid == 0) {
        carry_c = 0;
        carry_f = 0;
        offsets[0] = 0;
        free_offsets[0] = 0;
    }
    __syncthreads();
    for (int base = 0; base < B; base += kCompactThreads) {
        const int b = base + tid;
        int c = 0, f = 0;
        if (b < B) {
            c = commit[b];
            f = lens[b] - c;
            f = f < 0 ? 0 : f;
        }
        sc[tid] = c;
        sf[tid] = f;
        __syncthreads();
        for (int o = 1; o < kCompactThreads; o <<= 1) {
            const int vc = tid >= o ? sc[tid - o] : 0, vf = tid >= o ? sf[tid - o] : 0;
            __syncthreads();
            sc[tid] += vc;
            sf[tid] += vf;
            __syncthreads();
        }
        if (b < B) {
            const int oc = carry_c + sc[tid] - c, of = carry_f + sf[tid] - f;
            offsets[b + 1] = oc + c;
            free_offsets[b + 1] = of + f;
            const int64_t row = slot_row[b];
            for (int i = 0; i < c; ++i) {
                tok_out[oc + i] = output[(int64_t)b * kT + i];
                const long long p = row + i;
                int32_t sl = -1;
                if (p >= 0 && p < slots_len) sl = slots[p];
                else atomicOr(err, 4u);
                slot_out[oc + i] = sl;
            }
            for (int j = 0; j < f; ++j) {
                const long long p = row + c + j;
                int32_t sl = -1;
                if (p >= 0 && p < slots_len) sl = slots[p];
                else atomicOr(err, 4u);
                free_out[of + j] = sl;
            }
        }
        __syncthreads();
        if (tid == kCompactThreads - 1) {
            carry_c += sc[tid];
            carry_f += sf[tid];
        }
        __syncthreads();
    }
}

}  // namespace sm

int launch_greedy(const GreedyArgs& g, cudaStream_t st) {
    const int threads = 128;
    sm::greedy_kernel<<<(g.B + threads - 1) / threads, threads, 0, st>>>(
        g.B, g.cand, g.top1, g.top1_stride, g.caps, g.prefix, g.accept, g.commit, g.bonus,
        g.output, g.new_seq);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

int launch_uniforms(int n, int width, const int64_t* seeds, const void* positions, int pos64,
                    int stream_id, float* out, cudaStream_t st) {
    const int64_t total = (int64_t)n * width;
    const int threads = 256;
    const unsigned blocks = (unsigned)((total + threads - 1) / threads);
    if (pos64)
        sm::uniforms_kernel<int64_t><<<blocks, threads, 0, st>>>(
            n, width, seeds, static_cast<const int64_t*>(positions), (uint32_t)stream_id, out);
    else
        sm::uniforms_kernel<int32_t><<<blocks, threads, 0, st>>>(
            n, width, seeds, static_cast<const int32_t*>(positions), (uint32_t)stream_id, out);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

int sps_max_batch() { return sm::kSpsMaxB; }

int launch_sps(int B, const float* raw, const float* table, int nbins, const float* bounds,
               int nbound, int budget, int32_t* lens, int64_t* qo, int64_t* index,
               cudaStream_t st) {
    if (cudaFuncSetAttribute(sm::sps_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             sm::kSpsSort * 8) != cudaSuccess)
        return kLaunchFailed;
    sm::sps_kernel<<<1, sm::kSpsThreads, sm::kSpsSort * 8, st>>>(B, raw, table, nbins, bounds,
                                                                 nbound, budget, lens, qo, index);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

int launch_compact(int B, const int32_t* commit, const int32_t* lens, const int64_t* output,
                   const int32_t* slots, long long slots_len, const int64_t* slot_row,
                   int64_t* tok_out, int32_t* slot_out, int32_t* offsets, int32_t* free_out,
                   int32_t* free_offsets, unsigned int* err, cudaStream_t st) {
    sm::compact_kernel<<<1, sm::kCompactThreads, 0, st>>>(B, commit, lens, output, slots, slots_len,
                                                           slot_row, tok_out, slot_out, offsets,
                                                           free_out, free_offsets, err);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

}  // namespace dsv

// ---- logit adjustments: sampling/compact.py:14-79 (adjust_logits) ------------------------------
//
// In place on bf16 or fp32 logit rows, in the reference's order: additive penalties, scaling
// penalties (l < 0 ? l * s : l / s), the grammar bitmask (bit clear: -inf), the logit bias.
// Each step rounds to the logit dtype like the torch ops it replaces (one pass over the rows).
namespace dsv {
namespace adj {

template <typename T>
__device__ __forceinline__ float ld(const T* p);
template <>
__device__ __forceinline__ float ld<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

template <typename T>
__device__ __forceinline__ float rnd(float x);
template <>
__device__ __forceinline__ float rnd<float>(float x) { return x; }
template <>
__device__ __forceinline__ float rnd<__nv_bfloat16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

template <typename T>
__device__ __forceinline__ void st(T* p, float x);
template <>
__device__ __forceinline__ void st<float>(float* p, float x) { *p = x; }
template <>
__device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }

// one element: the four steps in the reference's order, each rounded to the logit dtype
template <typename T>
__device__ __forceinline__ float adjust_one(float l, float add, float sc, bool allowed, float bias,
                                            const AdjustArgs& a) {
    if (a.additive) l = rnd<T>(__fadd_rn(l, add));
    if (a.scaling) l = rnd<T>(l < 0.0f ? __fmul_rn(l, sc) : __fdiv_rn(l, sc));
    if (a.mask && !allowed) l = -INFINITY;
    if (a.bias) l = rnd<T>(__fadd_rn(l, bias));
    return l;
}

// Thread t of CTA (x, g) owns columns [8 (256 x + t), + 8) of row group g: the request's rows
// (full blocks: rows_per_request consecutive rows) or one mapped row.  The request's penalties,
// mask bits and bias for its columns are loaded once and applied to every row of the group;
// 16-byte accesses where the row and the parameter rows allow them, element by element else.
template <typename T>
__global__ void __launch_bounds__(256) adjust_kernel(AdjustArgs a, bool vec) {
    const long long g = blockIdx.y;
    const long long r0 = a.row_to_request ? g : g * a.rows_per_request;
    const long long r1 = a.row_to_request ? g + 1
                                          : min((g + 1) * (long long)a.rows_per_request, a.rows);
    const long long req = a.row_to_request ? a.row_to_request[g] : g;
    const int c0 = (blockIdx.x * 256 + threadIdx.x) * 8;
    if (c0 >= a.V) return;
    const int n = min(8, a.V - c0);
    float add[8], sc[8], bi[8];
    bool ok[8];
    const long long pr = req * (long long)a.V + c0;
    uint32_t bits = 0xFFFFFFFFu;
    if (a.mask) {
        bits = a.mask[req * a.mask_words + (c0 >> 5)] >> (c0 & 31);  // 8 columns in one word
    }
    const bool full = vec && n == 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        add[e] = 0.0f;
        sc[e] = 1.0f;
        bi[e] = 0.0f;
        ok[e] = (bits >> e) & 1u;
    }
    if (full) {
        if (a.additive) {
            const float4 u = *reinterpret_cast<const float4*>(a.additive + pr);
            const float4 v = *reinterpret_cast<const float4*>(a.additive + pr + 4);
            add[0] = u.x; add[1] = u.y; add[2] = u.z; add[3] = u.w;
            add[4] = v.x; add[5] = v.y; add[6] = v.z; add[7] = v.w;
        }
        if (a.scaling) {
            const float4 u = *reinterpret_cast<const float4*>(a.scaling + pr);
            const float4 v = *reinterpret_cast<const float4*>(a.scaling + pr + 4);
            sc[0] = u.x; sc[1] = u.y; sc[2] = u.z; sc[3] = u.w;
            sc[4] = v.x; sc[5] = v.y; sc[6] = v.z; sc[7] = v.w;
        }
        if (a.bias) {
            const float4 u = *reinterpret_cast<const float4*>(a.bias + pr);
            const float4 v = *reinterpret_cast<const float4*>(a.bias + pr + 4);
            bi[0] = u.x; bi[1] = u.y; bi[2] = u.z; bi[3] = u.w;
            bi[4] = v.x; bi[5] = v.y; bi[6] = v.z; bi[7] = v.w;
        }
    } else {
        for (int e = 0; e < n; ++e) {
            if (a.additive) add[e] = a.additive[pr + e];
            if (a.scaling) sc[e] = a.scaling[pr + e];
            if (a.bias) bi[e] = a.bias[pr + e];
        }
    }
    for (long long r = r0; r < r1; ++r) {
        T* row = reinterpret_cast<T*>(a.logits) + r * a.stride + c0;
        if (full) {
            if (sizeof(T) == 2) {
                uint4 w = *reinterpret_cast<const uint4*>(row);
                uint32_t* h = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const uint32_t bitsv = (e & 1) ? (h[e >> 1] >> 16) : (h[e >> 1] & 0xFFFFu);
                    const float l = adjust_one<T>(__uint_as_float(bitsv << 16), add[e], sc[e], ok[e], bi[e], a);
                    const uint32_t ob = __bfloat16_as_ushort(__float2bfloat16_rn(l));
                    h[e >> 1] = (e & 1) ? ((h[e >> 1] & 0xFFFFu) | (ob << 16)) : ((h[e >> 1] & 0xFFFF0000u) | ob);
                }
                *reinterpret_cast<uint4*>(row) = w;
            } else {
                float4* rp = reinterpret_cast<float4*>(row);
                float4 u = rp[0], v = rp[1];
                float x[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) x[e] = adjust_one<T>(x[e], add[e], sc[e], ok[e], bi[e], a);
                rp[0] = make_float4(x[0], x[1], x[2], x[3]);
                rp[1] = make_float4(x[4], x[5], x[6], x[7]);
            }
        } else {
            for (int e = 0; e < n; ++e) st<T>(row + e, adjust_one<T>(ld<T>(row + e), add[e], sc[e], ok[e], bi[e], a));
        }
    }
}

}  // namespace adj

int launch_adjust(const AdjustArgs& a, int dtype, cudaStream_t st) {
    const long long groups = a.row_to_request ? a.rows
                                              : (a.rows + a.rows_per_request - 1) / a.rows_per_request;
    if (groups > 65535) {
        // more groups than a grid column holds: one launch per slice of groups
        AdjustArgs b = a;
        for (long long g0 = 0; g0 < groups; g0 += 65535) {
            const long long ng = groups - g0 < 65535 ? groups - g0 : 65535;
            const long long rpg = a.row_to_request ? 1 : a.rows_per_request;
            b.logits = static_cast<char*>(a.logits) + g0 * rpg * a.stride * (dtype == 0 ? 2 : 4);
            b.rows = (a.rows - g0 * rpg) < ng * rpg ? (a.rows - g0 * rpg) : ng * rpg;
            b.row_to_request = a.row_to_request ? a.row_to_request + g0 : nullptr;
            if (!a.row_to_request) {
                const long long off = g0 * a.V;
                b.additive = a.additive ? a.additive + off : nullptr;
                b.scaling = a.scaling ? a.scaling + off : nullptr;
                b.bias = a.bias ? a.bias + off : nullptr;
                b.mask = a.mask ? a.mask + g0 * a.mask_words : nullptr;
            }
            const int stb = launch_adjust(b, dtype, st);
            if (stb != kOk) return stb;
        }
        return kOk;
    }
    const size_t esz = dtype == 0 ? 2 : 4;
    const bool vec = (reinterpret_cast<uintptr_t>(a.logits) % 16 == 0) &&
                     ((a.stride * esz) % 16 == 0) && (a.V % 4 == 0) &&
                     (!a.additive || reinterpret_cast<uintptr_t>(a.additive) % 16 == 0) &&
                     (!a.scaling || reinterpret_cast<uintptr_t>(a.scaling) % 16 == 0) &&
                     (!a.bias || reinterpret_cast<uintptr_t>(a.bias) % 16 == 0);
    const dim3 grid((unsigned)((a.V + 2047) / 2048), (unsigned)groups);
    if (dtype == 0) adj::adjust_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(a, vec);
    else adj::adjust_kernel<float><<<grid, 256, 0, st>>>(a, vec);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

}  // namespace dsv
