// topk.cu -- ids of the k largest logits of each row, ascending by id (sm_100a).
//
// Replaces kernels/dspine.py:111-207 (_chunk_max, _select_topk, topk_ids): the reference keeps
// the max of every 64-wide chunk, takes the k chunks with the largest maxima (ties to the lower
// chunk) and the k largest elements of those k * 64 (ties to the lower id).  The k largest
// elements of a row always lie in those chunks, so the result is the row's top-k by
// (value desc, id asc); this kernel computes it in the same two stages, one CTA per row:
//
//   1. chunk maxima (all warps): 16-byte streaming vector loads (no L1 allocation; 8 bf16 /
//      fp16 or 4 fp32 values per thread, 8 vectors in flight per thread; 9% faster than
//      L1-allocating loads on 794 x 151936 bf16), a packed NaN-ignoring max per vector, the 8 or
//      16 threads of a chunk combine theirs by shuffles; kept as 64-bit keys (ordered value
//      bits << 32 | ~chunk) in shared memory;
//   2. the k chunks with the largest keys: thread t's maximum over chunks t, t + 128, ...
//      gives 128 keys whose k-th largest, L (warp 0, bit search), has at least k chunk keys at
//      or above it; every warp compacts those few keys, and warp 0 finds the k-th largest among
//      them by a bit search (one warp-wide count per bit; for bf16 the 16 widening bits of the
//      value are not searched);
//   3. candidates (all threads, every load of the row's selected chunks issued together): the
//      elements of the selected chunks whose value reaches the k-th chunk maximum (every top-k
//      element does), as keys (ordered value bits << 32 | ~id);
//   4. the k largest candidates (warp 0, the same bit search), written in ascending id order.
//
// Values compare as fp32 (bf16 / fp16 widen exactly); -0 equals +0; NaN ranks below every
// number.  One pass over each row (HBM-bound); the selection works in shared memory.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>
#include <mutex>
#include <type_traits>

#include "dsv_common.cuh"
#include "dsv_kernels.h"

namespace dsv {
namespace tk {

// Threads per CTA: 128 when the row's shared memory allows six CTAs per SM (one row each, a
// batch of rows in one wave), 256 for large k or long rows (at most two or three per SM).
constexpr int kThreadsSmall = 128;
constexpr int kThreadsLarge = 256;
constexpr size_t kSmallSmemMax = 40 * 1024;
constexpr int kChunk = 64;
constexpr int kMaxChunks = 4096;           // vocabularies up to 262144
constexpr int kMaxK = 128;                 // 64 for topk_ids, 128 for the ranked form
constexpr int kChunkBits = 12;             // chunk index < 2^12
constexpr int kIdBits = 18;                // element id < 2^18

// Dynamic shared memory: this head, then ck[nch] (chunk keys), then cand[k * 64] (compacted
// chunk keys, then candidate keys), both sized by the launch's row length and k.
struct Smem {
    unsigned long long tmax[kThreadsLarge];  // thread t: max of chunk keys t, t + NT, ...
    unsigned long long selk[kMaxK];        // the selected candidate keys
    int selc[kMaxK];                       // the selected chunks, then the selected ids
    unsigned int ncand;
    unsigned int pad[3];
};
static_assert(sizeof(Smem) % 16 == 0, "ck starts 16-byte aligned");

__host__ __device__ constexpr int chunks_of(int V) { return (V + kChunk - 1) / kChunk; }

constexpr size_t smem_bytes(int V, int k) {
    return sizeof(Smem) + ((size_t)chunks_of(V) + (size_t)k * kChunk) * sizeof(unsigned long long);
}

__device__ __forceinline__ uint32_t ordered(float v) {
    if (v != v) return 0u;                 // NaN: below -inf
    uint32_t u = __float_as_uint(v);
    if (u == 0x80000000u) u = 0u;          // -0 == +0
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <typename T> __device__ __forceinline__ float as_float(T x);
template <> __device__ __forceinline__ float as_float<float>(float x) { return x; }
template <> __device__ __forceinline__ float as_float<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float as_float<__half>(__half x) { return __half2float(x); }

// The largest value of a 16-byte vector, NaN only if every lane is NaN (NaN-ignoring max:
// __hmax2 / __hmax / fmaxf return the other operand when one is NaN).
template <typename T> __device__ __forceinline__ float vec_max(const uint4& v);
template <> __device__ __forceinline__ float vec_max<float>(const uint4& v) {
    return fmaxf(fmaxf(__uint_as_float(v.x), __uint_as_float(v.y)),
                 fmaxf(__uint_as_float(v.z), __uint_as_float(v.w)));
}
template <> __device__ __forceinline__ float vec_max<__nv_bfloat16>(const uint4& v) {
    __nv_bfloat162 a, b, c, d;
    memcpy(&a, &v.x, 4); memcpy(&b, &v.y, 4); memcpy(&c, &v.z, 4); memcpy(&d, &v.w, 4);
    const __nv_bfloat162 m = __hmax2(__hmax2(a, b), __hmax2(c, d));
    return __bfloat162float(__hmax(m.x, m.y));
}
template <> __device__ __forceinline__ float vec_max<__half>(const uint4& v) {
    __half2 a, b, c, d;
    memcpy(&a, &v.x, 4); memcpy(&b, &v.y, 4); memcpy(&c, &v.z, 4); memcpy(&d, &v.w, 4);
    const __half2 m = __hmax2(__hmax2(a, b), __hmax2(c, d));
    return __half2float(__hmax(m.x, m.y));
}

template <typename T> __device__ __forceinline__ T nan_value();
template <> __device__ __forceinline__ float nan_value<float>() { return __uint_as_float(0x7FC00000u); }
template <> __device__ __forceinline__ __nv_bfloat16 nan_value<__nv_bfloat16>() { return __ushort_as_bfloat16(0x7FC0u); }
template <> __device__ __forceinline__ __half nan_value<__half>() { return __ushort_as_half(0x7E00u); }

// The k-th largest of the n distinct 64-bit keys keys[0, n) (k <= n), by one warp: a bit
// search from the top bit, one warp-wide count per bit.  The low word of every key is ~index
// with index < 2^lowbits, so its bits 31..lowbits are set in every key and need no count.  Keys
// of value 0 (empty slots) never count.  Every lane gets the result.
// bf16: every key's high word is the ordered value of a bf16 number widened to fp32, whose low
// 16 bits are 0 (non-negative values) or all ones (negative values; NaN's key is 0), so once bits
// 63..48 are known those 16 bits follow and are not searched.
__device__ __forceinline__ unsigned long long kth_largest_warp(const unsigned long long* keys, int n,
                                                               int k, int lowbits, bool bf16 = false) {
    const int lane = threadIdx.x & 31;
    constexpr int kReg = 8;                 // up to 256 keys are held in registers
    unsigned long long held[kReg];
    const bool in_regs = n <= 32 * kReg;
    if (in_regs) {
#pragma unroll
        for (int q = 0; q < kReg; ++q) held[q] = lane + 32 * q < n ? keys[lane + 32 * q] : 0ull;
    }
    unsigned long long prefix = 0ull;
    for (int bit = 63; bit >= 0; --bit) {
        if (bf16 && bit == 47) {
            if ((prefix >> 48) != 0ull && (prefix >> 63) == 0ull) prefix |= 0xFFFFull << 32;
            bit = 32;
            continue;
        }
        if (bit == 31) {
            prefix |= 0xFFFFFFFFull & (0xFFFFFFFFull << lowbits);
            bit = lowbits;
            continue;
        }
        const unsigned long long trial = prefix | (1ull << bit);
        unsigned int c = 0;
        if (in_regs) {
#pragma unroll
            for (int q = 0; q < kReg; ++q) c += held[q] >= trial;
        } else {
            for (int i = lane; i < n; i += 32) c += keys[i] >= trial;
        }
        if (__reduce_add_sync(0xffffffffu, c) >= (unsigned int)k) prefix = trial;
    }
    return prefix;
}

// Chunk maxima of one row into ck[0, nch): thread t of the CTA handles 16-byte vectors
// t, t + NT, ... (kUnroll loads issued before any is used); the kTpc consecutive threads whose
// vectors form one chunk combine their maxima by xor-shuffles.  vec_ok: the row start and pitch
// are 16-byte aligned, so full vectors load as one uint4; the last, partial vector (and every
// vector of an unaligned row) loads element by element within the row, NaN beyond it.
template <typename T, int NT>
__device__ __forceinline__ void chunk_maxima(const T* __restrict__ row, int V, bool vec_ok,
                                             unsigned long long* ck) {
    constexpr int kE = 16 / sizeof(T);          // values per vector
    constexpr int kTpc = kChunk / kE;           // threads per chunk (8 or 16)
    constexpr int kUnroll = 8;
    const int tid = threadIdx.x;
    const int nvec = (V + kE - 1) / kE;
    const int nfull = V / kE;
    for (int j0 = 0; j0 < nvec; j0 += NT * kUnroll) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int j = j0 + u * NT + tid;
            if (vec_ok && j < nfull) {
                v[u] = __ldcs(reinterpret_cast<const uint4*>(row) + j);  // streaming: no L1 allocation
            } else {
                T e[kE];
#pragma unroll
                for (int q = 0; q < kE; ++q) {
                    const int i = j * kE + q;
                    e[q] = i < V ? row[i] : nan_value<T>();
                }
                memcpy(&v[u], e, 16);
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int j = j0 + u * NT + tid;
            uint32_t m = ordered(vec_max<T>(v[u]));
#pragma unroll
            for (int o = 1; o < kTpc; o <<= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
            const int c = j / kTpc;
            if ((tid & (kTpc - 1)) == 0 && j < nvec)
                ck[c] = ((unsigned long long)m << 32) | (0xFFFFFFFFu - (uint32_t)c);
        }
    }
}

template <typename T, int NT>
__global__ void __launch_bounds__(NT, NT == kThreadsSmall ? 6 : 3) topk_ids_kernel(const T* __restrict__ x, long long rows,
                                                            int V, long long stride, int k,
                                                            bool vec_ok, bool ranked,
                                                            int64_t* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem* sh = reinterpret_cast<Smem*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int nch = chunks_of(V);
    constexpr bool kBf16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;
    unsigned long long* ck = reinterpret_cast<unsigned long long*>(smem_raw + sizeof(Smem));
    unsigned long long* cand = ck + nch;
    for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
        const T* row = x + r * stride;
        // 1. chunk maxima
        chunk_maxima<T, NT>(row, V, vec_ok, ck);
        __syncthreads();
        {
            unsigned long long t = 0ull;
            for (int c = tid; c < nch; c += NT) t = max(t, ck[c]);
            sh->tmax[tid] = t;
        }
        __syncthreads();
        // 2. the k chunks with the largest keys (ties to the lower chunk); a row of at most k
        //    chunks (the ranked form only) keeps all of them and every element is a candidate
        const int nsel = nch < k ? nch : k;
        if (nch <= k) {
            for (int c = tid; c < nch; c += NT) sh->selc[c] = c;
            if (tid == 0) {
                sh->ncand = 0u;
                sh->tmax[0] = 0ull;
            }
        } else {
            // at least k threads hold a key >= lo, so at least k chunk keys are >= lo; the
            // search runs over those (all chunk keys when they overflow the candidate buffer),
            // compacted by every warp (order is not kept: only the set matters)
            if (wid == 0) {
                const unsigned long long lo = kth_largest_warp(sh->tmax, NT, k, kChunkBits, kBf16);
                if (lane == 0) {
                    sh->selk[0] = lo;
                    sh->ncand = 0u;
                }
            }
            __syncthreads();
            const unsigned long long lo = sh->selk[0];
            const int cap = k * kChunk;
            for (int base = wid * 32; base < nch; base += NT) {
                const int i = base + lane;
                const unsigned long long key = i < nch ? ck[i] : 0ull;
                const bool take = i < nch && key >= lo;
                const unsigned int b = __ballot_sync(0xffffffffu, take);
                unsigned int at = 0;
                if (lane == 0 && b) at = atomicAdd(&sh->ncand, (unsigned int)__popc(b));
                at = __shfl_sync(0xffffffffu, at, 0);
                const unsigned int pos = at + __popc(b & ((1u << lane) - 1u));
                if (take && pos < (unsigned int)cap) cand[pos] = key;
            }
            __syncthreads();
        }
        if (nch > k && wid == 0) {
            const int m = (int)sh->ncand;
            const unsigned long long* pool = m <= k * kChunk ? cand : ck;
            const int np = m <= k * kChunk ? m : nch;
            const unsigned long long kc = kth_largest_warp(pool, np, k, kChunkBits, kBf16);
            int s = 0;
            for (int base = 0; base < np; base += 32) {
                const int i = base + lane;
                const unsigned long long key = i < np ? pool[i] : 0ull;
                const bool take = i < np && key >= kc;
                const unsigned int b = __ballot_sync(0xffffffffu, take);
                if (take) sh->selc[s + __popc(b & ((1u << lane) - 1u))] =
                    (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
                s += __popc(b);
            }
            if (lane == 0) {
                sh->ncand = 0u;
                sh->tmax[0] = kc;                  // the k-th chunk key, for step 3
            }
        }
        __syncthreads();
        // 3. candidates: elements of the selected chunks that reach the k-th chunk maximum.
        //    Element e of the nsel chunks (chunk s = e / 64) goes to thread e % NT, kCU of
        //    them per thread whose loads issue together (a row's candidates in one round trip).
        const uint32_t vmin = (uint32_t)(sh->tmax[0] >> 32);
        constexpr int kCU = 8;
        for (int e0 = 0; e0 < nsel * kChunk; e0 += NT * kCU) {
            T raw[kCU];
#pragma unroll
            for (int u = 0; u < kCU; ++u) {
                const int e = e0 + u * NT + tid;
                const int i = e < nsel * kChunk ? sh->selc[e / kChunk] * kChunk + (e % kChunk) : V;
                if (i < V) raw[u] = row[i];
            }
#pragma unroll
            for (int u = 0; u < kCU; ++u) {
                const int e = e0 + u * NT + tid;
                const int i = e < nsel * kChunk ? sh->selc[e / kChunk] * kChunk + (e % kChunk) : V;
                const uint32_t key = i < V ? ordered(as_float<T>(raw[u])) : 0u;
                const bool take = i < V && key >= vmin;
                const unsigned int m = __ballot_sync(0xffffffffu, take);
                unsigned int base = 0;
                if (lane == 0 && m) base = atomicAdd(&sh->ncand, (unsigned int)__popc(m));
                base = __shfl_sync(0xffffffffu, base, 0);
                if (take) {
                    const unsigned int pos = base + __popc(m & ((1u << lane) - 1u));
                    cand[pos] = ((unsigned long long)key << 32) | (0xFFFFFFFFu - (uint32_t)i);
                }
            }
        }
        __syncthreads();
        // 4. the k largest candidates, written by ascending id (ranked: by descending key,
        //    i.e. value desc, id asc)
        if (wid == 0) {
            const int n = (int)sh->ncand;
            const unsigned long long kk = kth_largest_warp(cand, n, k, kIdBits, kBf16);
            int s = 0;
            for (int base = 0; base < n; base += 32) {
                const int i = base + lane;
                const unsigned long long key = i < n ? cand[i] : 0ull;
                const bool take = i < n && key >= kk;
                const unsigned int b = __ballot_sync(0xffffffffu, take);
                if (take) sh->selk[s + __popc(b & ((1u << lane) - 1u))] = key;
                s += __popc(b);
            }
            __syncwarp();
            for (int q = lane; q < k; q += 32) {
                const unsigned long long key = sh->selk[q];
                const uint32_t low = (uint32_t)(key & 0xFFFFFFFFull);   // ~id
                int rank = 0;
                for (int j = 0; j < k; ++j)
                    rank += ranked ? sh->selk[j] > key : (uint32_t)(sh->selk[j] & 0xFFFFFFFFull) > low;
                out[r * k + rank] = (int64_t)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
            }
        }
        __syncthreads();  // shared state is reused by the next row
    }
}

}  // namespace tk

int topk_max_k() { return 64; }
int topk_ranked_max_k() { return tk::kMaxK; }
int topk_max_vocab() { return tk::kMaxChunks * tk::kChunk; }

namespace {

template <typename T, int NT>
int launch_nt(const void* logits, long long rows, int V, long long stride, int k, bool vec_ok,
              bool ranked, int64_t* out, size_t smem, cudaStream_t st) {
    // Per device: the dynamic shared memory opt-in (once, for the largest row and k) and the
    // resident CTAs for the last shared-memory size launched (re-queried when it changes).
    constexpr int kMaxDev = 64;
    struct Cache {
        bool ready;
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
        if (!c.ready) {
            if (cudaFuncSetAttribute(tk::topk_ids_kernel<T, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)tk::smem_bytes(tk::kMaxChunks * tk::kChunk, tk::kMaxK)) != cudaSuccess)
                return kLaunchFailed;
            c.ready = true;
            c.smem = 0;
        }
        if (c.smem != smem) {
            int per_sm = 0, sms = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tk::topk_ids_kernel<T, NT>, NT,
                                                              smem) != cudaSuccess ||
                cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
                per_sm < 1)
                return kLaunchFailed;
            c.smem = smem;
            c.blocks = per_sm * sms;
        }
        blocks = c.blocks;
    }
    const unsigned grid = (unsigned)(rows < blocks ? rows : blocks);
    tk::topk_ids_kernel<T, NT><<<grid, NT, smem, st>>>(static_cast<const T*>(logits), rows, V,
                                                        stride, k, vec_ok, ranked, out);
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

template <typename T>
int launch_typed(const void* logits, long long rows, int V, long long stride, int k, bool vec_ok,
                 bool ranked, int64_t* out, cudaStream_t st) {
    const size_t smem = tk::smem_bytes(V, k);
    // 128-thread CTAs where six fit an SM (794 x 151936, k = 16: 0.070 ms against 0.100 with
    // 256); 256 threads where shared memory allows only two or three (ranked top-128 of
    // 960 x 248320: 255 us against 387 with 128)
    return smem <= tk::kSmallSmemMax
               ? launch_nt<T, tk::kThreadsSmall>(logits, rows, V, stride, k, vec_ok, ranked, out, smem, st)
               : launch_nt<T, tk::kThreadsLarge>(logits, rows, V, stride, k, vec_ok, ranked, out, smem, st);
}

int launch_any(const void* logits, int dtype, long long rows, int V, long long stride, int k,
               bool ranked, int64_t* out, cudaStream_t st) {
    const size_t esz = dtype == 1 ? 4 : 2;
    const bool vec_ok = (reinterpret_cast<uintptr_t>(logits) % 16 == 0) && ((stride * esz) % 16 == 0);
    switch (dtype) {
        case 0: return launch_typed<__nv_bfloat16>(logits, rows, V, stride, k, vec_ok, ranked, out, st);
        case 1: return launch_typed<float>(logits, rows, V, stride, k, vec_ok, ranked, out, st);
        case 2: return launch_typed<__half>(logits, rows, V, stride, k, vec_ok, ranked, out, st);
        default: return kBadDtype;
    }
}

}  // namespace

int launch_topk_ids(const void* logits, int dtype, long long rows, int V, long long stride, int k,
                    int64_t* out, cudaStream_t st) {
    return launch_any(logits, dtype, rows, V, stride, k, false, out, st);
}

int launch_topk_ranked(const void* logits, int dtype, long long rows, int V, long long stride, int k,
                       int64_t* out, cudaStream_t st) {
    return launch_any(logits, dtype, rows, V, stride, k, true, out, st);
}

}  // namespace dsv
