// topk.cu -- ids of the k largest logits of each row, ascending by id (sm_100a).
//
// Replaces kernels/dspine.py:111-207 (_chunk_max, _select_topk, topk_ids): the reference keeps
// the max of every 64-wide chunk, takes the k chunks with the largest maxima (ties to the lower
// chunk) and the k largest elements of those k * 64 (ties to the lower id).  The k largest
// elements of a row always lie in those chunks, so the result is the row's top-k by
// (value desc, id asc); this kernel computes it in the same two stages, one CTA per row:
//
//   1. chunk maxima: one warp per chunk (lane l reads elements l and l + 32, coalesced), kept
//      as 64-bit keys (ordered value bits << 32 | ~chunk) in shared memory;
//   2. the k-th largest chunk key by a bit search (one block-wide count per bit), so the
//      selected chunks are those with keys at or above it;
//   3. candidates: the elements of the selected chunks whose value reaches the k-th chunk
//      maximum (every top-k element does), as keys (ordered value bits << 32 | ~id);
//   4. the k-th largest candidate key by the same bit search; the k candidates at or above it
//      are the answer, written in ascending id order.
//
// Values compare as fp32 (bf16 / fp16 widen exactly); -0 equals +0; NaN ranks below every
// number.  One pass over each row (HBM-bound), the selection works in shared memory.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "dsv_common.cuh"
#include "dsv_kernels.h"

namespace dsv {
namespace tk {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kChunk = 64;
constexpr int kMaxChunks = 4096;           // vocabularies up to 262144
constexpr int kMaxK = 64;
constexpr int kCandCap = kMaxK * kChunk;   // every element of the selected chunks

struct Smem {
    unsigned long long ck[kMaxChunks];     // chunk keys
    unsigned long long cand[kCandCap];     // candidate keys
    unsigned int wsum[2][kWarps];
    unsigned int ncand;
    unsigned int nsel;
    long long sel[kMaxK];
};

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

// The k-th largest of the n distinct 64-bit keys keys[0, n) (k <= n): a bit search from the top
// bit, one block-wide count per bit.  All threads call it; every thread gets the result.
__device__ unsigned long long kth_largest(const unsigned long long* keys, int n, int k, Smem* sh) {
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    unsigned long long prefix = 0ull;
    for (int bit = 63; bit >= 0; --bit) {
        const unsigned long long trial = prefix | (1ull << bit);
        unsigned int c = 0;
        for (int i = tid; i < n; i += kThreads) c += keys[i] >= trial;
        c = __reduce_add_sync(0xffffffffu, c);
        const int buf = bit & 1;            // alternate buffers: one barrier per bit
        if (lane == 0) sh->wsum[buf][wid] = c;
        __syncthreads();
        unsigned int total = 0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) total += sh->wsum[buf][w];
        if (total >= (unsigned int)k) prefix = trial;
    }
    return prefix;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) topk_ids_kernel(const T* __restrict__ x, long long rows,
                                                            int V, long long stride, int k,
                                                            int64_t* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem* sh = reinterpret_cast<Smem*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int nch = (V + kChunk - 1) / kChunk;
    for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
        const T* row = x + r * stride;
        // 1. chunk maxima
#pragma unroll 4
        for (int c = wid; c < nch; c += kWarps) {
            const int i0 = c * kChunk + lane, i1 = i0 + 32;
            uint32_t m = 0u;
            if (i0 < V) m = ordered(as_float<T>(row[i0]));
            if (i1 < V) m = max(m, ordered(as_float<T>(row[i1])));
            m = __reduce_max_sync(0xffffffffu, m);
            if (lane == 0) sh->ck[c] = ((unsigned long long)m << 32) | (0xFFFFFFFFu - (uint32_t)c);
        }
        if (tid == 0) {
            sh->ncand = 0u;
            sh->nsel = 0u;
        }
        __syncthreads();
        // 2. the k chunks with the largest maxima (ties to the lower chunk)
        const unsigned long long kc = kth_largest(sh->ck, nch, k, sh);
        const uint32_t vmin = (uint32_t)(kc >> 32);   // the k-th largest chunk maximum
        // 3. candidates: elements of the selected chunks that reach it
        for (int c = wid; c < nch; c += kWarps) {
            if (sh->ck[c] < kc) continue;             // warp-uniform
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int i = c * kChunk + lane + 32 * h;
                const uint32_t key = i < V ? ordered(as_float<T>(row[i])) : 0u;
                const bool take = i < V && key >= vmin;
                const unsigned int m = __ballot_sync(0xffffffffu, take);
                unsigned int base = 0;
                if (lane == 0 && m) base = atomicAdd(&sh->ncand, (unsigned int)__popc(m));
                base = __shfl_sync(0xffffffffu, base, 0);
                if (take) {
                    const unsigned int pos = base + __popc(m & ((1u << lane) - 1u));
                    sh->cand[pos] = ((unsigned long long)key << 32) | (0xFFFFFFFFu - (uint32_t)i);
                }
            }
        }
        __syncthreads();
        // 4. the k largest candidates, written by ascending id
        const int n = (int)sh->ncand;
        const unsigned long long kk = kth_largest(sh->cand, n, k, sh);
        for (int i = tid; i < n; i += kThreads) {
            const unsigned long long key = sh->cand[i];
            if (key >= kk) {
                const unsigned int p = atomicAdd(&sh->nsel, 1u);
                if (p < (unsigned int)kMaxK) sh->sel[p] = (long long)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
            }
        }
        __syncthreads();
        if (tid < k) {
            const long long id = sh->sel[tid];
            int rank = 0;
            for (int j = 0; j < k; ++j) rank += sh->sel[j] < id;
            out[r * k + rank] = id;
        }
        __syncthreads();  // shared state is reused by the next row
    }
}

}  // namespace tk

int topk_max_k() { return tk::kMaxK; }
int topk_max_vocab() { return tk::kMaxChunks * tk::kChunk; }

int launch_topk_ids(const void* logits, int dtype, long long rows, int V, long long stride, int k,
                    int64_t* out, cudaStream_t st) {
    const size_t smem = sizeof(tk::Smem);
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) != cudaSuccess) return kLaunchFailed;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long cap = (long long)sms * 3;
    const unsigned grid = (unsigned)(rows < cap ? rows : cap);
    switch (dtype) {
        case 0:
            if (cudaFuncSetAttribute(tk::topk_ids_kernel<__nv_bfloat16>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
                return kLaunchFailed;
            tk::topk_ids_kernel<__nv_bfloat16><<<grid, tk::kThreads, smem, st>>>(
                static_cast<const __nv_bfloat16*>(logits), rows, V, stride, k, out);
            break;
        case 1:
            if (cudaFuncSetAttribute(tk::topk_ids_kernel<float>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
                return kLaunchFailed;
            tk::topk_ids_kernel<float><<<grid, tk::kThreads, smem, st>>>(
                static_cast<const float*>(logits), rows, V, stride, k, out);
            break;
        case 2:
            if (cudaFuncSetAttribute(tk::topk_ids_kernel<__half>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
                return kLaunchFailed;
            tk::topk_ids_kernel<__half><<<grid, tk::kThreads, smem, st>>>(
                static_cast<const __half*>(logits), rows, V, stride, k, out);
            break;
        default:
            return kBadDtype;
    }
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

}  // namespace dsv
