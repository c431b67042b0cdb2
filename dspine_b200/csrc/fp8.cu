// fp8.cu -- row-scaled FP8 quantization and the BF16 rescore + top-16 of the coarse retrieval
// (sm_100a).
//
//   quantize_kernel   layers/fp8/coarse.py:41-55 (_scale, _quantize): per row
//                     scale = amax(|x|) / 448 (1 when the row is all zero) and
//                     q = e4m3(clamp(x / scale, -448, 448)), IEEE division, round to nearest
//                     even.  One CTA per row: one pass for the maximum, one for the codes
//                     (the second pass hits L2).  Used once per weight load for the head and
//                     per step for the hidden rows.
//   rescore16_kernel  layers/fp8/gather.py:7-79 (gather_dot, global_top16, rescore, select16):
//                     scores[m, c] = sum_h W[ids[m, c], h] * hidden[m, h] in fp32, stored in
//                     the hidden dtype (or fp32), then the 16 best of the row's candidates by
//                     (stored score desc, token asc), written ascending.  One CTA per row: the
//                     hidden row is staged in shared memory as fp32, each warp takes candidates
//                     wid, wid + 8, ... with two gathered weight rows in flight (16-byte loads),
//                     warp 0 runs the 16 selection rounds.  Without a weight the stored scores
//                     are the input and only the selection runs (select16 alone).
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>

#include "dsv_common.cuh"
#include "dsv_kernels.h"

namespace dsv {
namespace f8 {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxC = 128;                 // candidates per row
constexpr int kMaxH = 16384;               // hidden size (fp32 row in shared memory)

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__global__ void __launch_bounds__(kThreads) quantize_kernel(const T* __restrict__ x, long long rows,
                                                            int cols, long long stride,
                                                            uint8_t* __restrict__ q, long long q_stride,
                                                            float* __restrict__ scale) {
    __shared__ float wmax[kWarps];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
        const T* xr = x + r * stride;
        // the row maximum of |x| propagates NaN, as torch's amax: a NaN row gets scale 1
        // (NaN > 0 is false) and its NaN entries stay NaN through the clamp
        float m = 0.f;
        bool nan = false;
        for (int i = tid; i < cols; i += kThreads) {
            const float a = fabsf(to_f32<T>(xr[i]));
            nan |= a != a;
            m = fmaxf(m, a);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        nan = __any_sync(0xffffffffu, nan);
        if (lane == 0) wmax[wid] = nan ? __int_as_float(0x7fc00000) : m;
        __syncthreads();
        float amax = wmax[0];
        bool any_nan = amax != amax;
#pragma unroll
        for (int w = 1; w < kWarps; ++w) {
            any_nan |= wmax[w] != wmax[w];
            amax = fmaxf(amax, wmax[w]);
        }
        const float s = (!any_nan && amax > 0.f) ? __fdiv_rn(amax, 448.0f) : 1.0f;
        if (tid == 0) scale[r] = s;
        uint8_t* qr = q + r * q_stride;
        for (int i = tid; i < cols; i += kThreads) {
            const float t = __fdiv_rn(to_f32<T>(xr[i]), s);
            const float v = (t != t) ? t : fminf(fmaxf(t, -448.0f), 448.0f);
            qr[i] = (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
        }
        __syncthreads();  // wmax is reused by the next row
    }
}

// 8 consecutive bf16 weights (one 16-byte load) dotted with 8 fp32 hidden values
__device__ __forceinline__ float dot8(const uint4& w, const float* h, float acc) {
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float lo = __uint_as_float(u[i] << 16);
        const float hi = __uint_as_float(u[i] & 0xFFFF0000u);
        acc = fmaf(lo, h[2 * i], acc);
        acc = fmaf(hi, h[2 * i + 1], acc);
    }
    return acc;
}

template <typename HT>
__global__ void __launch_bounds__(kThreads) rescore16_kernel(int M, int C, int H, int V,
                                                             const __nv_bfloat16* __restrict__ w,
                                                             long long w_stride,
                                                             const int64_t* __restrict__ ids,
                                                             const HT* __restrict__ hidden,
                                                             long long h_stride, void* scores,
                                                             int scores_f32, int64_t* __restrict__ out16) {
    extern __shared__ __align__(16) float hs[];        // [H] hidden row, then [kMaxC] scores
    float* sc = hs + H;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    for (int m = blockIdx.x; m < M; m += gridDim.x) {
        if (w == nullptr) {
            // selection only (select16): the stored scores are the input
            for (int c = tid; c < C; c += kThreads)
                sc[c] = scores_f32 ? static_cast<const float*>(scores)[(long long)m * C + c]
                                   : __bfloat162float(static_cast<const __nv_bfloat16*>(scores)[(long long)m * C + c]);
        } else {
            const HT* hr = hidden + (long long)m * h_stride;
            for (int i = tid; i < H; i += kThreads) hs[i] = to_f32<HT>(hr[i]);
        }
        __syncthreads();
        // two candidates per warp step: both weight rows' loads are in flight together
        for (int c0 = wid; w != nullptr && c0 < C; c0 += 2 * kWarps) {
            const int c1 = c0 + kWarps;
            const int64_t t0 = ids[(long long)m * C + c0];
            const int64_t t1 = c1 < C ? ids[(long long)m * C + c1] : -1;
            const bool v0 = t0 >= 0 && t0 < V, v1 = c1 < C && t1 >= 0 && t1 < V;
            const __nv_bfloat16* w0 = w + (v0 ? t0 : 0) * w_stride;
            const __nv_bfloat16* w1 = w + (v1 ? t1 : 0) * w_stride;
            float a0 = 0.f, a1 = 0.f;
            for (int h0 = lane * 8; h0 < H; h0 += 256) {
                const uint4 x0 = v0 ? __ldg(reinterpret_cast<const uint4*>(w0 + h0)) : make_uint4(0, 0, 0, 0);
                const uint4 x1 = v1 ? __ldg(reinterpret_cast<const uint4*>(w1 + h0)) : make_uint4(0, 0, 0, 0);
                a0 = dot8(x0, hs + h0, a0);
                a1 = dot8(x1, hs + h0, a1);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                a0 += __shfl_xor_sync(0xffffffffu, a0, o);
                a1 += __shfl_xor_sync(0xffffffffu, a1, o);
            }
            if (lane == 0) {
                const float s0 = v0 ? a0 : -INFINITY;
                const float s1 = v1 ? a1 : -INFINITY;
                if (scores_f32) {
                    float* so = static_cast<float*>(scores) + (long long)m * C;
                    so[c0] = s0;
                    sc[c0] = s0;
                    if (c1 < C) {
                        so[c1] = s1;
                        sc[c1] = s1;
                    }
                } else {
                    __nv_bfloat16* so = static_cast<__nv_bfloat16*>(scores) + (long long)m * C;
                    const __nv_bfloat16 b0 = __float2bfloat16_rn(s0);
                    so[c0] = b0;
                    sc[c0] = __bfloat162float(b0);
                    if (c1 < C) {
                        const __nv_bfloat16 b1 = __float2bfloat16_rn(s1);
                        so[c1] = b1;
                        sc[c1] = __bfloat162float(b1);
                    }
                }
            }
        }
        __syncthreads();
        if (out16 && wid == 0) {
            // 16 rounds: the largest stored score, the lowest token holding it; that token's
            // scores drop to -inf (gather.py:37-50); the chosen tokens are written ascending
            float val[kMaxC / 32];
            int64_t tok[kMaxC / 32];
#pragma unroll
            for (int i = 0; i < kMaxC / 32; ++i) {
                const int c = lane + 32 * i;
                val[i] = c < C ? sc[c] : -INFINITY;
                tok[i] = c < C ? ids[(long long)m * C + c] : INT64_MAX;
            }
            int64_t chosen = INT64_MAX;
            for (int j = 0; j < 16; ++j) {
                float best = val[0];
#pragma unroll
                for (int i = 1; i < kMaxC / 32; ++i) best = fmaxf(best, val[i]);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, o));
                int64_t t = INT64_MAX;
#pragma unroll
                for (int i = 0; i < kMaxC / 32; ++i)
                    if (val[i] == best && tok[i] < t) t = tok[i];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const int64_t ot = __shfl_xor_sync(0xffffffffu, t, o);
                    t = ot < t ? ot : t;
                }
                if (lane == j) chosen = t;
#pragma unroll
                for (int i = 0; i < kMaxC / 32; ++i)
                    if (tok[i] == t) val[i] = -INFINITY;
            }
            // ascending order: rank among the 16 chosen (equal tokens keep lane order)
            int rank = 0;
            for (int o = 0; o < 16; ++o) {
                const int64_t ot = __shfl_sync(0xffffffffu, chosen, o);
                rank += (ot < chosen) || (ot == chosen && o < lane);
            }
            if (lane < 16) out16[(long long)m * 16 + rank] = chosen;
        }
        __syncthreads();  // hs and sc are reused by the next row
    }
}

int grid_for(long long rows) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long cap = (long long)sms * 8;
    return (int)(rows < cap ? rows : cap);
}

}  // namespace f8

int launch_fp8_quantize(const void* x, int dtype, long long rows, int cols, long long stride,
                        uint8_t* q, long long q_stride, float* scale, cudaStream_t st) {
    const int grid = f8::grid_for(rows);
    if (dtype == 0)
        f8::quantize_kernel<__nv_bfloat16><<<grid, f8::kThreads, 0, st>>>(
            static_cast<const __nv_bfloat16*>(x), rows, cols, stride, q, q_stride, scale);
    else if (dtype == 1)
        f8::quantize_kernel<float><<<grid, f8::kThreads, 0, st>>>(static_cast<const float*>(x), rows, cols,
                                                                   stride, q, q_stride, scale);
    else
        return kBadDtype;
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

int launch_rescore16(int M, int C, int H, int V, const void* w, long long w_stride, const int64_t* ids,
                     const void* hidden, int hidden_dtype, long long h_stride, void* scores,
                     int scores_f32, int64_t* out16, cudaStream_t st) {
    const size_t smem = (size_t)(H + f8::kMaxC) * sizeof(float);
    const int grid = f8::grid_for(M);
    const auto* wb = static_cast<const __nv_bfloat16*>(w);
    if (hidden_dtype == 0) {
        if (smem > 48 * 1024 &&
            cudaFuncSetAttribute(f8::rescore16_kernel<__nv_bfloat16>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return kLaunchFailed;
        f8::rescore16_kernel<__nv_bfloat16><<<grid, f8::kThreads, smem, st>>>(
            M, C, H, V, wb, w_stride, ids, static_cast<const __nv_bfloat16*>(hidden), h_stride, scores,
            scores_f32, out16);
    } else if (hidden_dtype == 1) {
        if (smem > 48 * 1024 &&
            cudaFuncSetAttribute(f8::rescore16_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess)
            return kLaunchFailed;
        f8::rescore16_kernel<float><<<grid, f8::kThreads, smem, st>>>(
            M, C, H, V, wb, w_stride, ids, static_cast<const float*>(hidden), h_stride, scores, scores_f32,
            out16);
    } else {
        return kBadDtype;
    }
    return cudaGetLastError() == cudaSuccess ? kOk : kLaunchFailed;
}

int fp8_max_candidates() { return f8::kMaxC; }
int fp8_max_hidden() { return f8::kMaxH; }

}  // namespace dsv
