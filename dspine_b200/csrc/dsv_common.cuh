// dsv_common.cuh -- shared device helpers for the DSpine verification kernels (sm_100a).
//
// Arithmetic contract (identical in every kernel, so results do not depend on launch shape):
//   fix(x)  = round-half-even(min(x, 1) * 2^40) for x > 0, else 0: every sum that feeds a
//             decision (softmax denominators, the top-p boundary, the residual CDF) is an
//             exact integer sum of fix() values.
//   exp2c   = Cody-Waite split y = n + f (|f| <= 1/2) and a degree-6 polynomial fitted for this
//             project (relative error < 1 ulp), evaluated with explicit round-to-nearest
//             intrinsics so no contraction changes a bit.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace dsv {

// ---- status codes shared with the C ABI -------------------------------------------------
enum Status : int {
    kOk = 0,
    kBadShape = 1,
    kBadDtype = 2,
    kBadPointer = 3,
    kBadAlignment = 4,
    kLaunchFailed = 5,
    kWorkspaceTooSmall = 6,
    kDeviceTimeout = 7,
    kUnsupported = 8,
};

constexpr int kT = 16;          // draft block width
constexpr int kFixBits = 40;

// ---- canonical arithmetic ----------------------------------------------------------------
__device__ __forceinline__ float exp2c(float y) {
    if (!(y >= -125.0f)) return 0.0f;
    const float magic = 12582912.0f;  // 1.5 * 2^23
    float t = __fadd_rn(y, magic);
    int n = (int)(__float_as_uint(t) - 0x4B400000u);
    float f = __fsub_rn(y, __fsub_rn(t, magic));
    float p = __uint_as_float(0x3920fddcu);
    p = __fmaf_rn(p, f, __uint_as_float(0x3aaf9f2bu));
    p = __fmaf_rn(p, f, __uint_as_float(0x3c1d96a6u));
    p = __fmaf_rn(p, f, __uint_as_float(0x3d635774u));
    p = __fmaf_rn(p, f, __uint_as_float(0x3e75fdeeu));
    p = __fmaf_rn(p, f, __uint_as_float(0x3f317218u));
    p = __fmaf_rn(p, f, 1.0f);
    return __uint_as_float(__float_as_uint(p) + ((unsigned)n << 23));
}

// fix(x) for x already known to lie in [0, 1] (no NaN): hi/lo magic-number split.
__device__ __forceinline__ uint64_t fix01(float x) {
    float e2 = __fmul_rn(x, 131072.0f);               // 2^17, exact
    float t = __fadd_rn(e2, 8388608.0f);              // 2^23 + rne(e2)
    uint32_t hi = __float_as_uint(t) - 0x4B000000u;
    float r = __fsub_rn(e2, __fsub_rn(t, 8388608.0f)); // exact remainder, |r| <= 1/2
    float u = __fmaf_rn(r, 8388608.0f, 12582912.0f);  // 1.5*2^23 + rne(r * 2^23)
    int32_t lo = (int32_t)(__float_as_uint(u) - 0x4B400000u);
    return (uint64_t)((int64_t)hi * 8388608 + lo);
}

__device__ __forceinline__ uint64_t fixv(float x) {
    if (!(x > 0.0f)) return 0;
    return fix01(fminf(x, 1.0f));
}

// floor(u * m) exactly; -1 for u < 0; -2 for u >= 1 or NaN (no crossing).
__device__ __forceinline__ int64_t scale_floor(float u, uint64_t m) {
    if (!(u < 1.0f)) return -2;
    if (u < 0.0f) return -1;
    uint32_t b = __float_as_uint(u);
    uint32_t e = (b >> 23) & 0xFFu;
    uint64_t mant = (b & 0x7FFFFFu) | (e ? 0x800000u : 0u);
    int shift = e ? (150 - (int)e) : 149;
    if (shift >= 128) return 0;
    uint64_t lo = mant * m;
    uint64_t hi = __umul64hi(mant, m);
    if (shift >= 64) return (int64_t)(hi >> (shift - 64));
    return (int64_t)((lo >> shift) | (hi << (64 - shift)));
}

__device__ __forceinline__ float log2e_over(float T) {
    return __fdiv_rn(__uint_as_float(0x3FB8AA3Bu), T);
}

__device__ __forceinline__ bool is_greedy(float T, int top_k, float c) {
    return (top_k <= 1) || !(T > 0.0f) || !(c < __int_as_float(0x7f800000));
}

// ---- filter modes of the target distribution (runtime/worker.py:473-508) ------------------
//   kModeJoint  flashinfer backend, no min-p in the batch: joint top-k / top-p on unfiltered p
//   kModeSeq    flashinfer backend, min-p in the batch: top-k, then top-p against the top-k's
//               own mass, then the min-p floor
//   kModeTorch  pytorch backend: joint top-k / top-p, then the min-p floor
enum FilterMode : int { kModeJoint = 0, kModeSeq = 1, kModeTorch = 2 };

// The min-p floor of a row with maximum m and c = log2(e) / T: "p >= min_p * max p" is
// e = exp2c((v - m) c) >= min_p (the maximum has e = 1).  exp2c is monotone only up to one-ulp
// ripples, so the floor is the result of a bisection over the 32-bit ordered keys between -inf
// (e = 0) and m (e = 1): elements whose 32-bit key is >= the returned key pass.  min_p > 1
// passes nothing.  Identical to the oracle's or_minp_floor.
__device__ __forceinline__ uint32_t minp_floor32(float m, float c, float min_p) {
    uint32_t lo = 0x007FFFFFu;  // key of -inf
    const uint32_t mb = __float_as_uint(m);
    uint32_t hi = (mb == 0x80000000u) ? 0x80000000u : ((mb & 0x80000000u) ? ~mb : (mb | 0x80000000u));
    if (!(min_p <= 1.0f)) return hi + 1u;
    while (hi - lo > 1u) {
        const uint32_t mid = lo + (hi - lo) / 2u;
        const uint32_t u = (mid & 0x80000000u) ? (mid & 0x7FFFFFFFu) : ~mid;
        const float e = exp2c(__fmul_rn(__fsub_rn(__uint_as_float(u), m), c));
        if (e >= min_p) hi = mid; else lo = mid;
    }
    return hi;
}

// the smallest bf16 ordered key whose element's 32-bit key is >= k32 (a bf16 value's 32-bit
// key is key16 << 16, with the low half all ones for negative values)
__device__ __forceinline__ uint32_t key16_floor(uint32_t k32) {
    uint32_t k16 = k32 >> 16;
    const uint32_t full = (k16 << 16) | ((k16 & 0x8000u) ? 0u : 0xFFFFu);
    if (full < k32) ++k16;
    return k16;
}

// 1 / (S * 2^-40) for an exact fixed-point sum S (0 -> 0)
__device__ __forceinline__ float inv_from_fix(uint64_t S) {
    if (S == 0) return 0.0f;
    float sf = __fmul_rn(__ll2float_rn((long long)S), 9.094947017729282e-13f);
    return __fdiv_rn(1.0f, sf);
}

// ---- element traits ----------------------------------------------------------------------
template <typename T> struct Elem;

template <> struct Elem<__nv_bfloat16> {
    static constexpr int kEV = 8;       // elements per 16 bytes
    static constexpr int kKeyBits = 16;
    __device__ static __forceinline__ uint32_t raw(const __nv_bfloat16* p, int i) {
        return reinterpret_cast<const uint16_t*>(p)[i];
    }
    __device__ static __forceinline__ float to_float(uint32_t u) { return __uint_as_float(u << 16); }
    __device__ static __forceinline__ uint32_t key(uint32_t u) {
        if (u == 0x8000u) u = 0;
        return (u & 0x8000u) ? (u ^ 0xFFFFu) : (u | 0x8000u);
    }
    // inverse of key() on canonical values
    __device__ static __forceinline__ float key_to_float(uint32_t k) {
        uint32_t u = (k & 0x8000u) ? (k & 0x7FFFu) : (k ^ 0xFFFFu);
        return to_float(u);
    }
    // unpack a 16-byte vector into raw element bits
    __device__ static __forceinline__ void unpack(const uint4& v, uint32_t (&out)[kEV]) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            out[2 * j] = w[j] & 0xFFFFu;
            out[2 * j + 1] = w[j] >> 16;
        }
    }
};

template <> struct Elem<float> {
    static constexpr int kEV = 4;
    static constexpr int kKeyBits = 32;
    __device__ static __forceinline__ uint32_t raw(const float* p, int i) {
        return __float_as_uint(p[i]);
    }
    __device__ static __forceinline__ float to_float(uint32_t u) { return __uint_as_float(u); }
    __device__ static __forceinline__ uint32_t key(uint32_t u) {
        if (u == 0x80000000u) u = 0;
        return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    }
    __device__ static __forceinline__ float key_to_float(uint32_t k) {
        uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
        return __uint_as_float(u);
    }
    __device__ static __forceinline__ void unpack(const uint4& v, uint32_t (&out)[kEV]) {
        out[0] = v.x; out[1] = v.y; out[2] = v.z; out[3] = v.w;
    }
};

// ---- PTX helpers: mbarrier + bulk copy ----------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait: gives up after ~2 s of device time and reports false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > 2000000000ull) return false;
    }
}

// global -> this CTA's shared memory, completion counted on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ uint64_t ld_cg_u64(const uint64_t* p) { return __ldcg((const unsigned long long*)p); }

// ---- warp helpers -------------------------------------------------------------------------
__device__ __forceinline__ uint64_t warp_sum_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ uint32_t warp_sum_u32(uint32_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// inclusive scan over lanes (lane order)
__device__ __forceinline__ uint64_t warp_incl_u64(uint64_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint64_t n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

__device__ __forceinline__ uint32_t warp_incl_u32(uint32_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    return v;
}

// Packed pair: for both halves of a bf16x2 word w (logit l), yc = max((l - m) * c, -64) (nm = -m)
// and the raw float bits of h = 2^23 + rne(x), lo = 1.5*2^23 + rne((x - rne(x)) * 2^23) with
// x = exp2c(yc) * 2^17, so fix(exp2c(yc)) = (h - 0x4B000000) * 2^23 + (lo - 0x4B400000) exactly
// as fix01(exp2c(y)) for y <= 0 (below -64 both give 0).  Two elements per fp32x2 instruction.
struct Pair {
    float2 yc;
    uint32_t h0, h1, l0, l1;
};

__device__ __forceinline__ Pair exp_pair(uint32_t w, float2 nm, float2 c2) {
    const float2 l = make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
    float2 y = __fmul2_rn(__fadd2_rn(l, nm), c2);
    y.x = fmaxf(y.x, -64.0f);
    y.y = fmaxf(y.y, -64.0f);
    const float M17 = 12582912.0f + 17.0f;
    const float2 t = __fadd2_rn(y, make_float2(M17, M17));
    const float2 tm = __fadd2_rn(t, make_float2(-M17, -M17));
    const float2 f = __ffma2_rn(tm, make_float2(-1.0f, -1.0f), y);
    float2 p = make_float2(__uint_as_float(0x3920fddcu), __uint_as_float(0x3920fddcu));
    p = __ffma2_rn(p, f, make_float2(__uint_as_float(0x3aaf9f2bu), __uint_as_float(0x3aaf9f2bu)));
    p = __ffma2_rn(p, f, make_float2(__uint_as_float(0x3c1d96a6u), __uint_as_float(0x3c1d96a6u)));
    p = __ffma2_rn(p, f, make_float2(__uint_as_float(0x3d635774u), __uint_as_float(0x3d635774u)));
    p = __ffma2_rn(p, f, make_float2(__uint_as_float(0x3e75fdeeu), __uint_as_float(0x3e75fdeeu)));
    p = __ffma2_rn(p, f, make_float2(__uint_as_float(0x3f317218u), __uint_as_float(0x3f317218u)));
    p = __ffma2_rn(p, f, make_float2(1.0f, 1.0f));
    const float2 x = make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                                 __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
    const float2 h = __fadd2_rn(x, make_float2(8388608.0f, 8388608.0f));
    const float2 hm = __fadd2_rn(h, make_float2(-8388608.0f, -8388608.0f));
    const float2 r = __ffma2_rn(hm, make_float2(-1.0f, -1.0f), x);
    const float2 lo = __ffma2_rn(r, make_float2(8388608.0f, 8388608.0f), make_float2(12582912.0f, 12582912.0f));
    Pair o;
    o.yc = y;
    o.h0 = __float_as_uint(h.x);
    o.h1 = __float_as_uint(h.y);
    o.l0 = __float_as_uint(lo.x);
    o.l1 = __float_as_uint(lo.y);
    return o;
}

}  // namespace dsv
