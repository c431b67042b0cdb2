// lmhead.cu -- draft LM head fused with top-k and logsumexp (sm_100a: tcgen05 + TMEM + TMA).
//
// Replaces `torch.matmul(rows, W.T)` followed by `topk_ids` (runtime/worker.py:283-285,
// kernels/dspine.py:165-207) and, per vocabulary shard, the local half of the TP head
// (sampling/tp_head.py:17-103): logits = X . W^T are never written to HBM.
//
//   lmhead_kernel   persistent, one CTA per SM, 192 threads:
//                     warp 0      TMA producer: X tile [128 x 64] and W tile [256 x 64] per stage
//                                 (128-byte swizzle, 4 stages of 48 KB, mbarrier completion)
//                     warp 1      TMEM allocation (512 columns = two 128 x 256 fp32 accumulators)
//                                 and the MMA issuer: tcgen05.mma kind::f16 (bf16 in, fp32
//                                 accumulate), 4 MMAs of K = 16 per stage, tcgen05.commit frees
//                                 the stage and, after the last stage, hands the accumulator over
//                     warps 2-5   epilogue: one accumulator row per thread (tcgen05.ld 32x32b),
//                                 running top-k and running (max, sum exp) over the CTA's columns
//                   CTA (m, j) owns row tile m and column tiles j, j + nsplit, ...; the CTAs of
//                   one j read the same W tile at the same time, so W streams from HBM once and
//                   the other row tiles hit it in L2.
//   merge_kernel    one warp per row: merges the nsplit partial lists (value desc, index asc)
//                   and their logsumexps; optionally sorts the ids ascending (topk_ids order).
//
// Ranking key: the logit rounded to bf16, exactly the value `torch.matmul` on bf16 tensors
// materialises and `topk_ids` ranks; ties go to the lower vocabulary index.  The logsumexp is
// taken over the fp32 accumulators.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <cstring>
#include <mutex>

#include "dsv_common.cuh"
#include "dsv_kernels.h"

namespace dsv {
namespace lm {

constexpr int kBM = 128;                   // rows per tile (MMA M)
constexpr int kBN = 256;                   // columns per tile (MMA N)
constexpr int kBK = 64;                    // K per stage: 64 bf16 = one 128-byte swizzle row
constexpr int kUK = 16;                    // K per tcgen05.mma (kind::f16)
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 2;     // 16 KB
constexpr int kBBytes = kBN * kBK * 2;     // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 192;
constexpr int kTmemCols = 2 * kBN;         // double-buffered accumulator
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /* barriers */ + 1024 /* alignment */;
constexpr int32_t kNoId = 0x7fffffff;      // empty top-k slot (ranks after every real index)

static_assert(kABytes % 1024 == 0 && kBBytes % 1024 == 0, "swizzle atoms are 1024-byte aligned");

struct Bars {
    uint64_t full[kStages];
    uint64_t empty[kStages];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};

struct LmArgs {
    int M, N, K;
    int mt, nsplit, ntiles;  // row tiles, CTAs per row tile, column tiles
    int topk;
    float* part_val;         // [M][nsplit][topk] ranking keys, descending
    int32_t* part_id;        // [M][nsplit][topk] local column
    float* part_lse;         // [M][nsplit]
    unsigned int* err;       // workspace error word
};

// ---- tcgen05 / TMA helpers -----------------------------------------------------------------

// UMMA shared-memory descriptor: K-major operand, 128-byte swizzle; rows 128 B apart, 8-row
// groups 1024 B apart (SBO), LBO unused by swizzled K-major layouts (encoded as 1), version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);        // start address
    d |= (uint64_t)1u << 16;                        // leading byte offset (16 B units)
    d |= (uint64_t)(1024u >> 4) << 32;              // stride byte offset
    d |= (uint64_t)1u << 46;                        // descriptor version (sm100)
    d |= (uint64_t)2u << 61;                        // SWIZZLE_128B
    return d;
}

// instruction descriptor, kind::f16: D f32, A and B bf16, both K-major, M = 128, N = 256
constexpr uint32_t kIdesc = (1u << 4)                 // D format f32
                          | (1u << 7)                 // A format bf16
                          | (1u << 10)                // B format bf16
                          | ((uint32_t)(kBN >> 3) << 17)
                          | ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes, one lane per thread
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float round_bf16(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
}

// bounded wait that also gives up when another role of the CTA has aborted
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort) return false;
        if (globaltimer_ns() - t0 > 2000000000ull) {
            *abort = 1;
            return false;
        }
    }
}

// insert (kv, col) into the descending list; equal keys keep the earlier (lower) index first
template <int TK>
__device__ __forceinline__ void topk_insert(float (&val)[TK], int32_t (&id)[TK], float kv, int32_t col) {
#pragma unroll
    for (int i = TK - 1; i > 0; --i) {
        const bool up = kv > val[i - 1];
        const bool here = !up && kv > val[i];
        val[i] = up ? val[i - 1] : (here ? kv : val[i]);
        id[i] = up ? id[i - 1] : (here ? col : id[i]);
    }
    if (kv > val[0]) {
        val[0] = kv;
        id[0] = col;
    }
}

template <int TK>
__global__ void __launch_bounds__(kThreads, 1)
    lmhead_kernel(const __grid_constant__ CUtensorMap tma_x, const __grid_constant__ CUtensorMap tma_w,
                  LmArgs a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* base = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t* sa = base;                                  // [kStages][kABytes]
    uint8_t* sb = base + kStages * kABytes;              // [kStages][kBBytes]
    Bars* bars = reinterpret_cast<Bars*>(base + kStages * kStageBytes);
    volatile int* abort = &bars->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tile = blockIdx.x % a.mt;
    const int j = blockIdx.x / a.mt;
    const int my_tiles = (j < a.ntiles) ? (a.ntiles - 1 - j) / a.nsplit + 1 : 0;
    const int nk = a.K / kBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->tfull[i], 1);
            mbar_init(&bars->tempty[i], 4);
        }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&bars->tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        uint32_t g = 0;
        bool ok = true;
        for (int t = 0; t < my_tiles && ok; ++t) {
            const int n_tile = j + t * a.nsplit;
            for (int kb = 0; kb < nk; ++kb, ++g) {
                const uint32_t s = g % kStages, ph = (g / kStages) & 1u;
                if (lane == 0) {
                    ok = wait_or_abort(&bars->empty[s], ph ^ 1u, abort);
                    if (ok) {
                        mbar_arrive_expect_tx(&bars->full[s], (uint32_t)kStageBytes);
                        tma_load_2d(sa + s * kABytes, &tma_x, kb * kBK, m_tile * kBM, &bars->full[s]);
                        tma_load_2d(sb + s * kBBytes, &tma_w, kb * kBK, n_tile * kBN, &bars->full[s]);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
            }
        }
        // every copy this thread issued has landed before the CTA may exit
        if (lane == 0) {
            for (uint32_t s = 0; s < kStages && s < g; ++s) {
                const uint32_t last = g - 1 - ((g - 1 - s) % kStages);  // last use of stage s
                if (!mbar_wait_bounded(&bars->full[s], (last / kStages) & 1u)) *abort = 1;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        uint32_t g = 0;
        bool ok = true;
        for (int t = 0; t < my_tiles && ok; ++t) {
            const uint32_t acc = t & 1, use = (uint32_t)t >> 1;
            if (lane == 0) {
                ok = wait_or_abort(&bars->tempty[acc], (use & 1u) ^ 1u, abort);
                tc_fence_after();
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            const uint32_t d_tmem = tmem + acc * kBN;
            for (int kb = 0; kb < nk; ++kb, ++g) {
                const uint32_t s = g % kStages, ph = (g / kStages) & 1u;
                if (lane == 0) {
                    ok = wait_or_abort(&bars->full[s], ph, abort);
                    if (ok) {
                        tc_fence_after();
                        const uint32_t a0 = smem_u32(sa + s * kABytes);
                        const uint32_t b0 = smem_u32(sb + s * kBBytes);
#pragma unroll
                        for (int kk = 0; kk < kBK / kUK; ++kk)
                            mma_bf16(d_tmem, umma_desc_sw128(a0 + kk * kUK * 2),
                                     umma_desc_sw128(b0 + kk * kUK * 2), (kb | kk) != 0);
                        mma_commit(&bars->empty[s]);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
            }
            if (ok && lane == 0) mma_commit(&bars->tfull[acc]);
        }
        // all MMAs this thread issued are complete before TMEM is released
        if (lane == 0) {
            mma_commit(&bars->drain);
            if (!mbar_wait_bounded(&bars->drain, 0)) *abort = 1;
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: one row per thread ----------------
        const int q = warp & 3;                      // TMEM lane quarter of this warp
        const int row = m_tile * kBM + q * 32 + lane;
        constexpr float kL2E = 1.4426950408889634f;
        float val[TK];
        int32_t id[TK];
#pragma unroll
        for (int i = 0; i < TK; ++i) {
            val[i] = -INFINITY;
            id[i] = kNoId;
        }
        float run_m = -INFINITY, run_s = 0.f;
        bool ok = true;
        for (int t = 0; t < my_tiles; ++t) {
            const uint32_t acc = t & 1, use = (uint32_t)t >> 1;
            const int col0 = (j + t * a.nsplit) * kBN;
            if (lane == 0) ok = wait_or_abort(&bars->tfull[acc], use & 1u, abort);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + acc * kBN;
#pragma unroll 1
            for (int c = 0; c < kBN / 32; ++c) {
                float v[32];
                __syncwarp();  // tcgen05.ld is warp-collective: reconverge after the insertions
                tmem_ld32(taddr + c * 32, v);
                const int cb = col0 + c * 32;
                if (cb + 32 > a.N) {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (cb + i >= a.N) v[i] = -INFINITY;
                }
                float cmax = v[0];
#pragma unroll
                for (int i = 1; i < 32; ++i) cmax = fmaxf(cmax, v[i]);
                if (cmax == -INFINITY) continue;  // only fully masked chunks (same for all lanes)
                const float nm = fmaxf(run_m, cmax);
                const float nml = nm * kL2E;
                float s = 0.f;
#pragma unroll
                for (int i = 0; i < 32; ++i) s += ex2_approx(fmaf(v[i], kL2E, -nml));
                run_s = run_s * ex2_approx((run_m - nm) * kL2E) + s;
                run_m = nm;
                if (round_bf16(cmax) > val[TK - 1]) {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        const float kv = round_bf16(v[i]);
                        if (kv > val[TK - 1]) topk_insert<TK>(val, id, kv, cb + i);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->tempty[acc]);
        }
        if (ok && row < a.M && my_tiles > 0) {
            const size_t p = (size_t)row * a.nsplit + j;
#pragma unroll
            for (int i = 0; i < TK; ++i) {
                a.part_val[p * TK + i] = val[i];
                a.part_id[p * TK + i] = id[i];
            }
            a.part_lse[p] = run_m == -INFINITY ? -INFINITY : run_m + logf(run_s);
        } else if (row < a.M && my_tiles > 0) {
            atomicOr(a.err, 1u);
        }
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

// ---- FP8 coarse scores (layers/fp8/coarse.py:84-93) ----------------------------------------
//
// scores[r, c] = bf16((sum_h xq[r, h] * wq[c, h]) * sx[r] * sw[c]) with e4m3 operands, the fp32
// accumulation of tcgen05.mma kind::f8f6f4 and one bf16 rounding: the row-scaled FP8 GEMM the
// reference runs through torch._scaled_mm (use_fast_accum=False, out_dtype bf16).  Same
// pipeline as lmhead_kernel: a K stage is 128 e4m3 values = one 128-byte swizzle row, so the
// stage bytes, the swizzle atoms and the 32-byte descriptor step per MMA (K = 32) are unchanged.

// instruction descriptor, kind::f8f6f4: D f32, A and B e4m3 (format 0), both K-major,
// M = 128, N = 256
constexpr uint32_t kIdescF8 = (1u << 4)               // D format f32
                            | (0u << 7)               // A format e4m3
                            | (0u << 10)              // B format e4m3
                            | ((uint32_t)(kBN >> 3) << 17)
                            | ((uint32_t)(kBM >> 4) << 24);
constexpr int kBK8 = 128;                  // e4m3 values per stage row (128 bytes)

__device__ __forceinline__ void mma_e4m3(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(kIdescF8), "r"(accumulate)
        : "memory");
}

struct CoarseArgs {
    int M, N, K;
    int mt, nsplit, ntiles;
    const float* sx;         // [M] row scales of the quantized rows
    const float* sw;         // [N] row scales of the quantized weight
    __nv_bfloat16* out;      // [M, N] scores, rows out_stride elements apart
    long long out_stride;
    unsigned int* err;       // bit 0 set when a wait timed out
};

__global__ void __launch_bounds__(kThreads, 1)
    coarse8_kernel(const __grid_constant__ CUtensorMap tma_x, const __grid_constant__ CUtensorMap tma_w,
                   CoarseArgs a) {
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    uint8_t* base = smem_raw + ((1024u - (raw_addr & 1023u)) & 1023u);
    uint8_t* sa = base;                                  // [kStages][kABytes]
    uint8_t* sb = base + kStages * kABytes;              // [kStages][kBBytes]
    Bars* bars = reinterpret_cast<Bars*>(base + kStages * kStageBytes);
    volatile int* abort = &bars->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tile = blockIdx.x % a.mt;
    const int j = blockIdx.x / a.mt;
    const int my_tiles = (j < a.ntiles) ? (a.ntiles - 1 - j) / a.nsplit + 1 : 0;
    const int nk = a.K / kBK8;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->tfull[i], 1);
            mbar_init(&bars->tempty[i], 4);
        }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&bars->tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        uint32_t g = 0;
        bool ok = true;
        for (int t = 0; t < my_tiles && ok; ++t) {
            const int n_tile = j + t * a.nsplit;
            for (int kb = 0; kb < nk; ++kb, ++g) {
                const uint32_t s = g % kStages, ph = (g / kStages) & 1u;
                if (lane == 0) {
                    ok = wait_or_abort(&bars->empty[s], ph ^ 1u, abort);
                    if (ok) {
                        mbar_arrive_expect_tx(&bars->full[s], (uint32_t)kStageBytes);
                        tma_load_2d(sa + s * kABytes, &tma_x, kb * kBK8, m_tile * kBM, &bars->full[s]);
                        tma_load_2d(sb + s * kBBytes, &tma_w, kb * kBK8, n_tile * kBN, &bars->full[s]);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
            }
        }
        if (lane == 0) {
            for (uint32_t s = 0; s < kStages && s < g; ++s) {
                const uint32_t last = g - 1 - ((g - 1 - s) % kStages);
                if (!mbar_wait_bounded(&bars->full[s], (last / kStages) & 1u)) *abort = 1;
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        uint32_t g = 0;
        bool ok = true;
        for (int t = 0; t < my_tiles && ok; ++t) {
            const uint32_t acc = t & 1, use = (uint32_t)t >> 1;
            if (lane == 0) {
                ok = wait_or_abort(&bars->tempty[acc], (use & 1u) ^ 1u, abort);
                tc_fence_after();
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            const uint32_t d_tmem = tmem + acc * kBN;
            for (int kb = 0; kb < nk; ++kb, ++g) {
                const uint32_t s = g % kStages, ph = (g / kStages) & 1u;
                if (lane == 0) {
                    ok = wait_or_abort(&bars->full[s], ph, abort);
                    if (ok) {
                        tc_fence_after();
                        const uint32_t a0 = smem_u32(sa + s * kABytes);
                        const uint32_t b0 = smem_u32(sb + s * kBBytes);
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)   // K = 32 e4m3 = 32 bytes per MMA
                            mma_e4m3(d_tmem, umma_desc_sw128(a0 + kk * 32),
                                     umma_desc_sw128(b0 + kk * 32), (kb | kk) != 0);
                        mma_commit(&bars->empty[s]);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
            }
            if (ok && lane == 0) mma_commit(&bars->tfull[acc]);
        }
        if (lane == 0) {
            mma_commit(&bars->drain);
            if (!mbar_wait_bounded(&bars->drain, 0)) *abort = 1;
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: one row per thread, scaled and rounded to bf16 -------------
        const int q = warp & 3;
        const int row = m_tile * kBM + q * 32 + lane;
        const float sxr = row < a.M ? a.sx[row] : 0.f;
        __nv_bfloat16* orow = a.out + (long long)(row < a.M ? row : 0) * a.out_stride;
        const bool vec = ((reinterpret_cast<uintptr_t>(a.out) | (uintptr_t)(a.out_stride * 2)) & 15u) == 0;
        bool ok = true;
        for (int t = 0; t < my_tiles; ++t) {
            const uint32_t acc = t & 1, use = (uint32_t)t >> 1;
            const int col0 = (j + t * a.nsplit) * kBN;
            if (lane == 0) ok = wait_or_abort(&bars->tfull[acc], use & 1u, abort);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            tc_fence_after();
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + acc * kBN;
#pragma unroll 1
            for (int c = 0; c < kBN / 32; ++c) {
                float v[32];
                __syncwarp();
                tmem_ld32(taddr + c * 32, v);
                const int cb = col0 + c * 32;
                if (row >= a.M || cb >= a.N) continue;
                if (vec && cb + 32 <= a.N) {
                    uint32_t pk[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float lo = v[2 * i] * sxr * __ldg(a.sw + cb + 2 * i);
                        const float hi = v[2 * i + 1] * sxr * __ldg(a.sw + cb + 2 * i + 1);
                        const __nv_bfloat162 b2 = __floats2bfloat162_rn(lo, hi);
                        memcpy(&pk[i], &b2, 4);
                    }
                    uint4* dst = reinterpret_cast<uint4*>(orow + cb);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        dst[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        if (cb + i < a.N) orow[cb + i] = __float2bfloat16_rn(v[i] * sxr * __ldg(a.sw + cb + i));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->tempty[acc]);
        }
        if (!ok) atomicOr(a.err, 1u);
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

// ---- merge of sorted partial lists ---------------------------------------------------------

__device__ __forceinline__ bool ahead(float va, int64_t ia, float vb, int64_t ib) {
    return va > vb || (va == vb && ia < ib);
}

// One warp per row.  List p of row r holds k entries (descending, ties by index):
// values at val[p * val_ps + r * val_rs + i], ids at ids[p * id_ps + r * id_rs + i] (IdT: int32
// local columns shifted by id_offset, or int64 global ids), and the list's logsumexp at
// lse[p * lse_ps + r * lse_rs].
template <typename IdT>
__global__ void merge_kernel(int M, int P, int k, const float* __restrict__ val, int64_t val_ps,
                             int64_t val_rs, const IdT* __restrict__ ids, int64_t id_ps,
                             int64_t id_rs, const float* __restrict__ lse, int64_t lse_ps,
                             int64_t lse_rs, int64_t id_offset, int64_t pad_id, int sort_ids,
                             int64_t* __restrict__ out_ids, float* __restrict__ out_val,
                             float* __restrict__ out_lse) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= M) return;
    const int r = warp;
    // logsumexp of the lists' logsumexps
    float m = -INFINITY;
    for (int p = lane; p < P; p += 32) m = fmaxf(m, lse[p * lse_ps + r * lse_rs]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
    if (m != -INFINITY)
        for (int p = lane; p < P; p += 32) {
            const float l = lse[p * lse_ps + r * lse_rs];
            if (l != -INFINITY) s += expf(l - m);
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0 && out_lse) out_lse[r] = m == -INFINITY ? -INFINITY : m + logf(s);

    // k rounds of "take the best head"; lane l owns lists l, l + 32, ... (heads in registers)
    constexpr int kMaxOwn = 8;  // P <= 256
    int head[kMaxOwn];
#pragma unroll
    for (int i = 0; i < kMaxOwn; ++i) head[i] = 0;
    float my_v = -INFINITY;
    int64_t my_id = pad_id;
    for (int round = 0; round < k; ++round) {
        float bv = -INFINITY;
        int64_t bi = INT64_MAX;
        int bown = -1;
#pragma unroll
        for (int i = 0; i < kMaxOwn; ++i) {
            const int p = lane + 32 * i;
            if (p < P && head[i] < k) {
                const float v = val[p * val_ps + r * val_rs + head[i]];
                const IdT raw = ids[p * id_ps + r * id_rs + head[i]];
                const int64_t gid = (sizeof(IdT) == 4 && (int32_t)raw == kNoId) ? INT64_MAX
                                                                                 : (int64_t)raw + id_offset;
                if (ahead(v, gid, bv, bi)) {
                    bv = v;
                    bi = gid;
                    bown = i;
                }
            }
        }
        // warp-wide best of (bv, bi)
        float wv = bv;
        int64_t wi = bi;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, wv, o);
            const int64_t oi = __shfl_xor_sync(0xffffffffu, wi, o);
            if (ahead(ov, oi, wv, wi)) {
                wv = ov;
                wi = oi;
            }
        }
        if (bown >= 0 && bv == wv && bi == wi) {
#pragma unroll
            for (int i = 0; i < kMaxOwn; ++i)
                if (i == bown) ++head[i];
        }
        if (lane == round) {
            my_v = wv;
            my_id = (wi == INT64_MAX || wv == -INFINITY) ? pad_id : wi;
        }
    }
    const int kk = k;  // k <= 32: one output per lane
    if (sort_ids) {
        // rank of this lane's id among the k ids (ids are distinct except padding)
        int rank = 0;
        for (int o = 0; o < kk; ++o) {
            const int64_t oid = __shfl_sync(0xffffffffu, my_id, o);
            rank += (oid < my_id) || (oid == my_id && o < lane);
        }
        if (lane < kk) {
            out_ids[(int64_t)r * k + rank] = my_id;
            out_val[(int64_t)r * k + rank] = my_v;
        }
    } else if (lane < kk) {
        out_ids[(int64_t)r * k + lane] = my_id;
        out_val[(int64_t)r * k + lane] = my_v;
    }
}

// ---- host side -----------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D bf16 tensor [rows, cols] (cols contiguous, `stride` elements between rows), box
// [box_rows, 64] with 128-byte swizzle; out-of-range rows read as zero
bool make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t stride,
              int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)stride * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D e4m3 tensor [rows, cols] (bytes), box [box_rows, 128] with 128-byte swizzle
bool make_map_u8(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t stride,
                 int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)stride};
    const cuuint32_t box[2] = {(cuuint32_t)kBK8, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    return n;
}

void geometry(int M, int N, int* mt, int* nsplit, int* ntiles) {
    const int sms = sm_count() > 0 ? sm_count() : 148;
    *mt = (M + kBM - 1) / kBM;
    *ntiles = (N + kBN - 1) / kBN;
    int ns = sms / *mt;
    if (ns < 1) ns = 1;
    if (ns > *ntiles) ns = *ntiles;
    if (ns > 256) ns = 256;
    *nsplit = ns;
}

template <int TK>
int launch_tk(const CUtensorMap& mx, const CUtensorMap& mw, const LmArgs& a, cudaStream_t st) {
    // once per device (the attribute belongs to the current device; no call during capture)
    static int attr_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kLaunchFailed;
    if (!attr_set[dev]) {
        if (cudaFuncSetAttribute(lmhead_kernel<TK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kSmemBytes) != cudaSuccess)
            return kLaunchFailed;
        attr_set[dev] = 1;
    }
    lmhead_kernel<TK><<<a.mt * a.nsplit, kThreads, kSmemBytes, st>>>(mx, mw, a);
    return cudaGetLastError() == cudaSuccess ? 0 : kLaunchFailed;
}

}  // namespace lm

size_t lmhead_workspace_bytes(int M, int N, int k) {
    int mt, ns, nt;
    lm::geometry(M, N, &mt, &ns, &nt);
    const int tk = lmhead_tk(k);
    return 64 + (size_t)M * ns * ((size_t)tk * 8 + 4) + 256;
}

int lmhead_tk(int k) { return k <= 8 ? 8 : (k <= 16 ? 16 : (k <= 20 ? 20 : (k <= 32 ? 32 : 0))); }

int launch_lmhead(const LmHeadArgs& h, cudaStream_t st) {
    using namespace lm;
    LmArgs a = {};
    a.M = h.M;
    a.N = h.N;
    a.K = h.K;
    geometry(h.M, h.N, &a.mt, &a.nsplit, &a.ntiles);
    const int tk = lmhead_tk(h.k);
    a.topk = tk;
    char* ws = reinterpret_cast<char*>(h.workspace);
    a.err = reinterpret_cast<unsigned int*>(ws + 12);
    char* p = ws + 64;
    a.part_val = reinterpret_cast<float*>(p);
    p += (size_t)h.M * a.nsplit * tk * 4;
    a.part_id = reinterpret_cast<int32_t*>(p);
    p += (size_t)h.M * a.nsplit * tk * 4;
    a.part_lse = reinterpret_cast<float*>(p);

    CUtensorMap mx, mw;
    if (!make_map(&mx, h.x, h.M, h.K, h.x_stride, kBM)) return kLaunchFailed;
    if (!make_map(&mw, h.w, h.N, h.K, h.w_stride, kBN)) return kLaunchFailed;
    int st_ = 0;
    switch (tk) {
        case 8: st_ = launch_tk<8>(mx, mw, a, st); break;
        case 16: st_ = launch_tk<16>(mx, mw, a, st); break;
        case 20: st_ = launch_tk<20>(mx, mw, a, st); break;
        case 32: st_ = launch_tk<32>(mx, mw, a, st); break;
        default: return kUnsupported;
    }
    if (st_) return st_;
    // merge the nsplit partial lists of every row (list p of row r at (r * nsplit + p) * tk)
    const int warps_per_block = 8;
    const int blocks = (h.M + warps_per_block - 1) / warps_per_block;
    merge_kernel<int32_t><<<blocks, 32 * warps_per_block, 0, st>>>(
        h.M, a.nsplit, h.k, a.part_val, tk, (int64_t)a.nsplit * tk, a.part_id, tk,
        (int64_t)a.nsplit * tk, a.part_lse, 1, a.nsplit, h.id_offset, h.pad_id, h.sort_ids,
        h.out_ids, h.out_val, h.out_lse);
    return cudaGetLastError() == cudaSuccess ? 0 : kLaunchFailed;
}

int launch_coarse8(const Coarse8Args& h, cudaStream_t st) {
    using namespace lm;
    CoarseArgs a = {};
    a.M = h.M;
    a.N = h.N;
    a.K = h.K;
    geometry(h.M, h.N, &a.mt, &a.nsplit, &a.ntiles);
    a.sx = h.sx;
    a.sw = h.sw;
    a.out = static_cast<__nv_bfloat16*>(h.out);
    a.out_stride = h.out_stride;
    a.err = h.err;
    CUtensorMap mx, mw;
    if (!make_map_u8(&mx, h.xq, h.M, h.K, h.x_stride, kBM)) return kLaunchFailed;
    if (!make_map_u8(&mw, h.wq, h.N, h.K, h.w_stride, kBN)) return kLaunchFailed;
    static int attr_set[64] = {};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kLaunchFailed;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!attr_set[dev]) {
            if (cudaFuncSetAttribute(coarse8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBytes) != cudaSuccess)
                return kLaunchFailed;
            attr_set[dev] = 1;
        }
    }
    coarse8_kernel<<<a.mt * a.nsplit, kThreads, kSmemBytes, st>>>(mx, mw, a);
    return cudaGetLastError() == cudaSuccess ? 0 : kLaunchFailed;
}

int launch_topk_merge(const TopkMergeArgs& m, cudaStream_t st) {
    const int warps_per_block = 8;
    const int blocks = (m.M + warps_per_block - 1) / warps_per_block;
    lm::merge_kernel<int64_t><<<blocks, 32 * warps_per_block, 0, st>>>(
        m.M, m.P, m.k, m.val, m.val_ps, m.k, m.ids, m.id_ps, m.k, m.lse, m.lse_ps, 1, 0, m.pad_id,
        m.sort_ids, m.out_ids, m.out_val, m.out_lse);
    return cudaGetLastError() == cudaSuccess ? 0 : kLaunchFailed;
}

}  // namespace dsv
