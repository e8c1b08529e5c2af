// Tensor-core GEMMs on sm_100a (tcgen05 + TMA) with two epilogues:
//
//     trace:  out += sum_{i < M, j < N} (A B^T)[i][j] * D[i][j]
//     store:  D = alpha * A B^T + beta * D
//
// and the calibration-Hessian accumulation built on the store GEMM
// (kq_accumulate_hessian, kquant/capture.py:713-730): an operand kernel
// (transpose, weighting, TF32 hi/lo split) and one symmetric 3xTF32 launch
// over the upper-triangle tiles (abt_seg_kernel<SYM, X3>, described below).
//
// A [M x Kd] and B [N x Kd] are row-major fp32 (both K-major); D [M x N]
// has row stride ldd.  The proxy error numerator of the encoder,
// tr(E^T H E) (kquant/exl3_encoder_backend.py:1466-1492), is this with
// A = D = E^T and B = H (H symmetric).  No product matrix is ever written:
// each 128 x 256 tile lives in tensor memory and is reduced in the epilogue.
//
// Per CTA (128 threads, one 128 x 256 output tile):
//  * warp 0, one lane: TMA loads of 128 x 32 (A) and 256 x 32 (B) fp32 tiles,
//    128-byte swizzle, into a 4-stage shared-memory ring (mbarrier complete_tx);
//  * warp 1, one lane: tcgen05.mma.cta_group::1.kind::tf32, M=128 N=256 K=8,
//    four per stage, accumulating in a 256-column TMEM tile; tcgen05.commit
//    frees each stage and finally signals the epilogue;
//  * all four warps: tcgen05.ld 32x32b (warp w owns TMEM lanes 32w..32w+31 =
//    tile rows), multiply by D, reduce in fp64, one atomicAdd per warp.
// Inputs enter the tensor cores as TF32 (10-bit mantissa), accumulation is
// fp32.  Every mbarrier wait is bounded: on timeout the kernel sets *err and
// still releases its tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include "kq_common.cuh"

namespace kq {
namespace {

constexpr int BM = 128, BN = 256, BK = 32, STAGES = 4;
constexpr int A_BYTES = BM * BK * 4;           // 16 KiB
constexpr int B_BYTES = BN * BK * 4;           // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;   // + alignment slack
constexpr uint32_t kSpinLimit = 1u << 24;
constexpr uint32_t kTmemCols = 256;

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

// Bounded wait for the phase with the given parity; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_addr(bar);
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_addr(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// UMMA shared-memory descriptor: K-major tile, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), LBO unused (1), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: D fp32, A and B TF32, both K-major, M = 128, N = 256.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// *out += sum (A B^T) * D.
__global__ void __launch_bounds__(128, 1)
abt_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
           const float* __restrict__ D, int64_t ldd, int M, int N, int Kd, double* __restrict__ out,
           int* __restrict__ err)
{
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[STAGES];
    __shared__ __align__(8) uint64_t empty_bar[STAGES];
    __shared__ __align__(8) uint64_t done_bar;
    __shared__ uint32_t tmem_slot;

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles = N / BN;
    const int m0 = (blockIdx.x / n_tiles) * BM;
    const int n0 = (blockIdx.x % n_tiles) * BN;
    const int k_iters = Kd / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&done_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_slot;
    bool ok = true;

    if (warp == 0 && lane == 0) {
        for (int it = 0; it < k_iters && ok; ++it) {
            const int s = it % STAGES;
            ok = mbar_wait(&empty_bar[s], ((it / STAGES) & 1) ^ 1);
            if (!ok) break;
            mbar_expect_tx(&full_bar[s], STAGE_BYTES);
            uint8_t* sa = smem + s * STAGE_BYTES;
            tma_load_2d(sa, &map_a, it * BK, m0, &full_bar[s]);
            tma_load_2d(sa + A_BYTES, &map_b, it * BK, n0, &full_bar[s]);
        }
        if (!ok) atomicExch(err, 1);
    } else if (warp == 1 && lane == 0) {
        for (int it = 0; it < k_iters && ok; ++it) {
            const int s = it % STAGES;
            ok = mbar_wait(&full_bar[s], (it / STAGES) & 1);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t a = smem_addr(smem + s * STAGE_BYTES);
            const uint64_t ad = smem_desc(a), bd = smem_desc(a + A_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / 8; ++kk)       // K = 8 tf32 = 32 bytes = +2 in the 16-byte address field
                mma_tf32(tmem, ad + 2 * kk, bd + 2 * kk, (it | kk) != 0);
            mma_commit(&empty_bar[s]);
        }
        if (ok) mma_commit(&done_bar);
        else atomicExch(err, 1);
    }
    __syncwarp();

    // Epilogue: all four warps, warp w reads accumulator rows 32w..32w+31.
    const bool ready = mbar_wait(&done_bar, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    double acc = 0.0;
    const bool go = __all_sync(0xFFFFFFFFu, ready && !*reinterpret_cast<volatile int*>(err));
    if (go) {
        const int row = m0 + warp * 32 + lane;
        const float* drow = D + (int64_t)row * ldd + n0;
        for (int c0 = 0; c0 < BN; c0 += 16) {
            uint32_t v[16];
            const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0;
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                  "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            {
                float part = 0.f;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 d = *reinterpret_cast<const float4*>(drow + c0 + 4 * q);
                    part += __uint_as_float(v[4 * q]) * d.x + __uint_as_float(v[4 * q + 1]) * d.y +
                            __uint_as_float(v[4 * q + 2]) * d.z + __uint_as_float(v[4 * q + 3]) * d.w;
                }
                acc += (double)part;
            }
        }
    } else if (threadIdx.x == 0) {
        atomicExch(err, 1);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_down_sync(0xFFFFFFFFu, acc, off);
    if (lane == 0 && acc != 0.0) atomicAdd(out, acc);

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// Store GEMM with a drained accumulator: D = alpha * sum_v A_v B_v^T + beta * D.
//
// The tensor-core accumulator is not an IEEE round-to-nearest fp32 adder;
// over thousands of K steps its error grows to ~1e-5 of the result.  This
// kernel therefore accumulates only a few k-tiles in tensor memory (128 K
// values, or 32 for X3, whose three products add 3x the terms), and the epilogue warps fold each such partial product into fp32
// registers (round-to-nearest adds), so the result carries the accuracy of
// an fp32 CUDA-core GEMM once the operands are exact in TF32 (the 3xTF32
// split).  Two 256-column TMEM buffers (all 512 columns) alternate: the MMA
// warp fills one while the epilogue drains the other.
//
// X3: the three products hi*lo + lo*hi + hi*hi of a 3xTF32 split run in one
// launch; pipeline iteration 3kt+v loads k-tile kt of (A_hi, B_lo), (A_lo,
// B_hi), (A_hi, B_hi) for v = 0, 1, 2 (small terms first, so they enter an
// accumulator of their own magnitude).
// SYM: D is square and symmetric (M == N); only output tiles that hold an
// element on or above the diagonal run, each writes its elements with
// col >= row directly and mirrors those with col > row to (col, row) with
// warp-coalesced stores.  Every element is written exactly once.
// Mr, Nr bound the written region (the operands may be zero-padded).
//
// 320 threads: warps 0..7 drain (warp w: TMEM lanes 32*(w%4).., columns
// 128*(w/4)..+127, 128 running sums per thread), warp 8 lane 0 issues TMA,
// warp 9 lane 0 issues tcgen05.mma.  All waits are bounded.
constexpr int SEG_KT = 4;      // k-tiles per drain, single product
constexpr int SEG_KT_X3 = 1;   // k-tiles per drain, 3xTF32
constexpr int SEG_THREADS = 320;

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

struct SegMaps {
    CUtensorMap a_hi, a_lo, b_hi, b_lo;
};

// Output tile of block b.  SYM (BN == 2 BM): column block ni holds row blocks
// 0 .. 2ni+1, enumerated column-major so neighbouring CTAs share a B tile.
template <bool SYM>
__device__ __forceinline__ void seg_tile(int b, int n_tiles, int& m0, int& n0) {
    if constexpr (SYM) {
        int ni = 0;
        while (b >= 2 * ni + 2) { b -= 2 * ni + 2; ++ni; }
        m0 = b * BM;
        n0 = ni * BN;
    } else {
        m0 = (b / n_tiles) * BM;
        n0 = (b % n_tiles) * BN;
    }
}

template <bool SYM, bool X3>
__global__ void __launch_bounds__(SEG_THREADS, 1)
abt_seg_kernel(const __grid_constant__ SegMaps maps, float* __restrict__ D, int64_t ldd, int Mr, int Nr, int N,
               int Kd, int* __restrict__ err, float alpha, float beta)
{
    constexpr int NV = X3 ? 3 : 1;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[STAGES];
    __shared__ __align__(8) uint64_t empty_bar[STAGES];
    __shared__ __align__(8) uint64_t seg_full[2];
    __shared__ __align__(8) uint64_t seg_empty[2];
    __shared__ uint32_t tmem_slot;

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int m0, n0;
    seg_tile<SYM>(blockIdx.x, N / BN, m0, n0);
    const int k_iters = Kd / BK * NV;
    const int seg_iters = X3 ? SEG_KT_X3 * 3 : SEG_KT;
    const int n_segs = (k_iters + seg_iters - 1) / seg_iters;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&seg_full[b], 1);
            mbar_init(&seg_empty[b], 8);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 8) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                     "r"(2 * kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_slot;

    if (warp == 8) {
        if (lane == 0) {
            bool ok = true;
            for (int it = 0; it < k_iters; ++it) {
                const int s = it % STAGES;
                if (!(ok = mbar_wait(&empty_bar[s], ((it / STAGES) & 1) ^ 1))) break;
                mbar_expect_tx(&full_bar[s], STAGE_BYTES);
                uint8_t* sa = smem + s * STAGE_BYTES;
                const int v = X3 ? it % 3 : 0;
                const int kx = (X3 ? it / 3 : it) * BK;
                tma_load_2d(sa, v == 1 ? &maps.a_lo : &maps.a_hi, kx, m0, &full_bar[s]);
                tma_load_2d(sa + A_BYTES, v == 0 ? &maps.b_lo : &maps.b_hi, kx, n0, &full_bar[s]);
            }
            if (!ok) atomicExch(err, 1);
        }
    } else if (warp == 9) {
        if (lane == 0) {
            bool ok = true;
            for (int seg = 0; seg < n_segs && ok; ++seg) {
                const int b = seg & 1;
                if (!(ok = mbar_wait(&seg_empty[b], ((seg >> 1) & 1) ^ 1))) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t acc = tmem + (uint32_t)(b * kTmemCols);
                const int it0 = seg * seg_iters, it_end = min(k_iters, it0 + seg_iters);
                for (int it = it0; it < it_end; ++it) {
                    const int s = it % STAGES;
                    if (!(ok = mbar_wait(&full_bar[s], (it / STAGES) & 1))) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t a = smem_addr(smem + s * STAGE_BYTES);
                    const uint64_t ad = smem_desc(a), bd = smem_desc(a + A_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 8; ++kk)
                        mma_tf32(acc, ad + 2 * kk, bd + 2 * kk, (it != it0 || kk != 0) ? 1u : 0u);
                    mma_commit(&empty_bar[s]);
                }
                if (ok) mma_commit(&seg_full[b]);
            }
            if (!ok) atomicExch(err, 1);
        }
    } else {
        // Drain warps.
        const int q = warp & 3, h = warp >> 2;
        float r[BN / 2];
#pragma unroll
        for (int i = 0; i < BN / 2; ++i) r[i] = 0.f;
        bool ok = true;
        for (int seg = 0; seg < n_segs; ++seg) {
            const int b = seg & 1;
            ok = __all_sync(0xFFFFFFFFu, mbar_wait(&seg_full[b], (seg >> 1) & 1));
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * kTmemCols + h * (BN / 2));
#pragma unroll
            for (int c0 = 0; c0 < BN / 2; c0 += 16) {
                uint32_t v[16];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                    : "r"(base + (uint32_t)c0));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int i = 0; i < 16; ++i) r[c0 + i] += __uint_as_float(v[i]);
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&seg_empty[b]);
        }
        if (ok && !*reinterpret_cast<volatile int*>(err)) {
            const int i = m0 + q * 32 + lane;
            const int j0 = n0 + h * (BN / 2);
            const bool vec = (ldd & 3) == 0 && (reinterpret_cast<uintptr_t>(D) & 15) == 0;
            // alpha == beta == 1 (accumulation): fire-and-forget reductions
            // (RED, round-to-nearest at L2); each element has one writer, so
            // the result equals a read-modify-write without its latency.
            const bool red = alpha == 1.f && beta == 1.f;
            if (i < Mr) {
                float* drow = D + (int64_t)i * ldd;
#pragma unroll
                for (int c = 0; c < BN / 2; c += 4) {
                    const int j = j0 + c;
                    if (vec && j + 3 < Nr && (!SYM || j >= i)) {
                        float4* dp = reinterpret_cast<float4*>(drow + j);
                        if (red) {
                            atomicAdd(dp, make_float4(r[c], r[c + 1], r[c + 2], r[c + 3]));
                        } else {
                            float4 d = make_float4(0.f, 0.f, 0.f, 0.f);
                            if (beta != 0.f) d = *dp;
                            d.x = alpha * r[c] + beta * d.x;
                            d.y = alpha * r[c + 1] + beta * d.y;
                            d.z = alpha * r[c + 2] + beta * d.z;
                            d.w = alpha * r[c + 3] + beta * d.w;
                            *dp = d;
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            if (j + e < Nr && (!SYM || j + e >= i)) {
                                float* dp = drow + j + e;
                                if (red) atomicAdd(dp, r[c + e]);
                                else *dp = alpha * r[c + e] + (beta != 0.f ? beta * *dp : 0.f);
                            }
                        }
                    }
                }
                if constexpr (SYM) {
                    // (col, row) for col > row: lanes hold consecutive rows, so
                    // each column is one coalesced 128-byte access per warp.
#pragma unroll
                    for (int c = 0; c < BN / 2; ++c) {
                        const int j = j0 + c;
                        if (j > i && j < Nr) {
                            float* dp = D + (int64_t)j * ldd + i;
                            if (red) atomicAdd(dp, r[c]);
                            else *dp = alpha * r[c] + (beta != 0.f ? beta * *dp : 0.f);
                        }
                    }
                }
            }
        } else if (lane == 0) {
            atomicExch(err, 1);
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 8) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kTmemCols));
    }
}

// Hessian operands from a chunk of samples x [T x d] (row stride ldx) and
// weights w [T] (NULL: all 1): the K-major operands A = x^T and B = (x w)^T,
// both [dpad x Tpad], zero-padded, each split into a TF32 high part
// (mantissa truncated to 10 bits) and the fp32 remainder (X3) or written
// whole.  64 x 64 tiles through shared memory; one read of x, 16-byte
// stores.
template <bool X3>
__global__ void __launch_bounds__(256) hess_operands_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                            int64_t T, int64_t d, int64_t ldx, int64_t Tpad,
                                                            float* __restrict__ a_hi, float* __restrict__ a_lo,
                                                            float* __restrict__ b_hi, float* __restrict__ b_lo) {
    constexpr int TT = 64;
    __shared__ float tile[TT][TT + 1];
    __shared__ float ws[TT];
    const int64_t t0 = (int64_t)blockIdx.x * TT, c0 = (int64_t)blockIdx.y * TT;
    const int tid = threadIdx.x;
    if (tid < TT) ws[tid] = (t0 + tid < T) ? (w ? w[t0 + tid] : 1.f) : 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int idx = tid + 256 * i;
        const int tt = idx >> 6, cc = idx & 63;
        const int64_t t = t0 + tt, c = c0 + cc;
        tile[tt][cc] = (t < T && c < d) ? __ldcs(x + t * ldx + c) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int idx = tid + 256 * i;
        const int cc = idx >> 4, ch = idx & 15;
        const int64_t off = (c0 + cc) * Tpad + t0 + ch * 4;
        float av[4], bv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            av[e] = tile[ch * 4 + e][cc];
            bv[e] = av[e] * ws[ch * 4 + e];
        }
        if constexpr (X3) {
            float ah[4], bh[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                ah[e] = __uint_as_float(__float_as_uint(av[e]) & 0xFFFFE000u);
                bh[e] = __uint_as_float(__float_as_uint(bv[e]) & 0xFFFFE000u);
            }
            __stcs(reinterpret_cast<float4*>(a_hi + off), make_float4(ah[0], ah[1], ah[2], ah[3]));
            __stcs(reinterpret_cast<float4*>(b_hi + off), make_float4(bh[0], bh[1], bh[2], bh[3]));
            __stcs(reinterpret_cast<float4*>(a_lo + off),
                   make_float4(av[0] - ah[0], av[1] - ah[1], av[2] - ah[2], av[3] - ah[3]));
            __stcs(reinterpret_cast<float4*>(b_lo + off),
                   make_float4(bv[0] - bh[0], bv[1] - bh[1], bv[2] - bh[2], bv[3] - bh[3]));
        } else {
            __stcs(reinterpret_cast<float4*>(a_hi + off), make_float4(av[0], av[1], av[2], av[3]));
            __stcs(reinterpret_cast<float4*>(b_hi + off), make_float4(bv[0], bv[1], bv[2], bv[3]));
        }
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

int make_map(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn) { set_error("cuTensorMapEncodeTiled unavailable"); return KQ_ERR_CUDA; }
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) { set_error("cuTensorMapEncodeTiled failed (%d)", (int)r); return KQ_ERR_CUDA; }
    return KQ_OK;
}

}  // namespace
}  // namespace kq

namespace kq {
namespace {

int check_abt(const float* A, const float* B, const float* D, int64_t M, int64_t N, int64_t Kd, int64_t ldd,
              const char* what) {
    if (!A || !B || !D) { set_error("%s: null pointer", what); return KQ_ERR_ARG; }
    if (M <= 0 || N <= 0 || Kd <= 0 || M % BM || N % BN || Kd % BK || ldd < N || ldd % 4) {
        set_error("%s: need M %% 128 == 0, N %% 256 == 0, Kd %% 32 == 0, ldd >= N, ldd %% 4 == 0 "
                  "(got M=%lld N=%lld Kd=%lld ldd=%lld)", what, (long long)M, (long long)N, (long long)Kd,
                  (long long)ldd);
        return KQ_ERR_ARG;
    }
    if (((uintptr_t)A | (uintptr_t)B | (uintptr_t)D) & 15) { set_error("%s: 16-byte alignment", what); return KQ_ERR_ALIGN; }
    if ((M / BM) * (N / BN) > 0x7FFFFFFF || M > 0x7FFFFFFF || N > 0x7FFFFFFF || Kd > 0x7FFFFFFF) {
        set_error("%s: problem too large", what);
        return KQ_ERR_ARG;
    }
    return KQ_OK;
}

int launch_trace(const float* A, const float* B, const float* D, int64_t M, int64_t N, int64_t Kd, int64_t ldd,
                 double* out, int* err, void* stream) {
    const char* what = "kq_trace_abt";
    if (int rc = check_abt(A, B, D, M, N, Kd, ldd, what)) return rc;
    if (!out || !err) { set_error("%s: null pointer", what); return KQ_ERR_ARG; }
    CUtensorMap ma, mb;
    if (int rc = make_map(&ma, A, M, Kd, BM)) return rc;
    if (int rc = make_map(&mb, B, N, Kd, BN)) return rc;
    cudaError_t e = cudaFuncSetAttribute(abt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) { set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e)); return KQ_ERR_CUDA; }
    abt_kernel<<<(int)((M / BM) * (N / BN)), 128, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(
        ma, mb, D, ldd, (int)M, (int)N, (int)Kd, out, err);
    return check_launch(what);
}

// A_lo / B_lo are used only when X3.  Grid: all tiles, or for SYM (M == N)
// the (N/256) (N/256 + 1) tiles that touch the upper triangle.
template <bool SYM, bool X3>
int launch_seg(const float* a_hi, const float* a_lo, const float* b_hi, const float* b_lo, float* D, int64_t M,
               int64_t N, int64_t Kd, int64_t ldd, int64_t Mr, int64_t Nr, int* err, float alpha, float beta,
               void* stream, const char* what) {
    SegMaps maps;
    if (int rc = make_map(&maps.a_hi, a_hi, M, Kd, BM)) return rc;
    if (int rc = make_map(&maps.b_hi, b_hi, N, Kd, BN)) return rc;
    if (int rc = make_map(&maps.a_lo, X3 ? a_lo : a_hi, M, Kd, BM)) return rc;
    if (int rc = make_map(&maps.b_lo, X3 ? b_lo : b_hi, N, Kd, BN)) return rc;
    const int64_t nt = N / BN;
    const int64_t grid = SYM ? nt * (nt + 1) : (M / BM) * nt;
    cudaError_t e = cudaFuncSetAttribute(abt_seg_kernel<SYM, X3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         SMEM_BYTES);
    if (e != cudaSuccess) { set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e)); return KQ_ERR_CUDA; }
    abt_seg_kernel<SYM, X3><<<(int)grid, SEG_THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(
        maps, D, ldd, (int)Mr, (int)Nr, (int)N, (int)Kd, err, alpha, beta);
    return check_launch(what);
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

}  // namespace
}  // namespace kq

extern "C" int kq_trace_abt(const float* A, const float* B, const float* D, int64_t M, int64_t N, int64_t Kd,
                            int64_t ldd, double* out, int* err, void* stream) {
    return kq::launch_trace(A, B, D, M, N, Kd, ldd, out, err, stream);
}

extern "C" int kq_gemm_abt_tf32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t Kd,
                                int64_t ldc, float alpha, float beta, int* err, void* stream) {
    using namespace kq;
    const char* what = "kq_gemm_abt_tf32";
    if (int rc = check_abt(A, B, C, M, N, Kd, ldc, what)) return rc;
    if (!err) { set_error("%s: null pointer", what); return KQ_ERR_ARG; }
    return launch_seg<false, false>(A, nullptr, B, nullptr, C, M, N, Kd, ldc, M, N, err, alpha, beta, stream, what);
}

extern "C" size_t kq_hessian_workspace_bytes(int64_t tokens, int64_t dim, int split) {
    if (tokens < 0 || dim <= 0 || (split != 1 && split != 3)) return 0;
    const int64_t tpad = kq::round_up(tokens > 0 ? tokens : 1, 64), dpad = kq::round_up(dim, kq::BN);
    return (size_t)(split == 3 ? 4 : 2) * (size_t)dpad * (size_t)tpad * sizeof(float);
}

extern "C" int kq_accumulate_hessian(const float* x, const float* w, int64_t tokens, int64_t dim, int64_t ldx,
                                     float* H, int64_t ldh, int split, void* workspace, size_t workspace_bytes,
                                     int* err, void* stream) {
    using namespace kq;
    const char* what = "kq_accumulate_hessian";
    if (tokens < 0 || dim <= 0 || ldx < dim || ldh < dim || (split != 1 && split != 3)) {
        set_error("%s: bad arguments (tokens=%lld dim=%lld ldx=%lld ldh=%lld split=%d)", what, (long long)tokens,
                  (long long)dim, (long long)ldx, (long long)ldh, split);
        return KQ_ERR_ARG;
    }
    if (tokens == 0) return KQ_OK;
    if (!x || !H || !err || !workspace) { set_error("%s: null pointer", what); return KQ_ERR_ARG; }
    const int64_t tpad = round_up(tokens, 64), dpad = round_up(dim, BN);
    if (dpad > (1 << 20) || tpad > 0x7FFFFFFF / 3) { set_error("%s: problem too large", what); return KQ_ERR_ARG; }
    if (workspace_bytes < kq_hessian_workspace_bytes(tokens, dim, split)) {
        set_error("%s: workspace too small", what);
        return KQ_ERR_WORKSPACE;
    }
    if ((uintptr_t)workspace & 15) { set_error("%s: workspace must be 16-byte aligned", what); return KQ_ERR_ALIGN; }
    float* ws = static_cast<float*>(workspace);
    const int64_t n = dpad * tpad;
    float *a_hi = ws, *b_hi = ws + n, *a_lo = ws + 2 * n, *b_lo = ws + 3 * n;
    dim3 grid((unsigned)(tpad / 64), (unsigned)(dpad / 64));
    if (grid.y > 65535) { set_error("%s: dim too large", what); return KQ_ERR_ARG; }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (split == 3)
        hess_operands_kernel<true><<<grid, 256, 0, s>>>(x, w, tokens, dim, ldx, tpad, a_hi, a_lo, b_hi, b_lo);
    else
        hess_operands_kernel<false><<<grid, 256, 0, s>>>(x, w, tokens, dim, ldx, tpad, a_hi, nullptr, b_hi, nullptr);
    if (int rc = check_launch("hess_operands_kernel")) return rc;
    if (split == 3)
        return launch_seg<true, true>(a_hi, a_lo, b_hi, b_lo, H, dpad, dpad, tpad, ldh, dim, dim, err, 1.f, 1.f,
                                      stream, what);
    return launch_seg<true, false>(a_hi, nullptr, b_hi, nullptr, H, dpad, dpad, tpad, ldh, dim, dim, err, 1.f, 1.f,
                                   stream, what);
}
