// Reconstruction of encoded weights in the original basis (row W):
//     out = had_r(had_l(What) * su) * sv
// had_l / had_r: 128-row / 128-column block Hadamard (Sylvester order,
// normalised 1/sqrt(128)), the decoder's contract in
// kquant/exl3_reference.py:195-230 and kquant/exl3_encoder_backend.py:2211-2216.
//
// One CTA per 128 x 128 block, HBM-bound (one read and one write of the
// block).  The left transform's first five butterfly stages run in registers
// (a thread holds 32 rows of one column), its last two while the rows are
// read back from shared memory; the right transform runs per row in
// registers, a warp holding a row as float4 per lane (two butterfly stages
// inside the lane, five across lanes by shuffles).  Both 1/sqrt(128) factors
// are applied once, as one exact 1/128 scaling.
#include "kq_common.cuh"

namespace kq {
namespace {

constexpr int kHB = 128;          // Hadamard block
constexpr int kHThreads = 512;
constexpr int kHStride = kHB + 4; // shared-memory row stride (floats), keeps float4 rows aligned

__global__ void __launch_bounds__(kHThreads)
reconstruct_kernel(const float* __restrict__ wq, const float* __restrict__ su, const float* __restrict__ sv,
                   int64_t n, float* __restrict__ out) {
    extern __shared__ __align__(16) float blk[];          // [128][kHStride]
    const int tid = threadIdx.x;
    const int64_t r0 = (int64_t)blockIdx.y * kHB, c0 = (int64_t)blockIdx.x * kHB;
    // Left transform, bits 0..4 of the row index: thread (column c, quarter q)
    // holds rows 32 q .. 32 q + 31 of its column in registers (a warp reads
    // 32 consecutive columns of a row per load).
    {
        const int c = tid & (kHB - 1), q = tid >> 7;
        float x[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = __ldcs(wq + (r0 + q * 32 + i) * n + c0 + c);
#pragma unroll
        for (int h = 1; h < 32; h <<= 1)
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (!(i & h)) {
                    const float a = x[i], b = x[i + h];
                    x[i] = a + b;
                    x[i + h] = a - b;
                }
#pragma unroll
        for (int i = 0; i < 32; ++i) blk[(q * 32 + i) * kHStride + c] = x[i];
    }
    __syncthreads();
    // Bits 5 and 6 of the row index (rows r, r + 32, r + 64, r + 96), then the
    // row scale su and the right transform per row: lane l holds columns
    // 4l .. 4l + 3 (two stages inside the lane, five across lanes by shuffles).
    const int warp = tid >> 5, lane = tid & 31;
    const float4 s4 = __ldg(reinterpret_cast<const float4*>(sv + c0) + lane);
    constexpr float kScale = 1.0f / 128.0f;
    for (int r = warp; r < 32; r += kHThreads / 32) {
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = *reinterpret_cast<const float4*>(blk + (r + 32 * j) * kHStride + 4 * lane);
        float y[4][4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float v0 = (&v[0].x)[e], v1 = (&v[1].x)[e], v2 = (&v[2].x)[e], v3 = (&v[3].x)[e];
            const float a0 = v0 + v1, a1 = v0 - v1, a2 = v2 + v3, a3 = v2 - v3;
            y[0][e] = a0 + a2;
            y[2][e] = a0 - a2;
            y[1][e] = a1 + a3;
            y[3][e] = a1 - a3;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int row = r + 32 * j;
            const float u = __ldg(su + r0 + row);
            float x0 = y[j][0] * u, x1 = y[j][1] * u, x2 = y[j][2] * u, x3 = y[j][3] * u;
            float z0 = x0 + x1, z1 = x0 - x1, z2 = x2 + x3, z3 = x2 - x3;
            x0 = z0 + z2; x2 = z0 - z2; x1 = z1 + z3; x3 = z1 - z3;
#pragma unroll
            for (int m = 1; m < 32; m <<= 1) {
                const float o0 = __shfl_xor_sync(0xFFFFFFFFu, x0, m);
                const float o1 = __shfl_xor_sync(0xFFFFFFFFu, x1, m);
                const float o2 = __shfl_xor_sync(0xFFFFFFFFu, x2, m);
                const float o3 = __shfl_xor_sync(0xFFFFFFFFu, x3, m);
                const bool hi = lane & m;                     // this lane holds the "+ h" element
                x0 = hi ? o0 - x0 : x0 + o0;
                x1 = hi ? o1 - x1 : x1 + o1;
                x2 = hi ? o2 - x2 : x2 + o2;
                x3 = hi ? o3 - x3 : x3 + o3;
            }
            const float4 o = make_float4(x0 * kScale * s4.x, x1 * kScale * s4.y, x2 * kScale * s4.z,
                                         x3 * kScale * s4.w);
            __stcs(reinterpret_cast<float4*>(out + (r0 + row) * n + c0) + lane, o);
        }
    }
}

}  // namespace

int reconstruct_rotated(const float* wq, const float* su, const float* sv, int64_t k, int64_t n, float* out,
                        cudaStream_t stream) {
    if (!wq || !su || !sv || !out || k <= 0 || n <= 0 || k % kHB || n % kHB) {
        set_error("reconstruct: bad arguments (k=%lld n=%lld; both must be multiples of 128)", (long long)k,
                  (long long)n);
        return KQ_ERR_ARG;
    }
    if (((uintptr_t)wq | (uintptr_t)out | (uintptr_t)sv) & 15) {
        set_error("reconstruct: What, out and sv must be 16-byte aligned");
        return KQ_ERR_ALIGN;
    }
    if (k / kHB > 65535) { set_error("reconstruct: k too large"); return KQ_ERR_ARG; }
    const size_t sm = (size_t)kHB * kHStride * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(reconstruct_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) { set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e)); return KQ_ERR_CUDA; }
    const dim3 grid((unsigned)(n / kHB), (unsigned)(k / kHB));
    reconstruct_kernel<<<grid, kHThreads, sm, stream>>>(wq, su, sv, n, out);
    return check_launch("reconstruct_kernel");
}

}  // namespace kq

extern "C" int kq_reconstruct_rotated(const float* wq, const float* su, const float* sv, int64_t k, int64_t n,
                                      float* out, void* stream) {
    return kq::reconstruct_rotated(wq, su, sv, k, n, out, static_cast<cudaStream_t>(stream));
}
