// bf16 weight [rows x cols] (HF [out, in]) -> fp32 [cols x rows] (EXL [in, out]),
// optionally gathering rows through a permutation: dst[c][r] = float(src[perm[r]][c]).
// HBM-bound: 64 x 64 tiles staged through shared memory, 16-byte loads of
// 8 bf16 and 16-byte stores of 4 fp32, both coalesced.  The conversion is
// exact (bf16 widens to fp32).
#include <cuda_bf16.h>
#include "kq_common.cuh"

namespace kq {
namespace {

constexpr int T = 64;

__global__ void __launch_bounds__(256) bf16_t_f32_kernel(const __nv_bfloat16* __restrict__ src, int64_t rows,
                                                         int64_t cols, int64_t ld, const int64_t* __restrict__ perm,
                                                         float* __restrict__ dst) {
    __shared__ float tile[T][T + 1];
    const int64_t r0 = (int64_t)blockIdx.y * T, c0 = (int64_t)blockIdx.x * T;
    const int tid = threadIdx.x;
    // load: 64 rows x 8 chunks of 8 bf16
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int idx = tid + 256 * i;
        const int rr = idx >> 3, ch = idx & 7;
        const int64_t r = r0 + rr;
        if (r < rows) {
            const int64_t sr = perm ? perm[r] : r;
            const int64_t c = c0 + ch * 8;
            if (c + 8 <= cols) {
                const uint4 v = __ldcs(reinterpret_cast<const uint4*>(src + sr * ld + c));
                const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float2 f = __bfloat1622float2(h[q]);
                    tile[rr][ch * 8 + 2 * q] = f.x;
                    tile[rr][ch * 8 + 2 * q + 1] = f.y;
                }
            } else {
                for (int q = 0; q < 8 && c + q < cols; ++q) tile[rr][ch * 8 + q] = __bfloat162float(src[sr * ld + c + q]);
            }
        }
    }
    __syncthreads();
    // store: 64 dst rows (source columns) x 16 chunks of 4 fp32
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int idx = tid + 256 * i;
        const int cc = idx >> 4, ch = idx & 15;
        const int64_t c = c0 + cc, r = r0 + ch * 4;
        if (c < cols) {
            if (r + 4 <= rows && (rows & 3) == 0) {
                __stcs(reinterpret_cast<float4*>(dst + c * rows + r),
                       make_float4(tile[ch * 4][cc], tile[ch * 4 + 1][cc], tile[ch * 4 + 2][cc], tile[ch * 4 + 3][cc]));
            } else {
                for (int q = 0; q < 4 && r + q < rows; ++q) dst[c * rows + r + q] = tile[ch * 4 + q][cc];
            }
        }
    }
}

}  // namespace
}  // namespace kq

extern "C" int kq_bf16_to_f32_transposed(const uint16_t* src, int64_t rows, int64_t cols, int64_t ld_src,
                                         const int64_t* row_perm, float* dst, void* stream) {
    using namespace kq;
    if (rows < 0 || cols < 0 || ld_src < cols || (rows * cols > 0 && (!src || !dst))) {
        set_error("kq_bf16_to_f32_transposed: bad arguments");
        return KQ_ERR_ARG;
    }
    if (rows == 0 || cols == 0) return KQ_OK;
    if (((uintptr_t)src & 15) || (ld_src & 7) || ((uintptr_t)dst & 15)) {
        set_error("kq_bf16_to_f32_transposed: src/dst must be 16-byte aligned and ld_src a multiple of 8");
        return KQ_ERR_ALIGN;
    }
    if ((rows + T - 1) / T > 65535) { set_error("kq_bf16_to_f32_transposed: too many rows"); return KQ_ERR_ARG; }
    dim3 grid((unsigned)((cols + T - 1) / T), (unsigned)((rows + T - 1) / T));
    bf16_t_f32_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const __nv_bfloat16*>(src), rows, cols, ld_src, row_perm, dst);
    return check_launch("bf16_t_f32_kernel");
}
