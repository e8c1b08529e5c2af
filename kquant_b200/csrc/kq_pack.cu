// Trellis bitstream packing in the native EXL word order, and its inverse.
//
// Per tile: 16 groups of 16 consecutive states.  The low K bits of each state
// are written MSB-first into a 16K-bit stream, which is cut into K uint16
// words.  The tile's 16K words are then swapped in adjacent pairs (SWAP16).
// This is the order pinned by the reference's golden prefixes
// (tests/test_qsrt.py:213-231) and restated in kquant/qsrt.py:811-857.
#include "kq_common.cuh"

namespace kq {
namespace {

__global__ void pack_kernel(const uint16_t* __restrict__ states, int64_t n, int K, uint16_t* __restrict__ packed) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // (tile, group)
    if (gid >= n * 16) return;
    const int64_t tile = gid >> 4;
    const int g = (int)(gid & 15);
    const uint4* src = reinterpret_cast<const uint4*>(states + tile * 256 + g * 16);
    uint4 a = __ldg(src), b = __ldg(src + 1);
    const uint32_t w32[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    const uint32_t mask = (1u << K) - 1u;
    unsigned __int128 S = 0;                 // 16K-bit big-endian stream
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const uint32_t v = (j & 1 ? (w32[j >> 1] >> 16) : w32[j >> 1]) & mask;
        S = (S << K) | v;
    }
    const int words = 16 * K;
    uint16_t* dst = packed + tile * words;
    for (int w = 0; w < K; ++w) {
        const uint16_t word = (uint16_t)(S >> (16 * (K - 1 - w)));
        dst[(g * K + w) ^ 1] = word;
    }
}

__global__ void unpack_states_kernel(const uint16_t* __restrict__ packed, int K, uint16_t* __restrict__ states) {
    __shared__ uint16_t flat[128];
    __shared__ uint16_t edges[256];
    const int64_t tile = blockIdx.x;
    const int i = threadIdx.x;
    const int words = 16 * K;
    if (i < words) flat[i] = packed[tile * words + (i ^ 1)];
    __syncthreads();
    const int g = i >> 4, j = i & 15;
    const int p = j * K;                          // bit position inside the group's stream
    const int w = g * K + (p >> 4);
    const uint32_t hi = flat[w];
    const uint32_t lo = ((p >> 4) + 1 < K) ? flat[w + 1] : 0u;
    const uint32_t win = (hi << 16) | lo;
    edges[i] = (uint16_t)((win >> (32 - (p & 15) - K)) & ((1u << K) - 1u));
    __syncthreads();
    uint32_t s = 0;
    const int lags = (16 + K - 1) / K;
    for (int lag = 0; lag < lags; ++lag) s |= (uint32_t)edges[(i - lag) & 255] << (lag * K);
    states[tile * 256 + i] = (uint16_t)(s & 0xFFFFu);
}

}  // namespace

int pack_trellis(const uint16_t* states, int64_t n, int K, uint16_t* packed, cudaStream_t stream) {
    if (K < 1 || K > 8) { set_error("pack_trellis: K must be in 1..8 (got %d)", K); return KQ_ERR_ARG; }
    if (n < 0 || (n > 0 && (!states || !packed))) { set_error("pack_trellis: bad arguments"); return KQ_ERR_ARG; }
    if (n == 0) return KQ_OK;
    if ((uintptr_t)states & 15) { set_error("pack_trellis: states must be 16-byte aligned"); return KQ_ERR_ALIGN; }
    const int64_t threads = n * 16;
    const int block = 256;
    pack_kernel<<<(unsigned)((threads + block - 1) / block), block, 0, stream>>>(states, n, K, packed);
    return check_launch("pack_kernel");
}

int unpack_trellis_states(const uint16_t* packed, int64_t n, int K, uint16_t* states, cudaStream_t stream) {
    if (K < 1 || K > 8) { set_error("unpack_trellis: K must be in 1..8 (got %d)", K); return KQ_ERR_ARG; }
    if (n < 0 || (n > 0 && (!states || !packed))) { set_error("unpack_trellis: bad arguments"); return KQ_ERR_ARG; }
    if (n == 0) return KQ_OK;
    if (n > 0x7FFFFFFF) { set_error("unpack_trellis: too many tiles"); return KQ_ERR_ARG; }
    unpack_states_kernel<<<(unsigned)n, 256, 0, stream>>>(packed, K, states);
    return check_launch("unpack_states_kernel");
}

}  // namespace kq
