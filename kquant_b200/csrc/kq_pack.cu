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

// One thread packs two 16-symbol groups (2g, 2g+1) of a tile: 64 bytes of
// states in, 2K words out.  2K words always start at an even index, so the
// SWAP16 pairs stay inside the thread and are written as K 32-bit words.
template <int K>
__global__ void pack_kernel(const uint16_t* __restrict__ states, int64_t n, uint16_t* __restrict__ packed) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // (tile, group pair)
    if (gid >= n * 8) return;
    const int64_t tile = gid >> 3;
    const int gp = (int)(gid & 7);
    const uint4* src = reinterpret_cast<const uint4*>(states + tile * 256 + gp * 32);
    uint4 q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = __ldcs(src + i);
    const uint32_t* w32 = reinterpret_cast<const uint32_t*>(q);
    const uint32_t mask = (1u << K) - 1u;
    uint32_t words[16];                      // 2K <= 16 words of this group pair, stream order
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        unsigned __int128 S = 0;             // 16K-bit big-endian stream of group 2gp+h
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const uint32_t word = w32[h * 8 + (j >> 1)];
            S = (S << K) | (((j & 1) ? (word >> 16) : word) & mask);
        }
#pragma unroll
        for (int w = 0; w < K; ++w) words[h * K + w] = (uint32_t)(S >> (16 * (K - 1 - w))) & 0xFFFFu;
    }
    // SWAP16: output word 2i holds stream word 2i+1 and vice versa, i.e. a
    // little-endian u32 of (stream[2i+1], stream[2i]) = (stream[2i] << 16) | stream[2i+1].
    uint32_t* dst = reinterpret_cast<uint32_t*>(packed + tile * 16 * K + gp * 2 * K);
#pragma unroll
    for (int i = 0; i < K; ++i) __stcs(dst + i, (words[2 * i] << 16) | words[2 * i + 1]);
}

// One warp per tile; lane l owns symbols 8l..8l+7.  Edges come from the
// lane's half of its group's stream; the cyclic closure needs the previous
// ceil(16/K)-1 edges (<= 7 for K >= 2, 15 for K = 1), taken from the one or
// two previous lanes, cyclically.
template <int K>
__global__ void unpack_states_kernel(const uint16_t* __restrict__ packed, int64_t n, uint16_t* __restrict__ states) {
    const int64_t tile = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (tile >= n) return;                   // whole warps exit together
    // The tile's 16K words are 8K 32-bit words: lanes 0..8K-1 load one each
    // (coalesced), then every lane gathers its group's K stream words by
    // shuffles.  Stream word w of group g is packed word (g K + w) ^ 1 (SWAP16).
    const uint32_t* src32 = reinterpret_cast<const uint32_t*>(packed + tile * 16 * K);
    uint32_t mine32 = 0;
    if (lane < 8 * K) mine32 = __ldcs(src32 + lane);
    uint32_t more32 = 0;                     // K > 4: 8K > 32 words, lanes take a second one
    if (K > 4 && lane + 32 < 8 * K) more32 = __ldcs(src32 + 32 + lane);
    const int g = lane >> 1, half = lane & 1;
    uint32_t win[K + 1];
#pragma unroll
    for (int w = 0; w < K; ++w) {
        const int idx = (g * K + w) ^ 1;     // 16-bit word index in the tile
        const int j = idx >> 1;              // its 32-bit word
        const uint32_t lo = __shfl_sync(0xFFFFFFFFu, mine32, j & 31);
        uint32_t v = lo;
        if (K > 4) {
            const uint32_t hi = __shfl_sync(0xFFFFFFFFu, more32, j & 31);
            v = (j >= 32) ? hi : lo;
        }
        win[w] = (idx & 1) ? (v >> 16) : (v & 0xFFFFu);
    }
    uint32_t e[8];
    const uint32_t mask = (1u << K) - 1u;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        const int p = (half * 8 + s) * K;    // bit position in the group's stream
        const int w = p >> 4;
        const uint32_t hi = win[w];
        const uint32_t lo = (w + 1 < K) ? win[w + 1] : 0u;
        e[s] = (((hi << 16) | lo) >> (32 - (p & 15) - K)) & mask;
    }
    // previous lane's 8 edges, packed 4 bits each (K <= 4 uses the low bits)
    uint32_t mine = 0;
#pragma unroll
    for (int s = 0; s < 8; ++s) mine |= (e[s] & 0xFu) << (4 * s);
    uint32_t mine_hi = 0;
#pragma unroll
    for (int s = 0; s < 8; ++s) mine_hi |= ((e[s] >> 4) & 0xFu) << (4 * s);
    const uint32_t prev = __shfl_sync(0xFFFFFFFFu, mine, (lane + 31) & 31);
    const uint32_t prev_hi = __shfl_sync(0xFFFFFFFFu, mine_hi, (lane + 31) & 31);
    const uint32_t prev2 = __shfl_sync(0xFFFFFFFFu, mine, (lane + 30) & 31);    // K = 1 reaches 15 back
    constexpr int lags = (16 + K - 1) / K;
    uint32_t out[8];
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        uint32_t st = 0;
#pragma unroll
        for (int lag = 0; lag < lags; ++lag) {
            const int t = s - lag;
            uint32_t ed;
            if (t >= 0) ed = e[t];
            else if (t >= -8) ed = ((prev >> (4 * (8 + t))) & 0xFu) | (((prev_hi >> (4 * (8 + t))) & 0xFu) << 4);
            else ed = (prev2 >> (4 * (16 + t))) & 0xFu;
            st |= ed << (lag * K);
        }
        out[s] = st & 0xFFFFu;
    }
    uint4 v = make_uint4(out[0] | (out[1] << 16), out[2] | (out[3] << 16), out[4] | (out[5] << 16),
                         out[6] | (out[7] << 16));
    __stcs(reinterpret_cast<uint4*>(states + tile * 256) + lane, v);
}

}  // namespace

int pack_trellis(const uint16_t* states, int64_t n, int K, uint16_t* packed, cudaStream_t stream) {
    if (K < 1 || K > 8) { set_error("pack_trellis: K must be in 1..8 (got %d)", K); return KQ_ERR_ARG; }
    if (n < 0 || (n > 0 && (!states || !packed))) { set_error("pack_trellis: bad arguments"); return KQ_ERR_ARG; }
    if (n == 0) return KQ_OK;
    if ((uintptr_t)states & 15) { set_error("pack_trellis: states must be 16-byte aligned"); return KQ_ERR_ALIGN; }
    if ((uintptr_t)packed & 3) { set_error("pack_trellis: packed must be 4-byte aligned"); return KQ_ERR_ALIGN; }
    const int64_t threads = n * 8;
    const int block = 256;
    const unsigned grid = (unsigned)((threads + block - 1) / block);
    switch (K) {
    case 1: pack_kernel<1><<<grid, block, 0, stream>>>(states, n, packed); break;
    case 2: pack_kernel<2><<<grid, block, 0, stream>>>(states, n, packed); break;
    case 3: pack_kernel<3><<<grid, block, 0, stream>>>(states, n, packed); break;
    case 4: pack_kernel<4><<<grid, block, 0, stream>>>(states, n, packed); break;
    case 5: pack_kernel<5><<<grid, block, 0, stream>>>(states, n, packed); break;
    case 6: pack_kernel<6><<<grid, block, 0, stream>>>(states, n, packed); break;
    case 7: pack_kernel<7><<<grid, block, 0, stream>>>(states, n, packed); break;
    default: pack_kernel<8><<<grid, block, 0, stream>>>(states, n, packed); break;
    }
    return check_launch("pack_kernel");
}

int unpack_trellis_states(const uint16_t* packed, int64_t n, int K, uint16_t* states, cudaStream_t stream) {
    if (K < 1 || K > 8) { set_error("unpack_trellis: K must be in 1..8 (got %d)", K); return KQ_ERR_ARG; }
    if (n < 0 || (n > 0 && (!states || !packed))) { set_error("unpack_trellis: bad arguments"); return KQ_ERR_ARG; }
    if (n == 0) return KQ_OK;
    if ((uintptr_t)states & 15) { set_error("unpack_trellis: states must be 16-byte aligned"); return KQ_ERR_ALIGN; }
    if ((uintptr_t)packed & 3) { set_error("unpack_trellis: packed must be 4-byte aligned"); return KQ_ERR_ALIGN; }
    const int64_t threads = n * 32;
    const unsigned grid = (unsigned)((threads + 255) / 256);
    switch (K) {
    case 1: unpack_states_kernel<1><<<grid, 256, 0, stream>>>(packed, n, states); break;
    case 2: unpack_states_kernel<2><<<grid, 256, 0, stream>>>(packed, n, states); break;
    case 3: unpack_states_kernel<3><<<grid, 256, 0, stream>>>(packed, n, states); break;
    case 4: unpack_states_kernel<4><<<grid, 256, 0, stream>>>(packed, n, states); break;
    case 5: unpack_states_kernel<5><<<grid, 256, 0, stream>>>(packed, n, states); break;
    case 6: unpack_states_kernel<6><<<grid, 256, 0, stream>>>(packed, n, states); break;
    case 7: unpack_states_kernel<7><<<grid, 256, 0, stream>>>(packed, n, states); break;
    default: unpack_states_kernel<8><<<grid, 256, 0, stream>>>(packed, n, states); break;
    }
    return check_launch("unpack_states_kernel");
}

}  // namespace kq
