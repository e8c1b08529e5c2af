// Helpers shared by the Viterbi kernels (tie order of the primer argmin).
#pragma once
#include "kq_common.cuh"

namespace kq {

enum ViterbiPhase : int { PH_IDLE = 0, PH_FP, PH_AM, PH_TP, PH_FF, PH_TF, PH_OUT };

__device__ __forceinline__ uint32_t brev5(uint32_t x) { return __brev(x) >> 27; }

// Tie key of node e in the reference's primer argmin order (smaller wins):
// (bitrev5(reduction slot), bitrev5(lane), per-thread scan index j), the
// order produced by the strict-less __shfl_down_sync tournaments of
// kquant/csrc/qsrt_quantize_tiles_kernel.cuh:330-413.
template <int K>
__device__ __forceinline__ uint32_t tie_key(int e) {
    if constexpr (K == 2) {
        const int t = e & 1023, j = e >> 10;
        return (brev5(t >> 5) << 9) | (brev5(t & 31) << 4) | j;
    } else {
        const int t = e & 511, s = (e >> 9) & 1, j = e >> 10;
        return (brev5(16 * s + (t >> 5)) << 9) | (brev5(t & 31) << 4) | j;
    }
}

template <int K>
__device__ __forceinline__ int key_node(uint32_t key) {
    const int j = key & 15;
    const int lane = brev5((key >> 4) & 31);
    const int slot = brev5((key >> 9) & 31);
    if constexpr (K == 2) return ((slot << 5) | lane) + (j << 10);
    else return (((slot & 15) << 5) | lane) + ((slot >> 4) << 9) + (j << 10);
}

// Tie key for any K in 1..8 (the wide kernel): K2 as above; every other K
// takes the reference's 512-thread two-stream scan (e = thread + 512 s +
// 1024 j, j up to 31 at K1), so j gets five bits.
template <int K>
__device__ __forceinline__ uint32_t wide_tie_key(int e) {
    if constexpr (K == 2) {
        return tie_key<2>(e);
    } else {
        const int t = e & 511, s = (e >> 9) & 1, j = e >> 10;
        return (brev5(16 * s + (t >> 5)) << 10) | (brev5(t & 31) << 5) | j;
    }
}

template <int K>
__device__ __forceinline__ int wide_key_node(uint32_t key) {
    if constexpr (K == 2) {
        return key_node<2>(key);
    } else {
        const int j = key & 31;
        const int lane = brev5((key >> 5) & 31);
        const int slot = brev5((key >> 10) & 31);
        return (((slot & 15) << 5) | lane) + ((slot >> 4) << 9) + (j << 10);
    }
}

}  // namespace kq
