// Test harness (oracle infrastructure only; never linked into the product).
//
// Compiles the reference's own tile-encoder translation unit
// (kquant/csrc/sqg_quantize.cu, which includes qsrt_quantize_tiles_kernel.cuh)
// where it lies in the reference tree, and exposes its launcher for every
// K in 1..8 with the procedural codebooks.  The reference template is written
// for any K (qsrt_quantize_tiles_kernel.cuh:14-21, 39-45, 186-194, 435-437);
// only its host binding restricts K to 2..4 (sqg_quantize.cu:190, 286).  The
// launch parameters (threads, shared memory, batch) are the binding's own
// (sqg_quantize.cu:124-159, 300-318).  Parity for K outside 2..4 is therefore
// pinned to the reference kernel's code, not to a reference test.
#include "sqg_quantize.cu"

extern "C" int kqref_quantize_procedural(const float* input, float* output, uint16_t* indices, void* costs,
                                         void* edges, int tiles, int max_batch, int K, int codebook,
                                         int tailbite_context, void* stream) {
    const int edges_per_state = 65536 >> K;
    const int shared_memory = 2 * edges_per_state * static_cast<int>(sizeof(half)) + 512 + 64 + 128;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    half* c = static_cast<half*>(costs);
    uint8_t* e = static_cast<uint8_t*>(edges);
#define KQREF_CASE(KV)                                                                                          \
    case KV:                                                                                                    \
        if (codebook == 1)                                                                                      \
            launch_trellis<KV, 1>(input, output, indices, c, e, tiles, max_batch, shared_memory,               \
                                  tailbite_context, s);                                                         \
        else                                                                                                    \
            launch_trellis<KV, 2>(input, output, indices, c, e, tiles, max_batch, shared_memory,               \
                                  tailbite_context, s);                                                         \
        break;
    switch (K) {
        KQREF_CASE(1)
        KQREF_CASE(2)
        KQREF_CASE(3)
        KQREF_CASE(4)
        KQREF_CASE(5)
        KQREF_CASE(6)
        KQREF_CASE(7)
        KQREF_CASE(8)
        default: return -1;
    }
#undef KQREF_CASE
    return static_cast<int>(cudaGetLastError());
}

// Bytes of the decision rows the reference kernel uses per tile at rate K
// (sqg_quantize.cu:201, qsrt_quantize_tiles_kernel.cuh:42-43).
extern "C" long long kqref_decision_bytes_per_tile(int K) {
    const int edges = 65536 >> K;
    const int per_row = K == 2 ? edges / 4 : (K <= 4 ? edges / 2 : edges);
    return 256LL * per_row;
}
