// Tail-biting Viterbi tile encoder for the 16-bit bitshift trellis, sm_100a.
//
// Semantics follow kquant/csrc/qsrt_quantize_tiles_kernel.cuh:21-471 bit for
// bit.  Node e at step i keeps cost
//   cost_i[e] = min_k fma(L(t_k) - w, L(t_k) - w, cost_{i-1}[p_k])
// in binary16, where t_k = (k << (16-K)) | e is the 16-bit state and
// p_k = (k << (16-2K)) | (e >> K) its predecessor node.  The lowest k wins a
// tie.  A primer pass over 2C steps around position 0 picks the cyclic end
// state.  The final pass over the 256 steps is constrained to start from it.
//
// The layout is B200-first, not the reference's:
//  * One persistent 512-thread CTA per SM.  All 65,536 labels of the codebook
//    live in registers: each thread owns 8 (K4), 16 (K3) or 32 (K2) nodes
//    (ThreadMap) and holds 64 half2 labels, one per owned node pair and
//    predecessor.  The inner
//    loop therefore has no codebook loads or decodes.  It is 5 half2/logic
//    instructions per 2 relaxations with decisions, and 3 without.
//  * Nodes sharing e >> K share all 2^K predecessors (one 2^K x 2^K butterfly
//    block).  A thread owns whole butterfly halves, so each predecessor cost
//    is one shared-memory broadcast load reused for 8 relaxations.
//  * Two tiles ("jobs") are in flight per CTA.  Each 512-thread step slot
//    runs one forward step of one job; the job with the shortest remaining
//    forward phase goes first.  The sequential tracebacks (one dependent
//    global load per step) advance one step per slot, so their latency hides
//    under the other job's forward step.
//  * Decisions go to global memory in a per-thread-word layout, written
//    coalesced and with an evict-first hint.  The traceback reads one word
//    per step.
//  * The primer argmin reproduces the reference's shuffle-tree tie order
//    exactly.  It is a plain u32 min over (cost_bits << 16 | tie_key(e)),
//    where tie_key orders nodes by (bitrev5(slot), bitrev5(lane), j) of the
//    reference reduction (:330-413).
#include <type_traits>
#include "kq_viterbi_common.cuh"

namespace kq {
namespace {

constexpr int kThreads = 512;
constexpr int kJobs = 2;
constexpr int kTbThread = 0;

template <int K>
struct ThreadMap {
    static constexpr int NODES = 1 << (16 - K);
    static constexpr int Q = 1 << K;                  // predecessors per node
    static constexpr int DSHIFT = 16 - 2 * K;         // predecessor = (k << DSHIFT) | (e >> K)
    static constexpr int G = (K == 4) ? 1 : (K == 3 ? 2 : 8);   // butterfly blocks per thread
    static constexpr int P = (K == 2) ? 2 : 4;        // node pairs per block
    static constexpr int DB = (K == 2) ? 2 : 4;       // decision bits per node
    static constexpr int WORD_BYTES = (K == 4) ? 4 : 8;
    static constexpr int ROW_BYTES = kThreads * WORD_BYTES;
    using Word = typename std::conditional<K == 4, unsigned int, unsigned long long>::type;

    // First node of block g owned by thread tid (always even, 8- or 16-byte aligned).
    __device__ static __forceinline__ int base(int tid, int g) {
        if constexpr (K == 4) return ((tid >> 1) << 4) | ((tid & 1) << 3);
        else return (tid + kThreads * g) << K;
    }
    // Thread owning node e, and the bit position of e's decision in its word.
    __device__ static __forceinline__ void locate(int e, int& tid, int& bit) {
        if constexpr (K == 4) {
            tid = ((e >> 4) << 1) | ((e >> 3) & 1);
            bit = 4 * (e & 7);
        } else {
            const int h = e >> K;
            tid = h & (kThreads - 1);
            bit = (h >> 9) * (2 * P * DB) + (e & (2 * P - 1)) * DB;
        }
    }
};

// One forward step of one tile.  STEP0: 0 = read cost_prev, 1 = virtual zero
// costs (primer step 0), 2 = zero at es and +inf elsewhere (final step 0).
template <int K, bool DEC, int STEP0>
__device__ __forceinline__ void fwd_step(
    const half2 (&L)[ThreadMap<K>::G][ThreadMap<K>::P][ThreadMap<K>::Q],
    const __half* __restrict__ cprev, __half* __restrict__ cnext, half2 w2, int es,
    typename ThreadMap<K>::Word* __restrict__ decrow, int tid)
{
    using M = ThreadMap<K>;
    typename M::Word word = 0;
    const half2 zero2 = __float2half2_rn(0.f);
    const half2 inf2 = __halves2half2(__ushort_as_half(KQ_H_INF_BITS), __ushort_as_half(KQ_H_INF_BITS));
#pragma unroll
    for (int g = 0; g < M::G; ++g) {
        const int e0 = M::base(tid, g);
        const int h = e0 >> K;
        half2 mn[M::P];
        uint32_t id[M::P];
#pragma unroll
        for (int k = 0; k < M::Q; ++k) {
            const int pk = (k << M::DSHIFT) | h;
            half2 c2;
            if constexpr (STEP0 == 0) c2 = __half2half2(cprev[pk]);
            else if constexpr (STEP0 == 1) c2 = zero2;
            else c2 = (pk == es) ? zero2 : inf2;
#pragma unroll
            for (int p = 0; p < M::P; ++p) {
                const half2 dh = __hsub2(L[g][p][k], w2);
                const half2 err = __hfma2(dh, dh, c2);
                if (k == 0) {
                    mn[p] = err;
                    if constexpr (DEC) id[p] = 0u;
                } else {
                    if constexpr (DEC) {
                        const uint32_t lt = __hlt2_mask(err, mn[p]);
                        id[p] = (lt & (uint32_t)(k * 0x10001)) | (~lt & id[p]);
                    }
                    mn[p] = __hmin2(err, mn[p]);
                }
            }
        }
        if constexpr (M::P == 4) {
            uint4 v;
            v.x = *reinterpret_cast<uint32_t*>(&mn[0]);
            v.y = *reinterpret_cast<uint32_t*>(&mn[1]);
            v.z = *reinterpret_cast<uint32_t*>(&mn[2]);
            v.w = *reinterpret_cast<uint32_t*>(&mn[3]);
            *reinterpret_cast<uint4*>(cnext + e0) = v;
        } else {
            uint2 v;
            v.x = *reinterpret_cast<uint32_t*>(&mn[0]);
            v.y = *reinterpret_cast<uint32_t*>(&mn[1]);
            *reinterpret_cast<uint2*>(cnext + e0) = v;
        }
        if constexpr (DEC) {
#pragma unroll
            for (int p = 0; p < M::P; ++p) {
                const uint32_t lo = id[p] & 0xFFFFu, hi = id[p] >> 16;
                const int b = g * (2 * M::P * M::DB) + 2 * p * M::DB;
                word |= (typename M::Word)lo << b;
                word |= (typename M::Word)hi << (b + M::DB);
            }
        }
    }
    if constexpr (DEC) __stcs(decrow + tid, word);
}

template <int K>
__global__ void __launch_bounds__(kThreads, 1)
viterbi_kernel(const float* __restrict__ tiles, int64_t n_tiles, const uint32_t* __restrict__ labels32,
               const __half* __restrict__ labels16, int C, int njobs,
               float* __restrict__ out_vals, uint16_t* __restrict__ out_states,
               uint8_t* __restrict__ decisions)
{
    using M = ThreadMap<K>;
    using Word = typename M::Word;
    extern __shared__ __align__(16) uint8_t smem[];
    __half* cost = reinterpret_cast<__half*>(smem);                 // [kJobs][2][NODES]
    __half* wsh = cost + kJobs * 2 * M::NODES;                      // [kJobs][256]
    uint16_t* enc = reinterpret_cast<uint16_t*>(wsh + kJobs * 256); // [kJobs][256]
    uint32_t* red = reinterpret_cast<uint32_t*>(enc + kJobs * 256); // [kJobs][16]
    int* es_sh = reinterpret_cast<int*>(red + kJobs * 16);          // [kJobs]

    const int tid = threadIdx.x;
    const bool tbt = (tid == kTbThread);

    // Labels of every (node pair, predecessor) this thread owns.
    half2 L[M::G][M::P][M::Q];
#pragma unroll
    for (int g = 0; g < M::G; ++g)
#pragma unroll
        for (int p = 0; p < M::P; ++p)
#pragma unroll
            for (int k = 0; k < M::Q; ++k) {
                const uint32_t t = ((uint32_t)k << (16 - K)) | (uint32_t)(M::base(tid, g) + 2 * p);
                const uint32_t v = __ldg(labels32 + (t >> 1));
                L[g][p][k] = *reinterpret_cast<const half2*>(&v);
            }

    Word* dec_base = reinterpret_cast<Word*>(decisions + (size_t)blockIdx.x * kJobs * 256 * M::ROW_BYTES);

    int phase[kJobs], step[kJobs], par[kJobs];
    int64_t tile[kJobs];
    int64_t taken = 0;
    int node[kJobs];                       // traceback thread only
#pragma unroll
    for (int j = 0; j < kJobs; ++j) {
        const int64_t t = (int64_t)blockIdx.x + (int64_t)gridDim.x * taken;
        tile[j] = t;
        step[j] = 0;
        par[j] = 0;
        node[j] = 0;
        if (j < njobs && t < n_tiles) {
            phase[j] = PH_FP;
            ++taken;
            if (tid < 256) wsh[j * 256 + tid] = __float2half_rn(tiles[t * 256 + tid]);
        } else {
            phase[j] = PH_IDLE;
        }
    }
    __syncthreads();

    while (true) {
        bool any = false;
#pragma unroll
        for (int j = 0; j < kJobs; ++j) any |= (phase[j] != PH_IDLE);
        if (!any) break;

        // Forward job: shortest remaining forward phase first.
        int F = -1, F_rem = 1 << 30;
#pragma unroll
        for (int j = 0; j < kJobs; ++j) {
            if (phase[j] == PH_FP || phase[j] == PH_FF) {
                const int rem = (phase[j] == PH_FP ? 2 * C : 256) - step[j];
                if (rem < F_rem) { F_rem = rem; F = j; }
            }
        }

        // Traceback: issue this slot's loads early.
        Word tbw[kJobs];
        int tbrow[kJobs];
        if (tbt) {
#pragma unroll
            for (int j = 0; j < kJobs; ++j) {
                tbw[j] = 0;
                tbrow[j] = 0;
                if (phase[j] == PH_TP || phase[j] == PH_TF) {
                    if (phase[j] == PH_TP && step[j] == 0) {
                        uint32_t best = 0xFFFFFFFFu;
                        for (int w = 0; w < kThreads / 32; ++w) best = min(best, red[j * 16 + w]);
                        node[j] = key_node<K>(best & 0xFFFFu);
                    }
                    const int row = (phase[j] == PH_TP) ? (C - 1 - step[j]) : (255 - step[j]);
                    int owner, bit;
                    M::locate(node[j], owner, bit);
                    tbrow[j] = row;
                    tbw[j] = __ldcg(dec_base + ((size_t)j * 256 + row) * kThreads + owner);
                }
            }
        }

        // Primer argmin over the second-to-last primer step (reference quirk).
#pragma unroll
        for (int j = 0; j < kJobs; ++j) {
            if (phase[j] == PH_AM) {
                const __half* c = cost + (j * 2 + (par[j] ^ 1)) * M::NODES;
                uint32_t best = 0xFFFFFFFFu;
#pragma unroll
                for (int g = 0; g < M::G; ++g)
#pragma unroll
                    for (int q = 0; q < 2 * M::P; ++q) {
                        const int e = M::base(tid, g) + q;
                        const uint32_t key = ((uint32_t)__half_as_ushort(c[e]) << 16) | tie_key<K>(e);
                        best = min(best, key);
                    }
                best = __reduce_min_sync(0xFFFFFFFFu, best);
                if ((tid & 31) == 0) red[j * 16 + (tid >> 5)] = best;
            }
        }

        // Next tile of every job that finishes this slot (uniform).
        int64_t tnext[kJobs];
        {
            int64_t cnt = taken;
#pragma unroll
            for (int j = 0; j < kJobs; ++j) {
                tnext[j] = n_tiles;
                if (phase[j] == PH_OUT) {
                    const int64_t t = (int64_t)blockIdx.x + (int64_t)gridDim.x * cnt;
                    if (t < n_tiles) { tnext[j] = t; ++cnt; }
                }
            }
        }

        // Output of a finished tile, and the next tile's values.
#pragma unroll
        for (int j = 0; j < kJobs; ++j) {
            if (phase[j] == PH_OUT && tid < 256) {
                const uint16_t s = enc[j * 256 + tid];
                out_states[tile[j] * 256 + tid] = s;
                out_vals[tile[j] * 256 + tid] = __half2float(labels16[s]);
                if (tnext[j] < n_tiles) wsh[j * 256 + tid] = __float2half_rn(tiles[tnext[j] * 256 + tid]);
            }
        }

        // Forward step.
        if (F >= 0) {
            const int ph = phase[F], i = step[F];
            const int ri = (ph == PH_FP) ? ((i + 256 - C) & 255) : i;
            const bool dec = (ph == PH_FF) || (i >= C);
            const __half* cprev = cost + (F * 2 + par[F]) * M::NODES;
            __half* cnext = cost + (F * 2 + (par[F] ^ 1)) * M::NODES;
            const half2 w2 = __half2half2(wsh[F * 256 + ri]);
            Word* drow = dec_base + ((size_t)F * 256 + ri) * kThreads;
            if (i == 0) {
                if (ph == PH_FP) fwd_step<K, false, 1>(L, cprev, cnext, w2, 0, drow, tid);
                else fwd_step<K, true, 2>(L, cprev, cnext, w2, es_sh[F], drow, tid);
            } else {
                if (dec) fwd_step<K, true, 0>(L, cprev, cnext, w2, 0, drow, tid);
                else fwd_step<K, false, 0>(L, cprev, cnext, w2, 0, drow, tid);
            }
        }

        // Traceback: consume the loads.
        if (tbt) {
#pragma unroll
            for (int j = 0; j < kJobs; ++j) {
                if (phase[j] == PH_TP || phase[j] == PH_TF) {
                    int owner, bit;
                    M::locate(node[j], owner, bit);
                    const int d = (int)((tbw[j] >> bit) & (Word)(M::Q - 1));
                    if (phase[j] == PH_TF) enc[j * 256 + tbrow[j]] = (uint16_t)((d << (16 - K)) | node[j]);
                    node[j] = (d << M::DSHIFT) | (node[j] >> K);
                    if (phase[j] == PH_TP && step[j] == C - 1) es_sh[j] = node[j];
                }
            }
        }

        __syncthreads();

        // Uniform state update.
#pragma unroll
        for (int j = 0; j < kJobs; ++j) {
            switch (phase[j]) {
            case PH_FP:
            case PH_FF:
                if (j == F) {
                    ++step[j];
                    par[j] ^= 1;
                    if (phase[j] == PH_FP && step[j] == 2 * C) { phase[j] = PH_AM; step[j] = 0; }
                    else if (phase[j] == PH_FF && step[j] == 256) { phase[j] = PH_TF; step[j] = 0; }
                }
                break;
            case PH_AM: phase[j] = PH_TP; step[j] = 0; break;
            case PH_TP:
                if (++step[j] == C) { phase[j] = PH_FF; step[j] = 0; }
                break;
            case PH_TF:
                if (++step[j] == 256) { phase[j] = PH_OUT; step[j] = 0; }
                break;
            case PH_OUT: {
                if (tnext[j] < n_tiles) { tile[j] = tnext[j]; ++taken; phase[j] = PH_FP; }
                else phase[j] = PH_IDLE;
                step[j] = 0;
                par[j] = 0;
                break;
            }
            default: break;
            }
        }
    }
}

template <int K>
constexpr size_t smem_bytes() {
    return (size_t)kJobs * 2 * ThreadMap<K>::NODES * 2 + kJobs * 256 * 2 + kJobs * 256 * 2 +
           kJobs * 16 * 4 + kJobs * 4;
}

template <int K>
int launch(const float* tiles, int64_t n, const uint16_t* labels, int C, float* vals, uint16_t* states,
           uint8_t* ws, size_t ws_bytes, cudaStream_t stream) {
    int sms = 0;
    if (int rc = sm_count(&sms)) return rc;
    int grid, njobs;
    if (n <= sms) { grid = (int)n; njobs = 1; }
    else { grid = sms; njobs = kJobs; }
    const size_t need = (size_t)grid * kJobs * 256 * ThreadMap<K>::ROW_BYTES;
    if (ws_bytes < need) {
        set_error("viterbi workspace too small: %zu < %zu", ws_bytes, need);
        return KQ_ERR_WORKSPACE;
    }
    const size_t sm = smem_bytes<K>();
    cudaError_t e = cudaFuncSetAttribute(viterbi_kernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) { set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e)); return KQ_ERR_CUDA; }
    viterbi_kernel<K><<<grid, kThreads, sm, stream>>>(
        tiles, n, reinterpret_cast<const uint32_t*>(labels), reinterpret_cast<const __half*>(labels), C, njobs,
        vals, states, ws);
    return check_launch("viterbi_kernel");
}

}  // namespace

size_t pair_decision_bytes(int K, int64_t n, int sms);
template <int K>
int pair_launch(const float* tiles, int64_t n, const uint16_t* labels, int C, float* vals, uint16_t* states,
                uint8_t* ws, size_t ws_bytes, cudaStream_t stream);

size_t viterbi_decision_bytes(int K, int64_t n) {
    int sms = 0;
    if (sm_count(&sms)) return 0;
    if (K == 3 || K == 4) return pair_decision_bytes(K, n, sms);
    const int64_t grid = n <= sms ? n : sms;
    const size_t row = (K == 4) ? (size_t)kThreads * 4 : (size_t)kThreads * 8;
    return (size_t)grid * kJobs * 256 * row;
}

int viterbi_encode(const float* tiles, int64_t n, int K, const uint16_t* labels, int C, float* vals,
                   uint16_t* states, void* ws, size_t ws_bytes, cudaStream_t stream) {
    if (n < 0 || !labels || (n > 0 && (!tiles || !vals || !states))) {
        set_error("viterbi: null pointer or negative tile count");
        return KQ_ERR_ARG;
    }
    if (C < 1 || C > 128) { set_error("tailbite_context must be in 1..128 (got %d)", C); return KQ_ERR_ARG; }
    if (n == 0) return KQ_OK;
    if (((uintptr_t)labels & 3) || ((uintptr_t)ws & 15)) {
        set_error("viterbi: labels must be 4-byte and workspace 16-byte aligned");
        return KQ_ERR_ALIGN;
    }
    auto* w = static_cast<uint8_t*>(ws);
    switch (K) {
    case 2: return launch<2>(tiles, n, labels, C, vals, states, w, ws_bytes, stream);
    case 3: return pair_launch<3>(tiles, n, labels, C, vals, states, w, ws_bytes, stream);
    case 4: return pair_launch<4>(tiles, n, labels, C, vals, states, w, ws_bytes, stream);
    default: set_error("viterbi: K must be 2, 3 or 4 (got %d)", K); return KQ_ERR_ARG;
    }
}

}  // namespace kq
