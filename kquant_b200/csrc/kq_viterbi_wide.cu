// Tail-biting Viterbi for K = 1 and K = 5..8 (any K in 1..8 compiles), sm_100a.
//
// Same recursion, tie rules and primer quirk as the K2..K4 pair kernel and
// as kquant/csrc/qsrt_quantize_tiles_kernel.cuh:21-471, whose template is
// written for any K (the reference host accepts only K2..K4,
// kquant/csrc/sqg_quantize.cu:190,286):
//   cost_i[e] = min_k fma(L(t_k) - w_i, L(t_k) - w_i, cost_{i-1}[p_k]),
//   t_k = (k << (16-K)) | e,  p_k = (k << (16-2K)) | (e >> K),
// the lowest k winning a tie, a 2C-step primer whose argmin reads the
// second-to-last step's costs, and the final 256-step pass from the primer's
// end state.
//
// Layout, one tile per CTA job (512 threads, persistent grid):
//   * 65,536 relaxations per step, 128 per thread: each thread owns NP node
//     pairs (2p, 2p+1, one per half2 lane) x QT predecessors, with their
//     labels in 64 registers (half2).  Wide butterflies (K >= 7, 2^K
//     predecessors) split a pair's predecessors over SP = 2^K / 64
//     threads, merged with shuffles in k order.
//   * Predecessor ranges are cut into S contiguous sub-chains so that every
//     thread keeps >= 8 independent min chains; they merge in k order with a
//     strict less-than, so the lowest k still wins every tie.
//   * One binary16 cost per node in shared memory, double-buffered (128 KiB
//     at K=1, 8 KiB at K=5).
//   * Decisions: K bits per node, placed at their final bit position as they
//     are selected (lane 0 nodes in the low 16 bits of a word, lane 1 nodes
//     in the high 16 bits); NW words per thread per step, written coalesced.
//   * Tracebacks stream the decision rows through shared memory with a
//     double-buffered cp.async pipeline; one lane walks them.  A tile's final
//     traceback is instead walked one row per primer step of the CTA's next
//     tile (decision rows in two areas, alternating by tile), so it hides
//     under that primer's forward steps; only the CTA's last tile and the
//     primer tracebacks stay exposed.
#include "kq_viterbi_common.cuh"

namespace kq {
namespace {

constexpr int kWThreads = 512;

template <int K>
struct WideMap {
    static_assert(K >= 1 && K <= 8, "wide kernel covers K1..K8");
    static constexpr int NODES = 1 << (16 - K);
    static constexpr int Q = 1 << K;                         // predecessors per node
    static constexpr int DSHIFT = 16 - 2 * K;
    static constexpr int QT = Q < 64 ? Q : 64;               // predecessors per thread
    static constexpr int SP = Q / QT;                        // threads per node pair
    static constexpr int NP = 64 / QT;                       // node pairs per thread
    static constexpr int PBW = NP < Q / 2 ? NP : (Q / 2 > 0 ? Q / 2 : 1);   // pairs sharing a block, per thread
    static constexpr int G = NP / PBW;                       // blocks per thread
    static constexpr int TPB = (Q / 2) / PBW > 0 ? (Q / 2) / PBW : 1;       // threads sharing a block (SP == 1)
    static constexpr int S = (8 / NP) > 1 ? (8 / NP) : 1;    // sub-chains per pair
    static constexpr int CH = QT / S;                        // predecessors per sub-chain
    static constexpr int SLOTS = 16 / K;                     // nodes per 16-bit half of a decision word
    static constexpr int NW = (NP + SLOTS - 1) / SLOTS;      // decision words per thread per step
    static constexpr int ROW_WORDS = NW * kWThreads;
    static constexpr int ROW_BYTES = ROW_WORDS * 4;
    static constexpr bool PAD = SP > 1;                      // padded cost layout (split predecessors)
    static constexpr int PADDED = PAD ? NODES + 2 * (NODES >> 6) : NODES;
    static_assert(NP * QT == 64 && G * PBW == NP && CH * S == QT, "ownership");

    // Shared-memory index of node e's cost.  With split predecessors (K7, K8)
    // 2 pad halves every 64 nodes keep the SP threads' loads on distinct banks;
    // otherwise the layout is plain, so every load and store of a step is a
    // per-thread base plus a compile-time offset.
    __host__ __device__ static constexpr int pad(int e) { return PAD ? e + ((e >> 6) << 1) : e; }

    // Block index h (= e >> K) of group g of thread tid and its first pair.
    __device__ static __forceinline__ void block_of(int tid, int g, int& h, int& pair0) {
        if constexpr (SP > 1) {
            const int pr = tid / SP;
            h = (2 * pr) >> K;
            pair0 = pr;
        } else if constexpr (G > 1) {
            h = tid + kWThreads * g;
            pair0 = h * (Q / 2);
        } else {
            h = tid / TPB;
            pair0 = h * (Q / 2) + (tid % TPB) * PBW;
        }
    }

    // Row word and bit shift of node e's decision.
    __device__ static __forceinline__ void locate(int e, int& word, int& shift) {
        const int p = e >> 1, lane = e & 1;
        int t, i;
        if constexpr (SP > 1) {
            t = p * SP;
            i = 0;
        } else if constexpr (G > 1) {
            const int h = e >> K, pb = p % (Q / 2 > 0 ? Q / 2 : 1);
            t = h % kWThreads;
            i = (h / kWThreads) * PBW + pb;
        } else {
            const int h = e >> K, q = p % (Q / 2);
            t = h * TPB + q / PBW;
            i = q % PBW;
        }
        word = (i / SLOTS) * kWThreads + t;
        shift = lane * 16 + (i % SLOTS) * K;
    }
};

template <int K>
__host__ __device__ constexpr size_t wide_smem_bytes() {
    // costs [2][PADDED] half, tile [256] half, reduction [16] u32, end state and
    // traceback hand-over [4] int, states of the previous tile [256] u16
    return (size_t)2 * WideMap<K>::PADDED * 2 + 256 * 2 + 16 * 4 + 16 + 256 * 2;
}

// One forward step.  STEP0: 0 = costs from cprev, 1 = zero prior cost (the
// primer's first step), 2 = prior cost 0 at the end state es, +inf elsewhere.
template <int K, bool DEC, int STEP0>
__device__ __forceinline__ void wide_step(const half2 (&L)[WideMap<K>::NP][WideMap<K>::QT],
                                          const __half* __restrict__ cprev, __half* __restrict__ cnext, half2 w2,
                                          int es, uint32_t* __restrict__ decrow, int tid) {
    using M = WideMap<K>;
    const half2 zero2 = __float2half2_rn(0.f);
    const half2 inf2 = __halves2half2(__ushort_as_half(KQ_H_INF_BITS), __ushort_as_half(KQ_H_INF_BITS));
    uint32_t words[M::NW];
#pragma unroll
    for (int w = 0; w < M::NW; ++w) words[w] = 0;
    const int kbase = (M::SP > 1) ? (tid % M::SP) * M::QT : 0;
#pragma unroll
    for (int g = 0; g < M::G; ++g) {
        int h, pair0;
        M::block_of(tid, g, h, pair0);
        half2 mn[M::PBW][M::S];
        uint32_t id[M::PBW][M::S];
        // Predecessor (kbase + kk) << DSHIFT | h sits at cbase + pad(kk << DSHIFT):
        // kbase << DSHIFT is a multiple of 64 and h < 2^DSHIFT, so the padding
        // splits into a per-thread part and a compile-time part.
        const __half* cbase = cprev + M::pad(kbase << M::DSHIFT) + h;
#pragma unroll
        for (int j = 0; j < M::CH; ++j) {
#pragma unroll
            for (int s = 0; s < M::S; ++s) {
                const int kk = s * M::CH + j;
                const int pk = ((kbase + kk) << M::DSHIFT) | h;
                half2 c2;
                if constexpr (STEP0 == 0) c2 = __half2half2(cbase[M::pad(kk << M::DSHIFT)]);
                else if constexpr (STEP0 == 1) c2 = zero2;
                else c2 = (pk == es) ? zero2 : inf2;
#pragma unroll
                for (int pb = 0; pb < M::PBW; ++pb) {
                    const int i = g * M::PBW + pb;
                    const half2 d = __hsub2(L[i][kk], w2);
                    const half2 e = __hfma2(d, d, c2);
                    if (j == 0) {
                        mn[pb][s] = e;
                        if constexpr (DEC) id[pb][s] = ((uint32_t)kk << ((i % M::SLOTS) * K)) * 0x10001u;
                    } else {
                        if constexpr (DEC) {
                            const uint32_t kv = ((uint32_t)kk << ((i % M::SLOTS) * K)) * 0x10001u;
                            const uint32_t lt = __hlt2_mask(e, mn[pb][s]);
                            id[pb][s] = (lt & kv) | (~lt & id[pb][s]);
                        }
                        mn[pb][s] = __hmin2(e, mn[pb][s]);
                    }
                }
            }
        }
#pragma unroll
        for (int pb = 0; pb < M::PBW; ++pb) {
            const int i = g * M::PBW + pb;
            half2 best = mn[pb][0];
            uint32_t bid = DEC ? id[pb][0] : 0u;
#pragma unroll
            for (int s = 1; s < M::S; ++s) {
                // chains cover ascending k ranges: a later chain wins only when strictly lower
                if constexpr (DEC) {
                    const uint32_t lt = __hlt2_mask(mn[pb][s], best);
                    bid = (lt & id[pb][s]) | (~lt & bid);
                }
                best = __hmin2(mn[pb][s], best);
            }
            if constexpr (M::SP > 1) {
                if constexpr (DEC) bid |= ((uint32_t)kbase << ((i % M::SLOTS) * K)) * 0x10001u;
                const int kp = tid % M::SP;
#pragma unroll
                for (int off = 1; off < M::SP; off <<= 1) {
                    const uint32_t ob = __shfl_xor_sync(0xFFFFFFFFu, *reinterpret_cast<uint32_t*>(&best), off);
                    const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bid, off);
                    const half2 other = *reinterpret_cast<const half2*>(&ob);
                    const bool mine_low = (kp & off) == 0;
                    const half2 lo = mine_low ? best : other, hi = mine_low ? other : best;
                    if constexpr (DEC) {
                        const uint32_t lo_i = mine_low ? bid : oi, hi_i = mine_low ? oi : bid;
                        const uint32_t lt = __hlt2_mask(hi, lo);
                        bid = (lt & hi_i) | (~lt & lo_i);
                    }
                    best = __hmin2(hi, lo);
                }
                if (kp == 0) *reinterpret_cast<half2*>(cnext + M::pad(2 * (pair0 + pb))) = best;
            } else {
                *reinterpret_cast<half2*>(cnext + M::pad(2 * (pair0 + pb))) = best;
            }
            if constexpr (DEC) words[i / M::SLOTS] |= bid;
        }
    }
    if constexpr (DEC) {
#pragma unroll
        for (int w = 0; w < M::NW; ++w) __stcs(decrow + w * kWThreads + tid, words[w]);
    }
}

// Walk `rows` decision rows backwards from `top` (row indices top, top-1, ...
// taken mod 256), starting at node `node`.  All threads stage the rows into
// `stage` (double-buffered cp.async); thread 0 walks.  Writes the states
// into enc[] when enc != nullptr.  Returns (in thread 0) the node reached.
template <int K>
__device__ int wide_traceback(const uint32_t* __restrict__ dec, int top, int rows, int node, uint8_t* stage,
                              int stage_bytes, uint16_t* enc, int tid) {
    using M = WideMap<K>;
    const int cap = stage_bytes / (2 * M::ROW_BYTES);         // rows per buffer
    const int nchunks = (rows + cap - 1) / cap;
    auto issue = [&](int c) {
        if (c < nchunks) {
            uint8_t* buf = stage + (size_t)(c & 1) * cap * M::ROW_BYTES;
            const int lo = c * cap, R = min(cap, rows - lo);
            for (int r = 0; r < R; ++r) {
                const int row = (top - lo - r) & 255;
                const uint8_t* src = reinterpret_cast<const uint8_t*>(dec) + (size_t)row * M::ROW_BYTES;
                uint8_t* dst = buf + (size_t)r * M::ROW_BYTES;
                for (int u = tid; u < M::ROW_BYTES / 16; u += kWThreads)
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                                 ::"r"((uint32_t)__cvta_generic_to_shared(dst + 16 * u)), "l"(src + 16 * u)
                                 : "memory");
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    issue(0);
    for (int c = 0; c < nchunks; ++c) {
        issue(c + 1);
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            const uint8_t* buf = stage + (size_t)(c & 1) * cap * M::ROW_BYTES;
            const int lo = c * cap, R = min(cap, rows - lo);
            for (int r = 0; r < R; ++r) {
                int word, shift;
                M::locate(node, word, shift);
                const uint32_t w = reinterpret_cast<const uint32_t*>(buf + (size_t)r * M::ROW_BYTES)[word];
                const int d = (int)((w >> shift) & (M::Q - 1));
                if (enc) enc[(top - lo - r) & 255] = (uint16_t)((d << (16 - K)) | node);
                node = (d << M::DSHIFT) | (node >> K);
            }
        }
        __syncthreads();
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    return node;
}

template <int K>
__global__ void __launch_bounds__(kWThreads, 1)
wide_kernel(const float* __restrict__ tiles, int64_t n_tiles, const uint32_t* __restrict__ labels32,
            const __half* __restrict__ labels16, int C, float* __restrict__ vals, uint16_t* __restrict__ states,
            uint8_t* __restrict__ decisions, int stage_bytes) {
    using M = WideMap<K>;
    extern __shared__ __align__(16) uint8_t smem[];
    __half* cost = reinterpret_cast<__half*>(smem);                           // [2][PADDED]
    __half* wsh = cost + 2 * M::PADDED;                                        // [256]
    uint32_t* red = reinterpret_cast<uint32_t*>(wsh + 256);                    // [16]
    int* es_sh = reinterpret_cast<int*>(red + 16);                             // [4]
    uint16_t* enc = reinterpret_cast<uint16_t*>(es_sh + 4);                    // [256] states of the tile in output
    uint8_t* stage = smem + ((wide_smem_bytes<K>() + 127) & ~(size_t)127);
    const int tid = threadIdx.x;
    // Two decision areas of 256 rows, alternating by tile: the final traceback
    // of a tile walks its rows while the next tile's primer writes the other area.
    uint32_t* dec_base = reinterpret_cast<uint32_t*>(decisions + (size_t)blockIdx.x * 2 * 256 * M::ROW_BYTES);

    half2 L[M::NP][M::QT];
    {
        const int kbase = (M::SP > 1) ? (tid % M::SP) * M::QT : 0;
#pragma unroll
        for (int g = 0; g < M::G; ++g) {
            int h, pair0;
            M::block_of(tid, g, h, pair0);
#pragma unroll
            for (int pb = 0; pb < M::PBW; ++pb)
#pragma unroll
                for (int kk = 0; kk < M::QT; ++kk) {
                    const uint32_t t = ((uint32_t)(kbase + kk) << (16 - K)) | (uint32_t)(2 * (pair0 + pb));
                    const uint32_t v = __ldg(labels32 + (t >> 1));
                    L[g * M::PBW + pb][kk] = *reinterpret_cast<const half2*>(&v);
                }
        }
    }

    // Pending final traceback of the previous tile (walked by thread 0, one row
    // per primer step of the current tile): its tile, node, row and decisions.
    bool pend = false;
    int64_t ptile = 0;
    int pnode = 0, prow = -1;
    const uint32_t* pdec = dec_base;
    auto output = [&](int64_t t) {
        if (tid < 256) {
            const uint16_t sv = enc[tid];
            states[t * 256 + tid] = sv;
            vals[t * 256 + tid] = __half2float(labels16[sv]);
        }
    };
    int parity = 0;
    for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, parity ^= 1) {
        uint32_t* dec = dec_base + (size_t)parity * 256 * M::ROW_WORDS;
        if (tid < 256) wsh[tid] = __float2half_rn(tiles[tile * 256 + tid]);
        __syncthreads();
        int par = 0;
        // primer: 2C steps from position 256 - C; decisions from step C on
        for (int i = 0; i < 2 * C; ++i) {
            const int ri = (i + 256 - C) & 255;
            const bool walk = pend && tid == 0 && prow >= 0;
            uint32_t tbw = 0;
            int tsh = 0;
            if (walk) {
                int word;
                M::locate(pnode, word, tsh);
                tbw = __ldcg(pdec + (size_t)prow * M::ROW_WORDS + word);
            }
            const half2 w2 = __half2half2(wsh[ri]);
            __half* cp = cost + par * M::PADDED;
            __half* cn = cost + (par ^ 1) * M::PADDED;
            uint32_t* row = dec + (size_t)ri * M::ROW_WORDS;
            if (i == 0) wide_step<K, false, 1>(L, cp, cn, w2, 0, row, tid);
            else if (i < C) wide_step<K, false, 0>(L, cp, cn, w2, 0, row, tid);
            else wide_step<K, true, 0>(L, cp, cn, w2, 0, row, tid);
            if (walk) {
                const int d = (int)((tbw >> tsh) & (M::Q - 1));
                enc[prow] = (uint16_t)((d << (16 - K)) | pnode);
                pnode = (d << M::DSHIFT) | (pnode >> K);
                --prow;
            }
            par ^= 1;
            __syncthreads();
        }
        if (pend) {
            // rows the primer did not cover (2C < 256), then the previous tile's output
            if (tid == 0) { es_sh[1] = pnode; es_sh[2] = prow; }
            __syncthreads();
            const int left = es_sh[2] + 1;
            if (left > 0) wide_traceback<K>(pdec, left - 1, left, es_sh[1], stage, stage_bytes, enc, tid);
            __syncthreads();
            output(ptile);
            __syncthreads();
            pend = false;
        }
        // argmin over the second-to-last primer step's costs, reference tie order
        {
            const __half* c = cost + (par ^ 1) * M::PADDED;
            uint32_t best = 0xFFFFFFFFu;
            for (int e = tid; e < M::NODES; e += kWThreads) {
                const uint32_t bits = __half_as_ushort(c[M::pad(e)]);
                best = min(best, (bits << 16) | wide_tie_key<K>(e));
            }
            best = __reduce_min_sync(0xFFFFFFFFu, best);
            if ((tid & 31) == 0) red[tid >> 5] = best;
            __syncthreads();
            if (tid == 0) {
                uint32_t b = red[0];
                for (int w = 1; w < kWThreads / 32; ++w) b = min(b, red[w]);
                es_sh[0] = wide_key_node<K>(b & 0xFFFFu);
            }
            __syncthreads();
        }
        // primer traceback: C rows (positions C-1 .. 0) to the end state
        {
            const int node = wide_traceback<K>(dec, C - 1, C, es_sh[0], stage, stage_bytes, nullptr, tid);
            if (tid == 0) es_sh[0] = node;
            __syncthreads();
        }
        const int es = es_sh[0];
        // final pass: 256 steps from position 0, step 0 constrained to the end state
        for (int i = 0; i < 256; ++i) {
            const half2 w2 = __half2half2(wsh[i]);
            __half* cp = cost + par * M::PADDED;
            __half* cn = cost + (par ^ 1) * M::PADDED;
            uint32_t* row = dec + (size_t)i * M::ROW_WORDS;
            if (i == 0) wide_step<K, true, 2>(L, cp, cn, w2, es, row, tid);
            else wide_step<K, true, 0>(L, cp, cn, w2, 0, row, tid);
            par ^= 1;
            __syncthreads();
        }
        if (tile + gridDim.x < n_tiles) {
            // hand the final traceback to the next tile's primer steps
            pend = true;
            ptile = tile;
            pnode = es;
            prow = 255;
            pdec = dec;
        } else {
            wide_traceback<K>(dec, 255, 256, es, stage, stage_bytes, enc, tid);
            __syncthreads();
            output(tile);
            __syncthreads();
        }
    }
}

template <int K>
size_t wide_stage_bytes() {
    // leave the rest of the 227 KiB opt-in shared memory to the traceback stage,
    // at most 64 rows per buffer
    const size_t base = (wide_smem_bytes<K>() + 127) & ~(size_t)127;
    size_t avail = 227 * 1024 - base;
    const size_t cap = 2 * (size_t)64 * WideMap<K>::ROW_BYTES;
    return (avail < cap ? avail : cap) / (2 * WideMap<K>::ROW_BYTES) * (2 * WideMap<K>::ROW_BYTES);
}

template <int K>
int wide_launch(const float* tiles, int64_t n, const uint16_t* labels, int C, float* vals, uint16_t* states,
                uint8_t* ws, size_t ws_bytes, int max_ctas, cudaStream_t stream) {
    int sms = 0;
    if (int rc = sm_count(&sms)) return rc;
    int64_t grid = n < sms ? n : sms;
    if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
    const size_t per_cta = (size_t)2 * 256 * WideMap<K>::ROW_BYTES;
    if (ws_bytes < (size_t)grid * per_cta) {
        const int64_t fit = (int64_t)(ws_bytes / per_cta);
        if (fit < 1) {
            set_error("viterbi workspace too small: %zu < %zu", ws_bytes, (size_t)grid * per_cta);
            return KQ_ERR_WORKSPACE;
        }
        grid = fit;
    }
    const size_t stage = wide_stage_bytes<K>();
    const size_t sm = ((wide_smem_bytes<K>() + 127) & ~(size_t)127) + stage;
    cudaError_t e = cudaFuncSetAttribute(wide_kernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) { set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e)); return KQ_ERR_CUDA; }
    wide_kernel<K><<<(int)grid, kWThreads, sm, stream>>>(tiles, n, reinterpret_cast<const uint32_t*>(labels),
                                                         reinterpret_cast<const __half*>(labels), C, vals, states,
                                                         ws, (int)stage);
    return check_launch("wide_kernel");
}

}  // namespace

bool wide_supported(int K) { return K == 1 || (K >= 5 && K <= 8); }

size_t wide_decision_bytes(int K, int64_t n, int sms) {
    const int64_t grid = n < sms ? n : sms;
    size_t row = 0;
    switch (K) {
    case 1: row = WideMap<1>::ROW_BYTES; break;
    case 5: row = WideMap<5>::ROW_BYTES; break;
    case 6: row = WideMap<6>::ROW_BYTES; break;
    case 7: row = WideMap<7>::ROW_BYTES; break;
    case 8: row = WideMap<8>::ROW_BYTES; break;
    case 2: row = WideMap<2>::ROW_BYTES; break;
    case 3: row = WideMap<3>::ROW_BYTES; break;
    case 4: row = WideMap<4>::ROW_BYTES; break;
    default: return 0;
    }
    return (size_t)(grid > 0 ? grid : 1) * 2 * 256 * row;
}

// K1 and K5..K8 in production; K2..K4 reachable here for cross-checks of this
// kernel against the pair kernel.
int wide_encode(const float* tiles, int64_t n, int K, const uint16_t* labels, int C, float* vals, uint16_t* states,
                uint8_t* ws, size_t ws_bytes, int max_ctas, cudaStream_t stream) {
    switch (K) {
    case 1: return wide_launch<1>(tiles, n, labels, C, vals, states, ws, ws_bytes, max_ctas, stream);
    case 2: return wide_launch<2>(tiles, n, labels, C, vals, states, ws, ws_bytes, max_ctas, stream);
    case 3: return wide_launch<3>(tiles, n, labels, C, vals, states, ws, ws_bytes, max_ctas, stream);
    case 4: return wide_launch<4>(tiles, n, labels, C, vals, states, ws, ws_bytes, max_ctas, stream);
    case 5: return wide_launch<5>(tiles, n, labels, C, vals, states, ws, ws_bytes, max_ctas, stream);
    case 6: return wide_launch<6>(tiles, n, labels, C, vals, states, ws, ws_bytes, max_ctas, stream);
    case 7: return wide_launch<7>(tiles, n, labels, C, vals, states, ws, ws_bytes, max_ctas, stream);
    case 8: return wide_launch<8>(tiles, n, labels, C, vals, states, ws, ws_bytes, max_ctas, stream);
    default: set_error("viterbi: K must be in 1..8 (got %d)", K); return KQ_ERR_ARG;
    }
}

}  // namespace kq
