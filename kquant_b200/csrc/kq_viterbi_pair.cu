// Tile-paired tail-biting Viterbi for K2 / K3 / K4, sm_100a.
//
// Same recursion and tie rules as kquant/csrc/qsrt_quantize_tiles_kernel.cuh:21-471
// (see kq_viterbi.cu for the statement).  The layout differs from the single-tile kernel:
//
//  * A job is a PAIR of tiles (A, B) run in lock-step.  Half2 lanes hold
//    node pairs (2p, 2p+1), so the register-resident labels (64 half2 per
//    thread) are used as they are.  The two tiles are two interleaved
//    instruction streams: each thread keeps 8 independent min chains per
//    butterfly block (4 node pairs x 2 tiles), which hides the half2
//    pipeline latency.  Costs live in shared memory as (A, B) half2 per
//    node: one 32-bit load per predecessor, broadcast once per tile.
//  * Two pair-jobs are staggered per CTA when the grid is full.  Forward
//    steps go shortest-remaining-phase first.  The four traceback chains
//    (2 jobs x 2 tiles) are walked by lanes 0..3 of warp 0, one step per
//    slot, with the load issued at slot start.  When no forward step is
//    pending, the chains run to the end of their phase without slot barriers.
//  * Decisions: 4 bits (K3, K4) or 2 bits (K2) per (node, tile), one 64-bit
//    (K4) or 128-bit (K2, K3) word per thread per step, tile A's bits first.
//  * One (A, B) cost double buffer per CTA: forward phases never preempt
//    one another, and a job's traceback phase (C or 256 steps) never
//    outlasts the other job's forward phase (2C or 256 steps), so the stagger
//    keeps the ALU busy without a second buffer.
//  * Tile I/O is a policy: FlatIO (tiles in trellis order), StepIO (one LDLQ
//    step: gather W + comp, scatter What / E / states) and ChainIO (LDLQ
//    chain items at their own rows, the feedback product computed in the
//    load).  pair_kernel_mk runs a single-wave chain launch whose items
//    differ in K, each CTA on its pair's K.
#include <algorithm>
#include "kq_viterbi_common.cuh"

namespace kq {
namespace {

constexpr int kThreads = 512;
constexpr int kJobs = 2;
constexpr int kStageBufs = 4;   // traceback row staging: buffers in the cp.async pipeline
constexpr int kMaxChainCtas = 160;   // CTAs of a mixed-K chain launch (one per SM)
constexpr int kMaxCtaPairs = 4;      // tile pairs per CTA of a mixed-K chain launch

template <int K>
struct PairMap {
    static_assert(K >= 2 && K <= 4, "pair kernel covers K2..K4");
    static constexpr int NODES = 1 << (16 - K);
    static constexpr int Q = 1 << K;
    static constexpr int DSHIFT = 16 - 2 * K;
    static constexpr int PB = (K == 2) ? 2 : 4;             // node pairs per block part
    static constexpr int G = (K == 4) ? 1 : (K == 3 ? 2 : 8);   // block parts per thread
    static constexpr int NPT = 2 * PB * G;                  // nodes per thread (8, 16, 32)
    static constexpr int DB = (K == 2) ? 2 : 4;             // decision bits per (node, tile)
    static constexpr int TILE_WORDS = NPT * DB / 32;        // 32-bit words per tile per thread
    static constexpr int GPW = 32 / (2 * PB * DB);          // block parts per decision word
    static constexpr int WORD_BYTES = 2 * TILE_WORDS * 4;   // both tiles
    static constexpr int ROW_BYTES = kThreads * WORD_BYTES;

    // First node of block part g of thread tid (even; 16-byte aligned as (A, B) half2).
    __device__ static __forceinline__ int base(int tid, int g) {
        if constexpr (K == 4) return ((tid >> 1) << 4) | ((tid & 1) << 3);
        else return (tid + kThreads * g) << K;
    }
    // Owner thread, 32-bit word and bit shift of node e's decision for tile t.
    __device__ static __forceinline__ void locate(int e, int t, int& tid, int& word, int& shift) {
        int g, j;
        if constexpr (K == 4) {
            tid = ((e >> 4) << 1) | ((e >> 3) & 1);
            g = 0;
            j = e & 7;
        } else {
            const int h = e >> K;
            tid = h & (kThreads - 1);
            g = h >> 9;
            j = e & (2 * PB - 1);
        }
        // Word layout: block parts g are packed GPW to a word; within a part,
        // even nodes (half2 lane 0) sit in the low 16 bits and odd nodes (lane 1)
        // in the high 16 bits, DB bits per node.
        word = t * TILE_WORDS + g / GPW;
        shift = (j & 1) * 16 + (g % GPW) * PB * DB + (j >> 1) * DB;
    }
    // Bit offset (within its 16-bit lane) of node pair p of block part g.
    __host__ __device__ static constexpr int field(int g, int p) { return (g % GPW) * PB * DB + p * DB; }
};

template <int K, bool DEC, int STEP0>
__device__ __forceinline__ void pair_step(
    const half2 (&L)[PairMap<K>::G][PairMap<K>::PB][PairMap<K>::Q],
    const half2* __restrict__ cprev, half2* __restrict__ cnext, half2 wA, half2 wB, int esA, int esB,
    uint8_t* __restrict__ decrow, int tid)
{
    // Lanes hold node pairs (2p, 2p+1); tiles A and B are two interleaved
    // instruction streams.  The shared (A, B) predecessor cost is loaded once
    // per k and broadcast per tile.
    using M = PairMap<K>;
    constexpr int PB = M::PB;
    const half2 zero2 = __float2half2_rn(0.f);
    const half2 inf2 = __halves2half2(__ushort_as_half(KQ_H_INF_BITS), __ushort_as_half(KQ_H_INF_BITS));
    uint32_t words[2 * M::TILE_WORDS];
#pragma unroll
    for (int w = 0; w < 2 * M::TILE_WORDS; ++w) words[w] = 0;
#pragma unroll
    for (int g = 0; g < M::G; ++g) {
        const int e0 = M::base(tid, g);
        const int h = e0 >> K;
        half2 mnA[PB], mnB[PB];
        uint32_t idA[PB], idB[PB];
#pragma unroll
        for (int k = 0; k < M::Q; ++k) {
            const int pk = (k << M::DSHIFT) | h;
            half2 cA, cB;
            if constexpr (STEP0 == 0) {
                const half2 c2 = cprev[pk];
                cA = __low2half2(c2);
                cB = __high2half2(c2);
            } else if constexpr (STEP0 == 1) {
                cA = zero2;
                cB = zero2;
            } else {
                cA = (pk == esA) ? zero2 : inf2;
                cB = (pk == esB) ? zero2 : inf2;
            }
#pragma unroll
            for (int p = 0; p < PB; ++p) {
                const half2 dA = __hsub2(L[g][p][k], wA);
                const half2 dB = __hsub2(L[g][p][k], wB);
                const half2 eA = __hfma2(dA, dA, cA);
                const half2 eB = __hfma2(dB, dB, cB);
                if (k == 0) {
                    mnA[p] = eA;
                    mnB[p] = eB;
                    if constexpr (DEC) { idA[p] = 0u; idB[p] = 0u; }
                } else {
                    if constexpr (DEC) {
                        // k placed at its node's final bit position in the decision word
                        const uint32_t kk = ((uint32_t)k << M::field(g, p)) * 0x10001u;
                        const uint32_t ltA = __hlt2_mask(eA, mnA[p]);
                        const uint32_t ltB = __hlt2_mask(eB, mnB[p]);
                        idA[p] = (ltA & kk) | (~ltA & idA[p]);
                        idB[p] = (ltB & kk) | (~ltB & idB[p]);
                    }
                    mnA[p] = __hmin2(eA, mnA[p]);
                    mnB[p] = __hmin2(eB, mnB[p]);
                }
            }
        }
        // Interleave to (A, B) per node and store 2*PB half2 (16 or 32 bytes).
        uint32_t v[2 * PB];
#pragma unroll
        for (int p = 0; p < PB; ++p) {
            const uint32_t a = *reinterpret_cast<uint32_t*>(&mnA[p]);
            const uint32_t b = *reinterpret_cast<uint32_t*>(&mnB[p]);
            v[2 * p] = __byte_perm(a, b, 0x5410);      // (A lo, B lo)
            v[2 * p + 1] = __byte_perm(a, b, 0x7632);  // (A hi, B hi)
        }
        uint4* dst = reinterpret_cast<uint4*>(cnext + e0);
        if constexpr (PB == 4) {
            // Lanes 4..7 of each 8-lane phase store their upper half first, so
            // a phase of 128-bit stores covers all 32 banks once.
            const int sw = (tid >> 2) & 1;
            const uint4 lo = make_uint4(v[0], v[1], v[2], v[3]);
            const uint4 hi = make_uint4(v[4], v[5], v[6], v[7]);
            dst[sw] = sw ? hi : lo;
            dst[sw ^ 1] = sw ? lo : hi;
        } else {
            dst[0] = make_uint4(v[0], v[1], v[2], v[3]);
        }
        if constexpr (DEC) {
            // decisions are already at their bit positions: OR the pairs in
#pragma unroll
            for (int p = 0; p < PB; ++p) {
                words[g / M::GPW] |= idA[p];
                words[M::TILE_WORDS + g / M::GPW] |= idB[p];
            }
        }
    }
    if constexpr (DEC) {
        if constexpr (M::TILE_WORDS == 1) {
            __stcs(reinterpret_cast<unsigned long long*>(decrow) + tid,
                   (unsigned long long)words[0] | ((unsigned long long)words[1] << 32));
        } else {
            __stcs(reinterpret_cast<uint4*>(decrow) + tid, make_uint4(words[0], words[1], words[2], words[3]));
        }
    }
}

// Traceback lane state: lanes 0..2*kJobs-1 of warp 0 walk chain (job, tile).
struct TbLane {
    int node;
    int row;
};

// S consecutive forward steps of job F (one template variant for the run),
// with one traceback step per forward step for every chain in a traceback
// phase.  Control decisions are made only between runs.
template <int K, bool DEC, int STEP0>
__device__ __forceinline__ void run_steps(
    const half2 (&L)[PairMap<K>::G][PairMap<K>::PB][PairMap<K>::Q], half2* cost_job, int& par, const half2* wsh_job,
    int ri, int S, int esA, int esB, uint8_t* dec_job, int tid,
    bool tb_on, bool tb_final, TbLane& tb, const uint8_t* tb_dec, int tb_tile, uint16_t* tb_enc)
{
    using M = PairMap<K>;
    for (int s = 0; s < S; ++s) {
        unsigned int tbw = 0;
        if (tb_on) {
            int owner, word, sh;
            M::locate(tb.node, tb_tile, owner, word, sh);
            tbw = __ldcg(reinterpret_cast<const unsigned int*>(tb_dec + (size_t)tb.row * M::ROW_BYTES +
                                                              (size_t)owner * M::WORD_BYTES) + word);
        }
        const half2 w2 = wsh_job[ri];
        pair_step<K, DEC, STEP0>(L, cost_job + par * M::NODES, cost_job + (par ^ 1) * M::NODES,
                                 __low2half2(w2), __high2half2(w2), esA, esB,
                                 dec_job + (size_t)ri * M::ROW_BYTES, tid);
        if (tb_on) {
            int owner, word, sh;
            M::locate(tb.node, tb_tile, owner, word, sh);
            const int d = (int)((tbw >> sh) & (M::Q - 1));
            if (tb_final) tb_enc[tb.row] = (uint16_t)((d << (16 - K)) | tb.node);
            tb.node = (d << M::DSHIFT) | (tb.node >> K);
            --tb.row;
        }
        par ^= 1;
        ri = (ri + 1) & 255;
        __syncthreads();
    }
}

// Tile I/O policies.  load(tile, j) returns element j (trellis order) of a
// tile; store(tile, j, state, value) receives its encoded state and value.
//
// FlatIO: tiles [n][256] already in trellis order, outputs alike.
struct FlatIO {
    static constexpr int kStageFloats = 0;
    const float* __restrict__ tiles;
    float* __restrict__ vals;
    uint16_t* __restrict__ states;
    __device__ __forceinline__ float load(int64_t tile, int j) const { return tiles[tile * 256 + j]; }
    __device__ __forceinline__ void store(int64_t tile, int j, uint16_t sv, float v) const {
        states[tile * 256 + j] = sv;
        vals[tile * 256 + j] = v;
    }
};

// StepIO: one 16-row LDLQ step of a batch of [k x n] matrices (row-major,
// contiguous): tile t is batch b = t / tiles_n, tile column c = t % tiles_n
// of rows r0..r0+15.  Trellis position j = 8 m + s of a tile holds row
// 2 (m % 4) + (s & 1) + 8 ((s >> 1) & 1), column m / 4 + 8 (s >> 2) (the
// tensor-core order of kquant/exl3_encoder_backend.py:27-50).  Loads
// W + comp, stores What = value, E = W - value and the state into
// enc [b][r0 / 16][c][j].
struct StepIO {
    static constexpr int kStageFloats = 0;
    const float* __restrict__ W;
    const float* __restrict__ comp;    // [batch][16][n]
    float* __restrict__ wq;
    float* __restrict__ err;
    uint16_t* __restrict__ enc;        // [batch][k / 16][n / 16][256]
    int64_t size_k, size_n, r0;
    int tiles_n;
    __device__ __forceinline__ void locate(int64_t tile, int j, int64_t& wi, int64_t& ci) const {
        const int m = j >> 3, s = j & 7;
        const int row = 2 * (m & 3) + (s & 1) + 8 * ((s >> 1) & 1);
        const int col = (m >> 2) + 8 * (s >> 2);
        const int64_t b = tile / tiles_n, c = tile - b * tiles_n;
        const int64_t x = c * 16 + col;
        wi = (b * size_k + r0 + row) * size_n + x;
        ci = (b * 16 + row) * size_n + x;
    }
    __device__ __forceinline__ float load(int64_t tile, int j) const {
        int64_t wi, ci;
        locate(tile, j, wi, ci);
        return W[wi] + comp[ci];
    }
    __device__ __forceinline__ void store(int64_t tile, int j, uint16_t sv, float v) const {
        int64_t wi, ci;
        locate(tile, j, wi, ci);
        wq[wi] = v;
        err[wi] = W[wi] - v;
        const int64_t b = tile / tiles_n, c = tile - b * tiles_n;
        enc[((b * (size_k >> 4) + (r0 >> 4)) * tiles_n + c) * 256 + j] = sv;
    }
};

// ChainIO: tiles of up to KQ_CHAIN_MAX_ITEMS LDLQ chain items (see
// kq_ldlq_chain_step); tile t belongs to the item whose [start, start + n)
// range holds it.  The load computes the item's feedback for the element.
struct ChainIO {
    // Feedback rows staged per chunk: [tile of the pair][L | err][row][16].
    static constexpr int kChunk = 112;
    static constexpr int kStageFloats = 2 * 2 * kChunk * 16;
    kq_chain_item it[KQ_CHAIN_MAX_ITEMS];
    int64_t start[KQ_CHAIN_MAX_ITEMS + 1];
    int n;
    // Mixed-K launches: the tile pairs of CTA b in order (-1: none), all of one K.
    int16_t cta_pair[kMaxChainCtas][kMaxCtaPairs];
    __device__ __forceinline__ int find(int64_t tile) const {
        int i = 0;
        while (i + 1 < n && tile >= start[i + 1]) ++i;
        return i;
    }
    __device__ __forceinline__ void locate(const kq_chain_item& c, int64_t lt, int j, int64_t& R, int64_t& x,
                                           int64_t& tc) const {
        const int m = j >> 3, s = j & 7;
        const int row = 2 * (m & 3) + (s & 1) + 8 * ((s >> 1) & 1);
        const int col = (m >> 2) + 8 * (s >> 2);
        tc = c.tile_col0 + lt;
        R = c.r0 + row;
        x = tc * 16 + col;
    }
    // Element j of tile (2q + t) for every thread of the CTA (t = tid / 256,
    // j = tid % 256), both tiles of the pair at once: the feedback rows of
    // each tile (L[r0+16+i][r0..r0+15], err[r0+16+i][16 tile columns]) go to
    // shared memory in chunks of kChunk rows with coalesced 16-byte loads,
    // then each thread sums its element's row in ascending order (the same
    // fp32 fma chain as load()).  Called by all threads; contains barriers.
    __device__ __forceinline__ float load_staged(int64_t tA, int64_t tB, int t, int j, float* stage,
                                                 int tid) const {
        const int iA = find(tA), iB = find(tB);
        const kq_chain_item& cA = it[iA];
        const kq_chain_item& cB = it[iB];
        const int64_t mA = cA.end - cA.r0 - 16, mB = cB.end - cB.r0 - 16;
        const int64_t tcA = cA.tile_col0 + (tA - start[iA]), tcB = cB.tile_col0 + (tB - start[iB]);
        const kq_chain_item& c = t ? cB : cA;
        int64_t R, x, tc;
        locate(c, (t ? tB : tA) - start[t ? iB : iA], j, R, x, tc);
        const int row = (int)(R - c.r0), col = (int)(x - tc * 16);
        const int64_t m = t ? mB : mA;
        const int64_t mmax = mA > mB ? mA : mB;
        float s = 0.f;
        for (int64_t c0 = 0; c0 < mmax; c0 += kChunk) {
            for (int idx = tid; idx < 2 * 2 * kChunk * 4; idx += kThreads) {
                const int tt = idx / (2 * kChunk * 4);
                const int rem = idx - tt * (2 * kChunk * 4);
                const int which = rem / (kChunk * 4);
                const int i = (rem >> 2) % kChunk, quad = rem & 3;
                const kq_chain_item& ci = tt ? cB : cA;
                const int64_t mi = tt ? mB : mA;
                if (c0 + i < mi) {
                    const int64_t q = ci.r0 + 16 + c0 + i;
                    const float4 v = which == 0
                        ? __ldg(reinterpret_cast<const float4*>(ci.L + q * ci.size_k + ci.r0) + quad)
                        : __ldcg(reinterpret_cast<const float4*>(ci.err + q * ci.size_n + (tt ? tcB : tcA) * 16) + quad);
                    reinterpret_cast<float4*>(stage + ((tt * 2 + which) * kChunk + i) * 16)[quad] = v;
                }
            }
            __syncthreads();
            const float* ls = stage + (t * 2 + 0) * kChunk * 16 + row;
            const float* es = stage + (t * 2 + 1) * kChunk * 16 + col;
            const int cnt = (int)((m - c0) < kChunk ? (m - c0) : kChunk);
            for (int i = 0; i < cnt; ++i) s = fmaf(ls[i * 16], es[i * 16], s);
            __syncthreads();
        }
        const int64_t n = c.size_n;
        const float comp = __ldcg(c.P + R * n + x) + s;
        return __ldg(c.W + R * n + x) + comp;
    }
    __device__ __forceinline__ void store(int64_t tile, int j, uint16_t sv, float v) const {
        const int i = find(tile);
        const kq_chain_item& c = it[i];
        int64_t R, x, tc;
        locate(c, tile - start[i], j, R, x, tc);
        const int64_t n = c.size_n;
        c.wq[R * n + x] = v;
        c.err[R * n + x] = c.W[R * n + x] - v;
        c.enc[(((c.r0 >> 4) * (n >> 4)) + tc) * 256 + j] = sv;
    }
};

template <int K>
__host__ __device__ constexpr size_t pair_smem_bytes() {
    return (size_t)2 * PairMap<K>::NODES * 4 + kJobs * 256 * 4 + kJobs * 2 * 256 * 2 + kJobs * 2 * 16 * 4 +
           kJobs * 2 * 4;
}

// The kernel body (kq_viterbi_pair_body.inc) is included inline in each
// kernel, with K, IO and the parameters in scope: the single-K kernels below
// and, once per K, the mixed-K chain kernel.  (A shared __device__ function
// taking the parameters by reference made every variant about 4% slower.)
template <int K, class IO>
__global__ void __launch_bounds__(kThreads, 1)
pair_kernel(const IO io, int64_t n_tiles, const uint32_t* __restrict__ labels32,
            const __half* __restrict__ labels16, int C, int njobs, uint8_t* __restrict__ decisions)
{
    uint8_t* dec_base = decisions + (size_t)blockIdx.x * kJobs * 256 * PairMap<K>::ROW_BYTES;
    auto pair_index = [&](int64_t t) { return (int64_t)blockIdx.x + (int64_t)gridDim.x * t; };
#include "kq_viterbi_pair_body.inc"
}

// Decision row bytes of the widest K (K2 and K3: 8 KiB).
constexpr size_t kMaxRowBytes =
    PairMap<2>::ROW_BYTES > PairMap<3>::ROW_BYTES
        ? (PairMap<2>::ROW_BYTES > PairMap<4>::ROW_BYTES ? PairMap<2>::ROW_BYTES : PairMap<4>::ROW_BYTES)
        : (PairMap<3>::ROW_BYTES > PairMap<4>::ROW_BYTES ? PairMap<3>::ROW_BYTES : PairMap<4>::ROW_BYTES);

// Chain launch whose items may differ in K: each CTA runs one to four tile
// pairs of one K (the host's per-CTA pair table, io.cta_pair), with the body
// for that K and that item's labels.  Two or more pairs per CTA stagger like
// the single-K kernel's jobs, hiding each pair's tracebacks under another's
// forward steps.  (A template on IO so that the body's `if constexpr`
// branches are discarded.)
template <class IO>
__global__ void __launch_bounds__(kThreads, 1)
pair_kernel_mk(const IO io, int64_t n_tiles, int C, uint8_t* __restrict__ decisions)
{
    const int64_t n_pairs_all = (n_tiles + 1) >> 1;
    auto pair_index = [&](int64_t t) -> int64_t {
        if (t >= kMaxCtaPairs) return n_pairs_all;
        const int q = io.cta_pair[blockIdx.x][t];
        return q < 0 ? n_pairs_all : (int64_t)q;
    };
    const kq_chain_item& item = io.it[io.find(2 * pair_index(0))];
    uint8_t* dec_base = decisions + (size_t)blockIdx.x * kJobs * 256 * kMaxRowBytes;
    const uint32_t* __restrict__ labels32 = reinterpret_cast<const uint32_t*>(item.labels);
    const __half* __restrict__ labels16 = reinterpret_cast<const __half*>(item.labels);
    const int njobs = io.cta_pair[blockIdx.x][1] >= 0 ? kJobs : 1;
    if (item.K == 2) {
        constexpr int K = 2;
#include "kq_viterbi_pair_body.inc"
    } else if (item.K == 3) {
        constexpr int K = 3;
#include "kq_viterbi_pair_body.inc"
    } else {
        constexpr int K = 4;
#include "kq_viterbi_pair_body.inc"
    }
}

template <int K>
void pair_grid(int64_t n, int sms, int& grid, int& njobs) {
    const int64_t pairs = (n + 1) / 2;
    if (pairs <= sms) { grid = (int)pairs; njobs = 1; }
    else { grid = sms; njobs = kJobs; }
}

template <int K, class IO>
int pair_run(const IO& io, int64_t n, const uint16_t* labels, int C, int grid, int njobs, uint8_t* dec,
             cudaStream_t stream) {
    const size_t sm = ((pair_smem_bytes<K>() + 15) & ~(size_t)15) + (size_t)IO::kStageFloats * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(pair_kernel<K, IO>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) { set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e)); return KQ_ERR_CUDA; }
    pair_kernel<K, IO><<<grid, kThreads, sm, stream>>>(io, n, reinterpret_cast<const uint32_t*>(labels),
                                                       reinterpret_cast<const __half*>(labels), C, njobs, dec);
    return check_launch("pair_kernel");
}

}  // namespace

size_t pair_decision_bytes(int K, int64_t n, int sms) {
    int grid, nj;
    pair_grid<3>(n, sms, grid, nj);
    const size_t row = (K == 4) ? PairMap<4>::ROW_BYTES : (K == 3 ? PairMap<3>::ROW_BYTES : PairMap<2>::ROW_BYTES);
    return (size_t)grid * kJobs * 256 * row;
}

template <int K>
int pair_launch(const float* tiles, int64_t n, const uint16_t* labels, int C, float* vals, uint16_t* states,
                uint8_t* ws, size_t ws_bytes, cudaStream_t stream) {
    int sms = 0;
    if (int rc = sm_count(&sms)) return rc;
    int grid, njobs;
    pair_grid<K>(n, sms, grid, njobs);
    const size_t need = (size_t)grid * kJobs * 256 * PairMap<K>::ROW_BYTES;
    if (ws_bytes < need) {
        set_error("viterbi workspace too small: %zu < %zu", ws_bytes, need);
        return KQ_ERR_WORKSPACE;
    }
    return pair_run<K>(FlatIO{tiles, vals, states}, n, labels, C, grid, njobs, ws, stream);
}

template int pair_launch<2>(const float*, int64_t, const uint16_t*, int, float*, uint16_t*, uint8_t*, size_t,
                            cudaStream_t);
template int pair_launch<3>(const float*, int64_t, const uint16_t*, int, float*, uint16_t*, uint8_t*, size_t,
                            cudaStream_t);
template int pair_launch<4>(const float*, int64_t, const uint16_t*, int, float*, uint16_t*, uint8_t*, size_t,
                            cudaStream_t);

// Launch with a grid bounded by a fixed decision buffer: at most
// dec_bytes / (2 jobs x 256 rows x row bytes) CTAs, each looping over pairs.
// Serves callers whose scratch is a fixed-size region (kq_noalloc.cu).
template <int K>
static int pair_launch_bounded(const float* tiles, int64_t n, const uint16_t* labels, int C, float* vals,
                               uint16_t* states, uint8_t* dec, size_t dec_bytes, cudaStream_t stream) {
    int sms = 0;
    if (int rc = sm_count(&sms)) return rc;
    const size_t per_cta = (size_t)kJobs * 256 * PairMap<K>::ROW_BYTES;
    const int64_t pairs = (n + 1) / 2;
    int64_t grid = (int64_t)(dec_bytes / per_cta);
    if (grid > sms) grid = sms;
    if (grid > pairs) grid = pairs;
    if (grid < 1) {
        set_error("bounded viterbi: decision buffer of %zu bytes holds no CTA (needs %zu)", dec_bytes, per_cta);
        return KQ_ERR_WORKSPACE;
    }
    const int njobs = pairs > grid ? kJobs : 1;
    return pair_run<K>(FlatIO{tiles, vals, states}, n, labels, C, (int)grid, njobs, dec, stream);
}

// One LDLQ step (StepIO) through the same kernel and grid policy as pair_launch.
template <int K, class IO>
int step_launch(const IO& io, int64_t n, const uint16_t* labels, int C, int max_ctas, uint8_t* ws,
                size_t ws_bytes, cudaStream_t stream) {
    int sms = 0;
    if (int rc = sm_count(&sms)) return rc;
    if (max_ctas > 0 && max_ctas < sms) sms = max_ctas;
    int grid, njobs;
    pair_grid<K>(n, sms, grid, njobs);
    const size_t need = (size_t)grid * kJobs * 256 * PairMap<K>::ROW_BYTES;
    if (ws_bytes < need) {
        set_error("viterbi workspace too small: %zu < %zu", ws_bytes, need);
        return KQ_ERR_WORKSPACE;
    }
    return pair_run<K>(io, n, labels, C, grid, njobs, ws, stream);
}

template <class IO>
int ldlq_step_encode(const IO& io, int64_t n, int K, const uint16_t* labels, int C, int max_ctas, uint8_t* ws,
                     size_t ws_bytes, cudaStream_t stream) {
    switch (K) {
    case 2: return step_launch<2, IO>(io, n, labels, C, max_ctas, ws, ws_bytes, stream);
    case 3: return step_launch<3, IO>(io, n, labels, C, max_ctas, ws, ws_bytes, stream);
    case 4: return step_launch<4, IO>(io, n, labels, C, max_ctas, ws, ws_bytes, stream);
    default: set_error("viterbi: K must be 2, 3 or 4 (got %d)", K); return KQ_ERR_ARG;
    }
}

int viterbi_encode_bounded(const float* tiles, int64_t n, int K, const uint16_t* labels, int C, float* vals,
                           uint16_t* states, uint8_t* dec, size_t dec_bytes, cudaStream_t stream) {
    switch (K) {
    case 2: return pair_launch_bounded<2>(tiles, n, labels, C, vals, states, dec, dec_bytes, stream);
    case 3: return pair_launch_bounded<3>(tiles, n, labels, C, vals, states, dec, dec_bytes, stream);
    case 4: return pair_launch_bounded<4>(tiles, n, labels, C, vals, states, dec, dec_bytes, stream);
    default: set_error("viterbi: K must be 2, 3 or 4 (got %d)", K); return KQ_ERR_ARG;
    }
}

}  // namespace kq

extern "C" int kq_ldlq_step_encode(const float* W, const float* comp, int64_t batch, int64_t size_k, int64_t size_n,
                                   int64_t r0, int K, const uint16_t* labels, int tailbite_ctx, float* wq,
                                   float* err, uint16_t* enc, int max_ctas, void* workspace,
                                   size_t workspace_bytes, void* stream) {
    using namespace kq;
    if (!W || !comp || !labels || !wq || !err || !enc) { set_error("kq_ldlq_step_encode: null pointer"); return KQ_ERR_ARG; }
    if (batch <= 0 || size_k <= 0 || size_n <= 0 || size_k % 16 || size_n % 16 || r0 < 0 || r0 % 16 ||
        r0 + 16 > size_k) {
        set_error("kq_ldlq_step_encode: bad shape (batch=%lld k=%lld n=%lld r0=%lld)", (long long)batch,
                  (long long)size_k, (long long)size_n, (long long)r0);
        return KQ_ERR_ARG;
    }
    if (tailbite_ctx < 1 || tailbite_ctx > 128) {
        set_error("tailbite_context must be in 1..128 (got %d)", tailbite_ctx);
        return KQ_ERR_ARG;
    }
    if (((uintptr_t)labels & 3) || ((uintptr_t)workspace & 15)) {
        set_error("kq_ldlq_step_encode: labels must be 4-byte and workspace 16-byte aligned");
        return KQ_ERR_ALIGN;
    }
    if (size_n / 16 > 0x7FFFFFFF) { set_error("kq_ldlq_step_encode: n too large"); return KQ_ERR_ARG; }
    StepIO io{W, comp, wq, err, enc, size_k, size_n, r0, (int)(size_n / 16)};
    return ldlq_step_encode(io, batch * (size_n / 16), K, labels, tailbite_ctx, max_ctas, static_cast<uint8_t*>(workspace),
                            workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int kq_ldlq_chain_step(const kq_chain_item* items, int n_items, int tailbite_ctx, int max_ctas,
                                  void* workspace, size_t workspace_bytes, void* stream) {
    using namespace kq;
    if (!items || n_items < 1 || n_items > KQ_CHAIN_MAX_ITEMS) {
        set_error("kq_ldlq_chain_step: need 1..%d items (got %d)", KQ_CHAIN_MAX_ITEMS, n_items);
        return KQ_ERR_ARG;
    }
    if (tailbite_ctx < 1 || tailbite_ctx > 128) {
        set_error("tailbite_context must be in 1..128 (got %d)", tailbite_ctx);
        return KQ_ERR_ARG;
    }
    if ((uintptr_t)workspace & 15) {
        set_error("kq_ldlq_chain_step: workspace must be 16-byte aligned");
        return KQ_ERR_ALIGN;
    }
    ChainIO io;
    io.n = n_items;
    int64_t total = 0;
    bool mixed = false, even = true;
    int kmask = 0;
    for (int i = 0; i < n_items; ++i) {
        const kq_chain_item& c = items[i];
        if (!c.W || !c.P || !c.L || !c.err || !c.wq || !c.enc || !c.labels) {
            set_error("kq_ldlq_chain_step: item %d has a null pointer", i);
            return KQ_ERR_ARG;
        }
        if (c.K < 2 || c.K > 4) { set_error("kq_ldlq_chain_step: item %d has K=%d", i, c.K); return KQ_ERR_ARG; }
        if ((uintptr_t)c.labels & 3) { set_error("kq_ldlq_chain_step: labels must be 4-byte aligned"); return KQ_ERR_ALIGN; }
        if (c.size_k <= 0 || c.size_n <= 0 || c.size_k % 16 || c.size_n % 16 || c.r0 < 0 || c.r0 % 16 ||
            c.end < c.r0 + 16 || c.end > c.size_k || c.n_tiles <= 0 || c.tile_col0 < 0 ||
            c.tile_col0 + c.n_tiles > c.size_n / 16) {
            set_error("kq_ldlq_chain_step: item %d has a bad shape (k=%lld n=%lld r0=%lld end=%lld tiles %lld+%lld)",
                      i, (long long)c.size_k, (long long)c.size_n, (long long)c.r0, (long long)c.end,
                      (long long)c.tile_col0, (long long)c.n_tiles);
            return KQ_ERR_ARG;
        }
        mixed |= c.K != items[0].K || c.labels != items[0].labels;
        even &= (total % 2) == 0;
        kmask |= 1 << c.K;
        io.it[i] = c;
        io.start[i] = total;
        total += c.n_tiles;
    }
    io.start[n_items] = total;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!mixed)
        return ldlq_step_encode(io, total, items[0].K, items[0].labels, tailbite_ctx, max_ctas,
                                static_cast<uint8_t*>(workspace), workspace_bytes, s);
    int sms = 0;
    if (int rc = sm_count(&sms)) return rc;
    if (sms > kMaxChainCtas) sms = kMaxChainCtas;
    if (!even) {
        set_error("kq_ldlq_chain_step: items of different K need even item starts");
        return KQ_ERR_ARG;
    }
    // Per-CTA pair table: the pairs of each (K, label table) group in runs of
    // m to a CTA, m the smallest count (from ceil(pairs / SMs) up to
    // kMaxCtaPairs) whose runs fit one CTA per SM, so every CTA runs one K and
    // one codebook.  At most one pair per SM gives one pair per CTA.
    const int64_t pairs = (total + 1) / 2;
    int64_t gp[KQ_CHAIN_MAX_ITEMS] = {};      // pairs of the group led by item g (0: not a leader)
    int leader[KQ_CHAIN_MAX_ITEMS];
    for (int i = 0; i < n_items; ++i) {
        leader[i] = i;
        for (int g = 0; g < i; ++g)
            if (leader[g] == g && items[g].K == items[i].K && items[g].labels == items[i].labels) { leader[i] = g; break; }
        gp[leader[i]] += (io.start[i + 1] + 1) / 2 - io.start[i] / 2;
    }
    int m = (int)std::max<int64_t>(1, (pairs + sms - 1) / sms), ctas = 0;
    for (; m <= kMaxCtaPairs; ++m) {
        int64_t c = 0;
        for (int g = 0; g < n_items; ++g) c += (gp[g] + m - 1) / m;
        if (c <= sms) { ctas = (int)c; break; }
    }
    if (m > kMaxCtaPairs || pairs > 0x7FFF) {
        set_error("kq_ldlq_chain_step: items of different K need at most %d same-K tile pairs per SM (%lld pairs)",
                  kMaxCtaPairs, (long long)pairs);
        return KQ_ERR_ARG;
    }
    {
        int cta = 0, fill = 0;
        for (int g = 0; g < n_items; ++g) {
            if (leader[g] != g) continue;
            for (int i = g; i < n_items; ++i) {
                if (leader[i] != g) continue;
                for (int64_t p = io.start[i] / 2; p < (io.start[i + 1] + 1) / 2; ++p) {
                    if (fill == 0) for (int t = 0; t < kMaxCtaPairs; ++t) io.cta_pair[cta][t] = -1;
                    io.cta_pair[cta][fill] = (int16_t)p;
                    if (++fill == m) { fill = 0; ++cta; }
                }
            }
            if (fill) { fill = 0; ++cta; }
        }
    }
    if (max_ctas > 0 && ctas > max_ctas) {
        set_error("kq_ldlq_chain_step: a mixed-K launch needs %d CTAs (max_ctas %d)", ctas, max_ctas);
        return KQ_ERR_ARG;
    }
    const size_t need = (size_t)ctas * kJobs * 256 * kMaxRowBytes;
    if (workspace_bytes < need) {
        set_error("viterbi workspace too small: %zu < %zu", workspace_bytes, need);
        return KQ_ERR_WORKSPACE;
    }
    size_t sm = 0;
    if (kmask & 4) sm = std::max(sm, pair_smem_bytes<2>());
    if (kmask & 8) sm = std::max(sm, pair_smem_bytes<3>());
    if (kmask & 16) sm = std::max(sm, pair_smem_bytes<4>());
    sm = ((sm + 15) & ~(size_t)15) + (size_t)ChainIO::kStageFloats * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute(pair_kernel_mk<ChainIO>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) { set_error("cudaFuncSetAttribute: %s", cudaGetErrorString(e)); return KQ_ERR_CUDA; }
    pair_kernel_mk<ChainIO><<<ctas, kThreads, sm, s>>>(io, total, tailbite_ctx, static_cast<uint8_t*>(workspace));
    return check_launch("pair_kernel_mk");
}
