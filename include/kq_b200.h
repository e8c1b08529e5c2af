/*
 * kq_b200.h -- C ABI of the kquant_b200 EXL3/QSRT trellis encoder for B200 (sm_100a).
 *
 * Every entry point takes plain device pointers, element counts and a
 * cudaStream_t (passed as void*).  It never allocates device memory, never
 * synchronizes the stream, and returns a KQ_* status code (0 on success).
 * kq_last_error() returns a readable message for the last failure of the
 * calling host thread.  Outputs and workspaces are caller-allocated, like the
 * reference extension's (kquant/csrc/sqg_quantize.cu:165-209).
 *
 * Layouts:
 *   tiles        float32 [n_tiles][256], 16x16 tiles already permuted to the
 *                tensor-core element order that the trellis runs along
 *                (kquant/exl3_encoder_backend.py:27-50)
 *   states       uint16  [n_tiles][256], 16-bit trellis state per element
 *   packed       uint16  [n_tiles][16*K], native EXL word order with SWAP16
 *   lut          uint8   [65536] E4M3 label bytes indexed by the 16-bit state
 *                (untransposed; kquant/sqg_e4m3.py:305-333)
 *   labels       uint16  [65536] binary16 labels indexed by state
 */
#ifndef KQ_B200_H
#define KQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KQ_OK 0
#define KQ_ERR_ARG (-1)        /* invalid argument (shape, K, context, pointer) */
#define KQ_ERR_WORKSPACE (-2)  /* workspace too small */
#define KQ_ERR_CUDA (-3)       /* CUDA runtime error (launch, attribute, device) */
#define KQ_ERR_ALIGN (-4)      /* pointer not aligned as the kernel requires */

/* Codebook kinds, numbered like the reference's `cb` template argument
 * (kquant/csrc/qsrt_quantize_tiles_kernel.cuh:21, exl3_compat/quant/codebook.cuh). */
#define KQ_CB_3INST 0
#define KQ_CB_MCG 1
#define KQ_CB_MUL1 2
#define KQ_CB_SQG 4

/* Message describing the last non-zero status returned on this host thread. */
const char* kq_last_error(void);

/* ABI version, bumped when a signature changes. */
int kq_abi_version(void);

/*
 * Decode a codebook into 65,536 binary16 labels (one per 16-bit state).
 * kind == KQ_CB_SQG reads `lut` (device, 65,536 E4M3 bytes); other kinds
 * ignore it.
 * Replaces the per-state label decoders inlined in the reference kernel:
 * kquant/csrc/sqg_quantize.cu:17-119 (SQG) and
 * kquant/csrc/exl3_compat/quant/codebook.cuh:28-124 (MCG, MUL1, 3INST).
 */
int kq_build_labels(int kind, const uint8_t* lut, uint16_t* labels, void* stream);

/*
 * Workspace bytes that kq_viterbi_encode / kq_quantize_tiles_* need for
 * n_tiles tiles at rate K on the current device.  The figure includes the
 * 128 KiB label table that kq_quantize_tiles_* build in the workspace.
 */
size_t kq_viterbi_workspace_bytes(int K, int64_t n_tiles);

/*
 * Tail-biting Viterbi encode of n_tiles tiles against prebuilt labels.
 * out_vals[i] = label(out_states[i]) as float32.  tailbite_ctx in 1..128.
 * K in {2, 3, 4}.  Bit-exact with the reference kernel
 * kquant/csrc/qsrt_quantize_tiles_kernel.cuh:21-471 (codes and values).
 */
int kq_viterbi_encode(const float* tiles, int64_t n_tiles, int K, const uint16_t* labels,
                      int tailbite_ctx, float* out_vals, uint16_t* out_states,
                      void* workspace, size_t workspace_bytes, void* stream);

/*
 * Drop-in counterpart of the reference binding quantize_tiles_sqg
 * (kquant/csrc/sqg_quantize.cpp:23-28, sqg_quantize.cu:165-259).  It differs
 * in two ways: the LUT is the untransposed state-indexed table, and a single
 * workspace replaces the temp_costs/temp_edges pair.
 */
int kq_quantize_tiles_sqg(const float* tiles, float* out_vals, uint16_t* out_states, int64_t n_tiles,
                          const uint8_t* lut, int K, int tailbite_ctx,
                          void* workspace, size_t workspace_bytes, void* stream);

/*
 * Drop-in counterpart of quantize_tiles_procedural
 * (kquant/csrc/sqg_quantize.cpp:29-32, sqg_quantize.cu:261-342).
 * codebook: KQ_CB_MCG or KQ_CB_MUL1 (KQ_CB_3INST is also accepted).
 */
int kq_quantize_tiles_procedural(const float* tiles, float* out_vals, uint16_t* out_states,
                                 int64_t n_tiles, int K, int codebook, int tailbite_ctx,
                                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * One 16-row step of the block-LDLQ traversal, fused around the Viterbi:
 * for a batch of row-major [size_k x size_n] fp32 matrices,
 *     tiles   = tensor-core-ordered 16x16 tiles of W[:, r0:r0+16] + comp
 *     What[:, r0:r0+16], enc[:, r0/16] = Viterbi(tiles)   (rows in W's layout)
 *     err[:, r0:r0+16] = W[:, r0:r0+16] - What[:, r0:r0+16]
 * comp [batch][16][size_n] is the LDLQ feedback of the step, enc
 * [batch][size_k/16][size_n/16][256] the 16-bit states.  Replaces the
 * tile gather / quantize_tiles / scatter sequence of one step of
 * kquant/exl3_encoder_backend.py:389-505 (ldlq); the arithmetic (one fp32
 * add, the Viterbi, one fp32 subtract) is the reference's.  Same labels,
 * K, context and workspace rules as kq_viterbi_encode with
 * n_tiles = batch * size_n / 16.  max_ctas > 0 caps the grid (each CTA
 * then loops over tile pairs), leaving the other SMs to concurrent work on
 * other streams; 0 uses every SM.
 */
int kq_ldlq_step_encode(const float* W, const float* comp, int64_t batch, int64_t size_k, int64_t size_n,
                        int64_t r0, int K, const uint16_t* labels, int tailbite_ctx, float* wq, float* err,
                        uint16_t* enc, int max_ctas, void* workspace, size_t workspace_bytes, void* stream);

/*
 * One LDLQ chain item: tiles [tile_col0, tile_col0 + n_tiles) of the 16-row
 * step r0 of one row-major [size_k x size_n] fp32 matrix W with its LDLQ
 * state (feedback P, error rows err, What, states enc [size_k/16][size_n/16]
 * [256]) and block-LDL factor L [size_k x size_k].  The step's feedback rows
 * are r0+16 .. end-1 (end = the end of the step's 128-row buffer).
 */
typedef struct {
    const float* W;
    const float* P;
    const float* L;
    float* err;
    float* wq;
    uint16_t* enc;
    int64_t size_k, size_n;
    int64_t r0, end;
    int64_t tile_col0, n_tiles;
    const uint16_t* labels;   /* binary16 label table of this item's codebook at rate K (kq_build_labels) */
    int32_t K;                /* 2, 3 or 4 */
    int32_t reserved;         /* 0 */
} kq_chain_item;

#define KQ_CHAIN_MAX_ITEMS 64

/*
 * One launch of LDLQ steps from up to KQ_CHAIN_MAX_ITEMS independent column
 * chains, each at its own row position:
 *     comp = P[r0:r0+16] + L[r0+16:end, r0:r0+16]^T err[r0+16:end]   (fp32)
 *     tiles = tensor-core-ordered 16x16 tiles of W[r0:r0+16] + comp
 *     What, enc = Viterbi(tiles);  err[r0:r0+16] = W - What
 * for the item's tile columns.  The feedback product is computed in the
 * kernel's tile load (one fp32 fma chain per element, in row order), so a
 * step is one launch and its result does not depend on which other items
 * share the launch.  Replaces the per-step feedback + quantize of
 * kquant/exl3_encoder_backend.py:389-505 (ldlq) / :1495-1583 (ldlq_batched);
 * the buffer-end update P[:begin] += L^T err stays with the caller.
 * Items carry their own K and label table.  When they all share both the
 * launch may hold any number of tiles.  Items of different K (or label
 * tables) share a launch when every item starts at an even tile (so each
 * tile pair has one K) and the pairs of each (K, labels) group, in runs of
 * m per CTA (m from ceil(pairs / SMs) up to 4), need at most one CTA per SM;
 * a CTA with two or more pairs hides each pair's tracebacks under another's
 * forward steps.  Workspace as
 * kq_viterbi_encode (K = 3) for the total tile count; max_ctas as
 * kq_ldlq_step_encode.
 */
int kq_ldlq_chain_step(const kq_chain_item* items, int n_items, int tailbite_ctx, int max_ctas, void* workspace,
                       size_t workspace_bytes, void* stream);

/*
 * Pack the low K bits of every state into 16*K uint16 words per tile in the
 * native EXL word order: MSB-first 16-symbol groups, then adjacent words
 * swapped (SWAP16).  Replaces ext.pack_trellis
 * (kquant/exl3_encoder_backend.py:1666-1677), whose word order
 * kquant/qsrt.py:811-833 restates.  K in 1..8.
 */
int kq_pack_trellis(const uint16_t* states, int64_t n_tiles, int K, uint16_t* packed, void* stream);

/*
 * Inverse of kq_pack_trellis, plus the cyclic state closure
 * state_i = ((state_{i-1} << K) | edge_i) & 0xFFFF.  Writes the 16-bit
 * states.  Replaces kquant/qsrt.py:836-863 (unpack_trellis_edges /
 * unpack_trellis_states) and kquant/exl3_reference.py:37-61
 * (reconstruct_trellis_states).  K in 1..8.
 */
int kq_unpack_trellis_states(const uint16_t* packed, int64_t n_tiles, int K, uint16_t* states,
                             void* stream);

/*
 * Allocation-free variant of kq_quantize_tiles_sqg for callers that cannot
 * allocate device memory themselves (a host whose allocator owns every byte
 * of the device, or code that must not trigger an allocation at an arbitrary
 * point).  No counterpart in the reference.  Same inputs, outputs and
 * results as kq_quantize_tiles_sqg, but no workspace argument: its scratch
 * (label table + decision rows, 32 MiB + 128 KiB) is a fixed __device__
 * array that every GPU loading this library holds until exit.  At most
 * KQ_NOALLOC_MAX_TILES tiles per call, a chosen bound on one call's latency
 * (not a limit of the scratch); larger counts return KQ_ERR_ARG.  The fixed
 * decision rows cap the grid at 8 CTAs (K2, K3) or 16 CTAs (K4), so a call
 * runs about 18x (K2, K3) or 9x (K4) slower than kq_quantize_tiles_sqg.
 * The first call on a device resolves the scratch address for that device
 * and caches it for the process: make that call before any stream capture,
 * and do not reset the device afterwards.  All calls share one scratch:
 * calls that overlap on the GPU (different streams, or different host
 * threads) race and corrupt each other's results; serialize them.
 */
#define KQ_NOALLOC_MAX_TILES 4096
int kq_quantize_tiles_sqg_noalloc(const float* tiles, float* out_vals, uint16_t* out_states, int64_t n_tiles,
                                  const uint8_t* lut, int K, int tailbite_ctx, void* stream);

/*
 * Fused tensor-core GEMM + trace (tcgen05 kind::tf32, TMA-fed):
 *     *out += sum_{i<M, j<N} (A B^T)[i][j] * D[i][j]
 * A [M x Kd], B [N x Kd] row-major fp32, D [M x N] with row stride ldd.
 * M % 128 == 0, N % 256 == 0, Kd % 32 == 0, 16-byte aligned rows.  Inputs
 * are rounded to TF32 by the tensor cores; accumulation is fp32, the final
 * reduction fp64.  With A = D = E^T and B = H (symmetric) this is the proxy
 * numerator tr(E^T H E) of kquant/exl3_encoder_backend.py:1466-1492
 * (block_trace).  *err is set to 1 if an internal wait timed out.
 */
int kq_trace_abt(const float* A, const float* B, const float* D, int64_t M, int64_t N, int64_t Kd, int64_t ldd,
                 double* out, int* err, void* stream);

/*
 * C = alpha * A B^T + beta * C on the tensor cores (tcgen05 kind::tf32, TMA
 * fed, TMEM accumulator).  Same shape rules as kq_trace_abt; C [M x N] with
 * row stride ldc.  The accumulator is drained into fp32 registers every
 * 128 K values, so with TF32-exact operands the result has fp32-GEMM
 * accuracy.  *err is set to 1 if an internal wait timed out.
 */
int kq_gemm_abt_tf32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t Kd, int64_t ldc,
                     float alpha, float beta, int* err, void* stream);

/*
 * Hessian accumulation, replacing the chunk body of
 * kquant/capture.py:713-730 (_accumulate_hessian, accumulator.addmm_(x.T,
 * x * w[:, None]) in FP32):
 *     H[d x d] (row stride ldh) += x^T diag(w) x
 * for samples x [tokens x d] (row stride ldx) and weights w [tokens] (NULL:
 * all ones).  One operand kernel (transpose, weighting, TF32 hi/lo split)
 * and one tcgen05 launch over the upper-triangle tiles, mirrored, so H
 * stays exactly symmetric.  split = 3: hi*hi + hi*lo + lo*hi (fp32-grade
 * accuracy, what the FP32 addmm of the reference gives); split = 1: TF32
 * operands.  Any tokens >= 0 and dim >= 1; the workspace holds the padded
 * operands, kq_hessian_workspace_bytes(tokens, dim, split) bytes, 16-byte
 * aligned (0 = invalid arguments).
 */
size_t kq_hessian_workspace_bytes(int64_t tokens, int64_t dim, int split);
int kq_accumulate_hessian(const float* x, const float* w, int64_t tokens, int64_t dim, int64_t ldx, float* H,
                          int64_t ldh, int split, void* workspace, size_t workspace_bytes, int* err, void* stream);

/*
 * Weight load: bf16 [rows x cols] (row stride ld_src elements; HF [out, in])
 * -> fp32 [cols x rows] (EXL [in, out]), dst[c][r] = src[row_perm[r]][c]
 * (row_perm may be NULL).  Replaces the caller-side
 * source.index_select(0, perm).T.contiguous() of
 * kquant/pack/qsrt_encoder.py:554-569 (_encoder_weight) for bf16 sources.
 */
int kq_bf16_to_f32_transposed(const uint16_t* src, int64_t rows, int64_t cols, int64_t ld_src,
                              const int64_t* row_perm, float* dst, void* stream);

/*
 * Reconstruction of encoded weights in the original basis:
 *     out = had_r(had_l(wq) * su[:, None]) * sv[None, :]
 * wq, out [k x n] fp32 row-major (k, n multiples of 128; 16-byte aligned),
 * su [k], sv [n] fp32; had_l / had_r are the 128-block Sylvester Hadamards
 * normalised 1/sqrt(128).  Replaces the matmul-based reconstruction of
 * kquant/exl3_encoder_backend.py:2211-2216 and :2492-2498 (fast
 * Walsh-Hadamard transforms; equal up to fp32 rounding).
 */
int kq_reconstruct_rotated(const float* wq, const float* su, const float* sv, int64_t k, int64_t n, float* out,
                           void* stream);

/*
 * Roofline probe (no reference counterpart): launches blocks x threads
 * threads that each issue iters*128 independent __hfma2 instructions.  Time
 * it with events on `stream`: HFMA2 rate = blocks*threads*iters*128 / time.
 * The Viterbi kernel's ALU roofline is derived from this measured rate.
 */
int kq_probe_hfma2(void* out, int iters, int blocks, int threads, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KQ_B200_H */
