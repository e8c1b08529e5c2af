// extern "C" entry points declared in include/kq_b200.h.
#include "kq_common.cuh"

namespace kq {
const char* last_error();
int build_labels(int kind, const uint8_t* lut, uint16_t* labels, cudaStream_t stream);
size_t viterbi_decision_bytes(int K, int64_t n);
int viterbi_encode(const float* tiles, int64_t n, int K, const uint16_t* labels, int C, float* vals,
                   uint16_t* states, void* ws, size_t ws_bytes, cudaStream_t stream);
int pack_trellis(const uint16_t* states, int64_t n, int K, uint16_t* packed, cudaStream_t stream);
int unpack_trellis_states(const uint16_t* packed, int64_t n, int K, uint16_t* states, cudaStream_t stream);
}  // namespace kq

namespace {
constexpr size_t kLabelBytes = 65536 * 2;

int quantize_with_kind(const float* tiles, float* vals, uint16_t* states, int64_t n, int kind, const uint8_t* lut,
                       int K, int C, void* ws, size_t ws_bytes, void* stream) {
    if (K < 1 || K > 8) { kq::set_error("quantize_tiles: K must be in 1..8 (got %d)", K); return KQ_ERR_ARG; }
    if (C < 1 || C > 128) { kq::set_error("tailbite_context must be in 1..128 (got %d)", C); return KQ_ERR_ARG; }
    if (n < 0) { kq::set_error("quantize_tiles: negative tile count"); return KQ_ERR_ARG; }
    if (n == 0) return KQ_OK;
    if (!ws || ws_bytes < kLabelBytes) { kq::set_error("quantize_tiles: workspace too small"); return KQ_ERR_WORKSPACE; }
    auto s = static_cast<cudaStream_t>(stream);
    auto* labels = static_cast<uint16_t*>(ws);
    if (int rc = kq::build_labels(kind, lut, labels, s)) return rc;
    return kq::viterbi_encode(tiles, n, K, labels, C, vals, states, static_cast<uint8_t*>(ws) + kLabelBytes,
                              ws_bytes - kLabelBytes, s);
}
}  // namespace

extern "C" {

const char* kq_last_error(void) { return kq::last_error(); }

int kq_abi_version(void) { return 1; }

int kq_build_labels(int kind, const uint8_t* lut, uint16_t* labels, void* stream) {
    return kq::build_labels(kind, lut, labels, static_cast<cudaStream_t>(stream));
}

size_t kq_viterbi_workspace_bytes(int K, int64_t n_tiles) {
    if (K < 1 || K > 8 || n_tiles < 0) return 0;
    return kLabelBytes + kq::viterbi_decision_bytes(K, n_tiles);
}

int kq_viterbi_encode(const float* tiles, int64_t n_tiles, int K, const uint16_t* labels, int tailbite_ctx,
                      float* out_vals, uint16_t* out_states, void* workspace, size_t workspace_bytes,
                      void* stream) {
    return kq::viterbi_encode(tiles, n_tiles, K, labels, tailbite_ctx, out_vals, out_states, workspace,
                              workspace_bytes, static_cast<cudaStream_t>(stream));
}

int kq_quantize_tiles_sqg(const float* tiles, float* out_vals, uint16_t* out_states, int64_t n_tiles,
                          const uint8_t* lut, int K, int tailbite_ctx, void* workspace, size_t workspace_bytes,
                          void* stream) {
    if (!lut) { kq::set_error("quantize_tiles_sqg: null LUT"); return KQ_ERR_ARG; }
    return quantize_with_kind(tiles, out_vals, out_states, n_tiles, KQ_CB_SQG, lut, K, tailbite_ctx, workspace,
                              workspace_bytes, stream);
}

int kq_quantize_tiles_procedural(const float* tiles, float* out_vals, uint16_t* out_states, int64_t n_tiles,
                                 int K, int codebook, int tailbite_ctx, void* workspace, size_t workspace_bytes,
                                 void* stream) {
    if (codebook != KQ_CB_MCG && codebook != KQ_CB_MUL1 && codebook != KQ_CB_3INST) {
        kq::set_error("quantize_tiles_procedural: codebook must be MCG (1), MUL1 (2) or 3INST (0)");
        return KQ_ERR_ARG;
    }
    return quantize_with_kind(tiles, out_vals, out_states, n_tiles, codebook, nullptr, K, tailbite_ctx, workspace,
                              workspace_bytes, stream);
}

int kq_pack_trellis(const uint16_t* states, int64_t n_tiles, int K, uint16_t* packed, void* stream) {
    return kq::pack_trellis(states, n_tiles, K, packed, static_cast<cudaStream_t>(stream));
}

int kq_unpack_trellis_states(const uint16_t* packed, int64_t n_tiles, int K, uint16_t* states, void* stream) {
    return kq::unpack_trellis_states(packed, n_tiles, K, states, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
