// Entry points of the tail-biting Viterbi tile encoder: K2..K4 dispatch to the
// tile-paired sm_100a kernel (kq_viterbi_pair.cu), K1 and K5..K8 to the
// wide-butterfly kernel (kq_viterbi_wide.cu).
#include "kq_common.cuh"

namespace kq {

size_t pair_decision_bytes(int K, int64_t n, int sms);
template <int K>
int pair_launch(const float* tiles, int64_t n, const uint16_t* labels, int C, float* vals, uint16_t* states,
                uint8_t* ws, size_t ws_bytes, cudaStream_t stream);

bool wide_supported(int K);
size_t wide_decision_bytes(int K, int64_t n, int sms);
int wide_encode(const float* tiles, int64_t n, int K, const uint16_t* labels, int C, float* vals, uint16_t* states,
                uint8_t* ws, size_t ws_bytes, int max_ctas, cudaStream_t stream);

size_t viterbi_decision_bytes(int K, int64_t n) {
    int sms = 0;
    if (sm_count(&sms)) return 0;
    if (wide_supported(K)) return wide_decision_bytes(K, n, sms);
    return pair_decision_bytes(K, n, sms);
}

int viterbi_encode(const float* tiles, int64_t n, int K, const uint16_t* labels, int C, float* vals,
                   uint16_t* states, void* ws, size_t ws_bytes, cudaStream_t stream) {
    if (n < 0 || !labels || (n > 0 && (!tiles || !vals || !states))) {
        set_error("viterbi: null pointer or negative tile count");
        return KQ_ERR_ARG;
    }
    if (K < 1 || K > 8) { set_error("viterbi: K must be in 1..8 (got %d)", K); return KQ_ERR_ARG; }
    if (C < 1 || C > 128) { set_error("tailbite_context must be in 1..128 (got %d)", C); return KQ_ERR_ARG; }
    if (n == 0) return KQ_OK;
    if (((uintptr_t)labels & 3) || ((uintptr_t)ws & 15)) {
        set_error("viterbi: labels must be 4-byte and workspace 16-byte aligned");
        return KQ_ERR_ALIGN;
    }
    auto* w = static_cast<uint8_t*>(ws);
    if (wide_supported(K)) return wide_encode(tiles, n, K, labels, C, vals, states, w, ws_bytes, 0, stream);
    switch (K) {
    case 2: return pair_launch<2>(tiles, n, labels, C, vals, states, w, ws_bytes, stream);
    case 3: return pair_launch<3>(tiles, n, labels, C, vals, states, w, ws_bytes, stream);
    default: return pair_launch<4>(tiles, n, labels, C, vals, states, w, ws_bytes, stream);
    }
}

}  // namespace kq
