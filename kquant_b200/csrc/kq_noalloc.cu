// Allocation-free tile quantization: kq_quantize_tiles_sqg_noalloc.
//
// Some callers cannot call cudaMalloc at all: code running inside a host
// that owns every device allocation through its own pool (an inference
// server or a framework allocator that would be bypassed and starved), or
// code running where a fresh allocation would synchronize the device at a
// point the caller does not control.  This entry point serves them.  Its
// scratch (the label table and the Viterbi decision rows) lives in one
// file-scope __device__ array of fixed size, which every GPU that loads this
// library holds until process exit.  The caller still passes its own input
// and output buffers.
//
// The decision rows bound the grid: 32 MiB / (2 jobs x 256 rows x row bytes)
// is 8 CTAs at K2 and K3 (8 KiB rows) and 16 at K4 (4 KiB rows), against 148
// SMs.  Each CTA loops over its tile pairs, so results are exact, but a call
// runs about 9x (K4) to 18x (K2, K3) slower than kq_quantize_tiles_sqg with a
// full workspace.  The 4,096-tile cap is a chosen per-call bound (it keeps one
// call to a few tens of milliseconds); the scratch itself would serve any count.
//
// The scratch address is resolved once per device index and cached for the
// life of the process: the entry point assumes one primary context per device
// that is never reset (cudaDeviceReset or a context teardown would leave the
// cached address stale).
#include <mutex>
#include "kq_common.cuh"

namespace kq {
int build_labels(int kind, const uint8_t* lut, uint16_t* labels, cudaStream_t stream);
int viterbi_encode_bounded(const float* tiles, int64_t n, int K, const uint16_t* labels, int C, float* vals,
                           uint16_t* states, uint8_t* dec, size_t dec_bytes, cudaStream_t stream);
}  // namespace kq

namespace {

constexpr size_t kLabelBytes = 65536 * 2;
constexpr size_t kDecisionBytes = (size_t)32 << 20;
constexpr size_t kScratchBytes = kLabelBytes + kDecisionBytes;
constexpr int kMaxDevices = 64;

// The scratch.  In host code this name is only a stand-in for the symbol, not
// a device address; kernels receive the address from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

std::mutex g_mutex;
uint8_t* g_scratch_ptr[kMaxDevices] = {};

// Per device, once, with that device current: resolve the scratch address.
int scratch_for_current_device(uint8_t** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) { kq::set_error("cudaGetDevice: %s", cudaGetErrorString(e)); return KQ_ERR_CUDA; }
    if (dev < 0 || dev >= kMaxDevices) { kq::set_error("noalloc: device index %d out of range", dev); return KQ_ERR_ARG; }
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            kq::set_error("cudaGetSymbolAddress(noalloc scratch): %s", cudaGetErrorString(e));
            return KQ_ERR_CUDA;
        }
        g_scratch_ptr[dev] = static_cast<uint8_t*>(p);
    }
    *out = g_scratch_ptr[dev];
    return KQ_OK;
}

}  // namespace

extern "C" int kq_quantize_tiles_sqg_noalloc(const float* tiles, float* out_vals, uint16_t* out_states,
                                             int64_t n_tiles, const uint8_t* lut, int K, int tailbite_ctx,
                                             void* stream) {
    if (n_tiles < 0 || n_tiles > KQ_NOALLOC_MAX_TILES) {
        kq::set_error("kq_quantize_tiles_sqg_noalloc: n_tiles=%lld outside 0..%d (the per-call bound)",
                      (long long)n_tiles, KQ_NOALLOC_MAX_TILES);
        return KQ_ERR_ARG;
    }
    if (!lut) { kq::set_error("kq_quantize_tiles_sqg_noalloc: null LUT"); return KQ_ERR_ARG; }
    if (K < 2 || K > 4) { kq::set_error("kq_quantize_tiles_sqg_noalloc: K must be 2, 3 or 4 (got %d)", K); return KQ_ERR_ARG; }
    if (tailbite_ctx < 1 || tailbite_ctx > 128) {
        kq::set_error("tailbite_context must be in 1..128 (got %d)", tailbite_ctx);
        return KQ_ERR_ARG;
    }
    if (n_tiles > 0 && (!tiles || !out_vals || !out_states)) {
        kq::set_error("kq_quantize_tiles_sqg_noalloc: null buffer");
        return KQ_ERR_ARG;
    }
    uint8_t* scratch = nullptr;
    if (int rc = scratch_for_current_device(&scratch)) return rc;
    if (n_tiles == 0) return KQ_OK;
    auto s = static_cast<cudaStream_t>(stream);
    // Labels are rebuilt every call and every decision row is written before
    // it is read, so no part of the scratch has to start at zero.
    auto* labels = reinterpret_cast<uint16_t*>(scratch);
    if (int rc = kq::build_labels(KQ_CB_SQG, lut, labels, s)) return rc;
    return kq::viterbi_encode_bounded(tiles, n_tiles, K, labels, tailbite_ctx, out_vals, out_states,
                                      scratch + kLabelBytes, kDecisionBytes, s);
}
