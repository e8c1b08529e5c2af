// ALU roofline probe: a dependent-free stream of __hfma2 instructions.
//
// The Viterbi kernel is bound by binary16x2 issue.  Its roofline denominator
// is the measured HFMA2 rate of this GPU.  The probe runs 8 independent FMA
// chains per thread over a grid that fills every SM.
#include "kq_common.cuh"

namespace kq {
namespace {

__global__ void __launch_bounds__(512) hfma2_probe_kernel(uint32_t* out, int iters) {
    half2 a[8];
    const half2 m = __float2half2_rn(0.999f), c = __float2half2_rn(1e-3f);
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = __float2half2_rn(0.001f * (threadIdx.x + j));
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int r = 0; r < 16; ++r)
#pragma unroll
            for (int j = 0; j < 8; ++j) a[j] = __hfma2(a[j], m, c);
    }
    half2 s = a[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) s = __hadd2(s, a[j]);
    if (__half2float(__low2half(s)) == 12345.f) out[blockIdx.x] = 1u;   // keep the chains alive
}

}  // namespace
}  // namespace kq

extern "C" int kq_probe_hfma2(void* out, int iters, int blocks, int threads, void* stream) {
    if (!out || iters <= 0 || blocks <= 0 || threads <= 0 || threads > 512) {
        kq::set_error("kq_probe_hfma2: bad arguments");
        return KQ_ERR_ARG;
    }
    kq::hfma2_probe_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<uint32_t*>(out), iters);
    return kq::check_launch("hfma2_probe_kernel");
}
