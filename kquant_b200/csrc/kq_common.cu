// Error state and device queries shared by the C ABI.
#include <cstdarg>
#include <cstdio>
#include "kq_common.cuh"

namespace kq {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

const char* last_error() { return g_err; }

int sm_count(int* out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
        set_error("device query: %s", cudaGetErrorString(e));
        return KQ_ERR_CUDA;
    }
    return KQ_OK;
}

}  // namespace kq
