// Shared definitions for the kquant_b200 sm_100a kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include "../../include/kq_b200.h"

#define KQ_H_INF_BITS 0x7C00u

namespace kq {

// Status reporting: the C-ABI never throws; it returns a KQ_* status code and
// keeps a per-thread message for kq_last_error().
void set_error(const char* fmt, ...);

inline int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s: %s", what, cudaGetErrorString(e));
        return KQ_ERR_CUDA;
    }
    return KQ_OK;
}

int sm_count(int* out);

}  // namespace kq
