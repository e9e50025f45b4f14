// Host-side helpers shared by the C-ABI translation units: the per-thread error message, status conversion and the
// per-device kernel status word.
#pragma once

#include "../../include/mkb_image.h"

#include <cuda_runtime.h>
#include <cstdint>
#include <string>

namespace mkb {

// Sets the calling thread's error message and returns `code`.
mkb_status fail(mkb_status code, const std::string& msg);
// MKB_OK for cudaSuccess, else MKB_ERR_CUDA with "<what>: <cuda error string>".
mkb_status cuda_status(cudaError_t e, const char* what);
// Counts kernel launches made by this library (mkb_kernel_launches).
void count_launch(unsigned long long n = 1);
// The current device's kernel status word (allocated on first use; lives until process exit).
uint32_t* device_status_word();

#ifndef MKB_TRY
#define MKB_TRY(expr)                                                                                                  \
    do {                                                                                                               \
        mkb_status s_ = (expr);                                                                                        \
        if (s_ != MKB_OK)                                                                                              \
            return s_;                                                                                                 \
    } while (0)
#endif

#define MKB_TRY_CUDA(expr, what)                                                                                       \
    do {                                                                                                               \
        cudaError_t e_ = (expr);                                                                                       \
        if (e_ != cudaSuccess)                                                                                         \
            return ::mkb::cuda_status(e_, what);                                                                       \
    } while (0)

}  // namespace mkb
