// common.hpp -- status plumbing shared by every C-ABI entry point.
#pragma once

#include <cstdarg>
#include <cstdio>
#include <string>

#include <cuda_runtime.h>

#include "../../include/tensoroperations_b200.h"

namespace to_b200 {

// Record a one-line reason for the calling thread and return `status`.
int set_error(int status, const char* fmt, ...);

// Clear the calling thread's reason (successful call).
inline int ok() { return TO_OK; }

// Convert a CUDA error into TO_ERR_CUDA with the call site's text.
inline int cuda_fail(cudaError_t e, const char* what) {
  return set_error(TO_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e),
                   cudaGetErrorString(e));
}

#define TO_CUDA_TRY(expr)                                  \
  do {                                                     \
    cudaError_t to_e_ = (expr);                            \
    if (to_e_ != cudaSuccess) return ::to_b200::cuda_fail(to_e_, #expr); \
  } while (0)

// SM count of the current device (cached per device id), or <0 on failure.
int device_sm_count(int* device_out);

// Status word of the tensor-core contraction kernels (their translation unit's
// own device symbol): *value = 0 or a to_status; reset clears it.
int chain_device_status(int reset, int* value);

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

}  // namespace to_b200
