// Host-side plumbing shared by the .cu files of libnvfp4_b200: status codes,
// the thread-local error message, and the per-device error word.
#pragma once
#include <cstdint>
#include <cstdio>
#include <cstdarg>
#include <cuda_runtime.h>
#include "../../include/nvfp4_b200.h"

namespace nvfp4 {

// Records a printf-style message for nvfp4_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);

// Maps a CUDA runtime error to NVFP4_ERR_CUDA with its name in the message.
inline int cuda_fail(cudaError_t e, const char* what) {
  return fail(NVFP4_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// Device address of this device's error word (bounded waits OR bits into it).
// Resolved once per device with cudaGetSymbolAddress; nullptr on failure.
uint32_t* device_error_word();

// Number of SMs of the current device (cached per device).
int sm_count();

// Launch-error check after a <<<>>> launch.
inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? NVFP4_OK : cuda_fail(e, what);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace nvfp4
