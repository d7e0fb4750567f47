// Shared helpers for the trnsparse_b200 CUDA library: status codes, the
// thread-local last-error string, launch checks and small device utilities.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/trnsparse_b200.h"

namespace tsb {

// Records a formatted message as the calling thread's last error and returns
// `code`, so entry points can `return fail(TRNSPARSE_ERR_ARG, "...")`.
int fail(int code, const char* fmt, ...);

// Converts a CUDA error into a status (TRNSPARSE_OK when `e == cudaSuccess`).
int cuda_status(cudaError_t e, const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs on the current device (cached per device).
int sm_count();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace tsb

#define TSB_CHECK_LAUNCH(what)                                        \
  do {                                                                \
    cudaError_t _e = cudaGetLastError();                              \
    if (_e != cudaSuccess) return ::tsb::cuda_status(_e, what);       \
  } while (0)

#define TSB_REQUIRE(cond, ...)                                        \
  do {                                                                \
    if (!(cond)) return ::tsb::fail(TRNSPARSE_ERR_ARG, __VA_ARGS__);  \
  } while (0)

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
