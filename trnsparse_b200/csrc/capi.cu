// Error plumbing shared by every C-ABI entry point.
#include "common.cuh"
#include "ptx.cuh"

#include <string.h>

namespace tsb {

__device__ int g_device_error = 0;

static thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return TRNSPARSE_OK;
  return fail(TRNSPARSE_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace tsb

extern "C" const char* trnsparse_last_error(void) { return tsb::g_last_error; }

extern "C" int trnsparse_version(void) { return 100; /* 0.1.0 */ }

extern "C" int trnsparse_device_error(int* code, int clear) {
  if (!code) return tsb::fail(TRNSPARSE_ERR_ARG, "device_error: null output");
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, tsb::g_device_error, sizeof(int));
  if (e != cudaSuccess) return tsb::cuda_status(e, "device_error: read");
  *code = v;
  if (clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(tsb::g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) return tsb::cuda_status(e, "device_error: clear");
  }
  return TRNSPARSE_OK;
}
