// Allocation-free BSR conjugate gradient.
//
// Some callers cannot call cudaMalloc at all: code running inside a custom
// allocator or a memory-pool callback, embedders whose memory budget is
// fixed up front, or hosts that forbid device allocation after start-up. For
// them this file provides one entry point, trnsparse_bsr_cg_noalloc, that runs
// the same device-resident PCG as trnsparse_bsr_cg_start/_iterate but keeps
// its scratch (status record, per-iteration scalars and the r, p, p', Ap
// vectors) in a fixed array compiled into the library instead of a workspace
// the caller allocates. Every GPU that loads the library holds that array
// (kNoAllocScratchBytes) until the process exits.
#include <mutex>

#include "common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;  // 64 MiB

// The scratch lives in device memory. Host code must not pass `g_cg_scratch`
// itself to a kernel: on the host that name is only a stand-in, so its device
// address is looked up with cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_cg_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (looked up once
// per device, with that device current, and kept for the life of the process:
// after a cudaDeviceReset the library's device module is loaded again and the
// array may move, so the entry point must not be used after a reset).
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return tsb::cuda_status(e, "bsr_cg_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return tsb::fail(TRNSPARSE_ERR_ARG, "bsr_cg_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_cg_scratch);
    if (e != cudaSuccess || !p) return tsb::cuda_status(e, "bsr_cg_noalloc: cudaGetSymbolAddress");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return TRNSPARSE_OK;
}

}  // namespace

extern "C" int trnsparse_bsr_cg_noalloc(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                                        const int* col_idx, const float* blocks, const float* b_vec, float* x,
                                        int x_is_zero, const float* inv_d, double tol, int max_iter,
                                        void* status_out, void* stream) {
  TSB_REQUIRE(n >= 0 && max_iter >= 0, "bsr_cg_noalloc: negative n or max_iter");
  const size_t need = trnsparse_bsr_cg_workspace_size(n, max_iter);
  if (need > kNoAllocScratchBytes)
    return tsb::fail(TRNSPARSE_ERR_ARG,
                     "bsr_cg_noalloc: n=%lld, max_iter=%d needs %zu bytes of scratch, more than the fixed %zu; "
                     "use trnsparse_bsr_cg_start/_iterate with a caller workspace",
                     (long long)n, max_iter, need, kNoAllocScratchBytes);
  void* ws = nullptr;
  int rc = scratch_address(&ws);
  if (rc) return rc;
  // cg_start clears the status record and the scalar slots and initialises r
  // and p_{-1}, so nothing left by an earlier call leaks into this solve.
  rc = trnsparse_bsr_cg_start(m, n, b, n_blocks, row_ptr, col_idx, blocks, b_vec, x, x_is_zero, inv_d, max_iter, ws,
                              kNoAllocScratchBytes, stream);
  if (rc) return rc;
  rc = trnsparse_bsr_cg_iterate(m, n, b, n_blocks, row_ptr, col_idx, blocks, x, inv_d, tol, max_iter, 0, max_iter + 1,
                                ws, stream);
  if (rc) return rc;
  if (status_out) {
    cudaError_t e = cudaMemcpyAsync(status_out, ws, 64, cudaMemcpyDeviceToDevice, tsb::as_stream(stream));
    if (e != cudaSuccess) return tsb::cuda_status(e, "bsr_cg_noalloc: copy status");
  }
  return TRNSPARSE_OK;
}
