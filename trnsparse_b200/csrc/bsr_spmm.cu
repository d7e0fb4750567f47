// BSR x dense (trnsparse/ops.py:162-210, `bsr_spmm`): generic CUDA-core path.
//
// Used for block sizes other than 128 and for shapes the tensor-core path
// does not take. One CTA computes a 32-row x 64-column tile of C; each
// thread owns one row and 8 consecutive columns and walks the stored blocks
// of its row's block-row (so block-rows of any size, including ones smaller
// than the tile, are handled), accumulating in float32 with FMA.
#include "common.cuh"

namespace tsb {
namespace {

__global__ void __launch_bounds__(256)
bsr_spmm_simt_kernel(int64_t m, int64_t n, int64_t k, int b, const int* __restrict__ row_ptr,
                     const int* __restrict__ col_idx, const float* __restrict__ blocks, const float* __restrict__ B,
                     int64_t ldb, float* __restrict__ C, int64_t ldc) {
  const int tx = threadIdx.x & 7, ty = threadIdx.x >> 3;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 32 + ty;
  const int64_t c0 = static_cast<int64_t>(blockIdx.y) * 64 + tx * 8;
  if (row >= m) return;
  float acc[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) acc[q] = 0.f;
  const int64_t i = row / b;
  const int rl = static_cast<int>(row - i * b);
  const int e = row_ptr[i + 1];
  for (int idx = row_ptr[i]; idx < e; ++idx) {
    const int64_t j = col_idx[idx];
    const float* ap = blocks + static_cast<int64_t>(idx) * b * b + static_cast<int64_t>(rl) * b;
    for (int c = 0; c < b; ++c) {
      const int64_t col = j * b + c;
      if (col >= n) break;
      const float a = __ldg(ap + c);
      const float* bp = B + col * ldb + c0;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (c0 + q < k) acc[q] = fmaf(a, __ldg(bp + q), acc[q]);
    }
  }
#pragma unroll
  for (int q = 0; q < 8; ++q)
    if (c0 + q < k) C[row * ldc + c0 + q] = acc[q];
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" int trnsparse_bsr_spmm_simt(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                                       const int* col_idx, const float* blocks, const float* B, int64_t k,
                                       int64_t ldb, float* C, int64_t ldc, void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && k >= 0 && b > 0 && n_blocks >= 0, "bsr_spmm: bad geometry");
  TSB_REQUIRE(ldb >= k && ldc >= k, "bsr_spmm: leading dimension smaller than k");
  if (m == 0 || k == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(row_ptr && C && (n_blocks == 0 || (col_idx && blocks && B)), "bsr_spmm: null pointer");
  dim3 grid((unsigned)((m + 31) / 32), (unsigned)((k + 63) / 64));
  TSB_REQUIRE(grid.y < 65536, "bsr_spmm: k=%lld too large for the CUDA-core path", (long long)k);
  bsr_spmm_simt_kernel<<<grid, 256, 0, as_stream(stream)>>>(m, n, k, b, row_ptr, col_idx, blocks, B, ldb, C, ldc);
  TSB_CHECK_LAUNCH("bsr_spmm_simt launch");
  return TRNSPARSE_OK;
}
