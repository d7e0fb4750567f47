// BSR matrix-vector product with pluggable input transform and epilogue.
//
// Every BSR solver iteration of the reference (trnsparse/iterative.py) is one
// `bsr_spmm(A, v[:, None])` followed by vector updates and inner products.
// Here the iteration is folded into the SpMV itself: an Op supplies the input
// vector on the fly (e.g. the CG direction p = z + beta * p_prev computed as
// it is gathered) and consumes each output row in an epilogue that performs
// the vector updates and block-reduces the partial inner products, which are
// accumulated in float64 with one atomic per CTA.
//
// Two kernels share the Op interface:
//  * bsr128_mv_kernel: block size 128, one CTA per block-row. Warp w owns
//    rows 16w..16w+15 of the block-row; lane l owns columns 4l..4l+3, so every
//    warp load is one fully coalesced 512-byte row of a block (streamed with
//    evict-first loads: the blocks are read once per product). HBM-bound.
//  * bsr_generic_mv_kernel: any block size; one thread per output row.
//
// Op interface (all __device__):
//   bool begin(int cta)                       uniform: false => CTA returns
//   float  x(int64_t col)                     input vector element
//   float4 x4(int64_t col)                    4 consecutive elements (col % 4 == 0)
//   void   row(int64_t row, float y, double* d0, double* d1)
//                                             epilogue; adds to 2 partial dots
//   void   finish(double d0, double d1)       CTA totals (thread 0 only)
#pragma once

#include <utility>

#include "common.cuh"

namespace tsb {

__device__ __forceinline__ double block_sum256(double v, double* red /* [8] */) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i];
  }
  return t;  // valid in thread 0
}

// Ops may define `void tail() const`, run by every thread of the CTA after
// finish() (used by the sharded solver to publish results from the last CTA).
template <class Op, class = void>
struct HasTail { static constexpr bool value = false; };
template <class Op>
struct HasTail<Op, decltype(void(std::declval<const Op&>().tail()))> { static constexpr bool value = true; };

template <class Op>
__device__ __forceinline__ void run_tail(const Op& op) {
  if constexpr (HasTail<Op>::value) op.tail();
}

#ifdef TSB_CG_TRACE
// Timing probe (compile-time only): CTA 0 of each launch takes a slot and
// stamps entry, after begin(), before finish() and after the tail.
extern __device__ unsigned long long g_cg_trace[512][8];
extern __device__ unsigned g_cg_trace_n;
extern __device__ unsigned long long g_cg_cta[512][4];  // per-CTA stamps of one iteration
__device__ __forceinline__ unsigned long long cgt_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
#define CGT_ENTER                                                              \
  __shared__ unsigned cgt_slot;                                                \
  if (blockIdx.x == 0 && threadIdx.x == 0) {                                   \
    cgt_slot = atomicAdd(&g_cg_trace_n, 1u) & 511u;                            \
    g_cg_trace[cgt_slot][0] = cgt_now();                                       \
  }
#define CGT(i) \
  if (blockIdx.x == 0 && threadIdx.x == 0) g_cg_trace[cgt_slot][i] = cgt_now()
#else
#define CGT_ENTER
#define CGT(i)
#endif

// KEEP: load the blocks with the default L2 policy (a matrix that fits in L2
// stays there across the iterations of a solver); otherwise stream them
// (evict-first), so a larger-than-L2 matrix does not flush the vectors.
template <class Op, bool KEEP = false>
__global__ void __launch_bounds__(256)
bsr128_mv_kernel(const int* __restrict__ row_ptr, const int* __restrict__ col_idx,
                 const float4* __restrict__ blocks, int n_block_rows, Op op) {
  __shared__ float ys[128];
  __shared__ double red[8];
  CGT_ENTER
  if (!op.begin(blockIdx.x)) return;
  CGT(1);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  double d0 = 0.0, d1 = 0.0;
  // one block-row per iteration; the grid may be smaller than the number of
  // block-rows (persistent CTAs), so per-CTA prologue costs are paid once
  for (int i = blockIdx.x; i < n_block_rows; i += gridDim.x) {
    float acc[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) acc[r] = 0.f;
    const int e = row_ptr[i + 1];
    for (int idx = row_ptr[i]; idx < e; ++idx) {
      const int64_t j = col_idx[idx];
      const float4 xv = op.x4(j * 128 + 4 * lane);
      const float4* bp = blocks + static_cast<int64_t>(idx) * 4096 + (w * 16) * 32 + lane;
      float4 a[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) a[r] = KEEP ? __ldg(bp + r * 32) : __ldcs(bp + r * 32);
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        acc[r] = fmaf(a[r].x, xv.x, acc[r]);
        acc[r] = fmaf(a[r].y, xv.y, acc[r]);
        acc[r] = fmaf(a[r].z, xv.z, acc[r]);
        acc[r] = fmaf(a[r].w, xv.w, acc[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const float v = warp_sum(acc[r]);
      if (lane == r) ys[w * 16 + r] = v;
    }
    __syncthreads();
    if (threadIdx.x < 128) op.row(static_cast<int64_t>(i) * 128 + threadIdx.x, ys[threadIdx.x], &d0, &d1);
    __syncthreads();
  }
  if (Op::kDots > 0) {
    const double t0 = block_sum256(d0, red);
    double t1 = 0.0;
    if (Op::kDots > 1) t1 = block_sum256(d1, red);
    if (threadIdx.x == 0) op.finish(t0, t1);
  }
  CGT(2);
  run_tail(op);
  CGT(3);
}

template <class Op>
__global__ void __launch_bounds__(256)
bsr_generic_mv_kernel(int64_t m, int64_t n, int b, const int* __restrict__ row_ptr,
                      const int* __restrict__ col_idx, const float* __restrict__ blocks, Op op) {
  __shared__ double red[8];
  if (!op.begin(blockIdx.x)) return;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  double d0 = 0.0, d1 = 0.0;
  if (row < m) {
    const int64_t i = row / b;
    const int rl = static_cast<int>(row - i * b);
    float acc = 0.f;
    const int e = row_ptr[i + 1];
    for (int idx = row_ptr[i]; idx < e; ++idx) {
      const int64_t j = col_idx[idx];
      const float* bp = blocks + static_cast<int64_t>(idx) * b * b + static_cast<int64_t>(rl) * b;
      for (int c = 0; c < b; ++c) {
        const int64_t col = j * b + c;
        if (col < n) acc = fmaf(bp[c], op.x(col), acc);
      }
    }
    op.row(row, acc, &d0, &d1);
  }
  if (Op::kDots > 0) {
    const double t0 = block_sum256(d0, red);
    double t1 = 0.0;
    if (Op::kDots > 1) t1 = block_sum256(d1, red);
    if (threadIdx.x == 0) op.finish(t0, t1);
  }
  run_tail(op);
}

// Geometry of a BSR operand as the kernels see it.
struct BsrDesc {
  int64_t m, n;          // element shape
  int b;                 // block size
  int64_t n_blocks;
  const int* row_ptr;    // ceil(m/b)+1, int32
  const int* col_idx;    // n_blocks, int32
  const float* blocks;   // n_blocks * b * b, row-major blocks
  bool fast() const {
    return b == 128 && m % 128 == 0 && n % 128 == 0 && aligned16(blocks);
  }
  int64_t block_rows() const { return (m + b - 1) / b; }
};

// Whether `bytes` of matrix blocks can stay resident in this device's L2
// across solver iterations (three quarters of it, leaving room for vectors).
inline bool fits_l2(size_t bytes) {
  static int l2 = -1;
  if (l2 < 0) {
    int dev = 0, v = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&v, cudaDevAttrL2CacheSize, dev) != cudaSuccess)
      v = 0;
    l2 = v;
  }
  return bytes * 4 <= static_cast<size_t>(l2) * 3;
}

// Launches the right kernel for `d`; `vec_ok` says the Op's x4 may be used.
// max_ctas > 0 caps the fast kernel's grid (persistent CTAs looping over block-rows).
template <class Op>
int launch_bsr_mv(const BsrDesc& d, const Op& op, bool vec_ok, cudaStream_t st, const char* what, int64_t max_ctas = 0,
                  bool keep_l2 = false) {
  if (d.fast() && vec_ok) {
    const int64_t nbr = d.block_rows();
    int64_t g = nbr;
    if (max_ctas > 0 && g > max_ctas) g = max_ctas;
    if (g > 0) {
      auto kern = keep_l2 ? bsr128_mv_kernel<Op, true> : bsr128_mv_kernel<Op, false>;
      kern<<<(unsigned)g, 256, 0, st>>>(d.row_ptr, d.col_idx, reinterpret_cast<const float4*>(d.blocks), (int)nbr, op);
    }
  } else {
    const int64_t g = (d.m + 255) / 256;
    if (g > 0) bsr_generic_mv_kernel<Op><<<(unsigned)g, 256, 0, st>>>(d.m, d.n, d.b, d.row_ptr, d.col_idx, d.blocks, op);
  }
  TSB_CHECK_LAUNCH(what);
  return TRNSPARSE_OK;
}

// Number of CTAs the launch above uses (for per-CTA bookkeeping).
inline int64_t bsr_mv_ctas(const BsrDesc& d, bool vec_ok) {
  return (d.fast() && vec_ok) ? d.block_rows() : (d.m + 255) / 256;
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

}  // namespace tsb
