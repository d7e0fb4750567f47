// CSR SpMV / SpMM kernels (HBM-bound).
//
// Both kernels are "CSR-stream" kernels: a CTA owns a contiguous run of rows,
// stages that run's slice of `values` and `col_indices` into shared memory
// with 16-byte cp.async copies (fully coalesced, many bytes in flight), and
// then computes its rows out of shared memory. x (SpMV) and B rows (SpMM)
// are gathered through the read-only path; their reuse in banded matrices
// is served by L1/L2. A CTA whose slice does not fit its shared-memory
// budget (rows much longer than average) falls back, for that CTA only, to a
// warp-per-row loop that streams the row straight from global memory, so any
// row-length distribution is handled.
//
// Semantics follow the reference's PyTorch path: trnsparse/ops.py:30-48
// (spmv: result = alpha * (A @ x); if y given and beta != 0: result + beta*y)
// and ops.py:51-78 (spmm, same with a dense right-hand side).
#include "common.cuh"

namespace tsb {
namespace {

constexpr int kThreads = 256;

template <typename T> struct Vec16;
template <> struct Vec16<float> { using type = float4; static constexpr int n = 4; };
template <> struct Vec16<double> { using type = double2; static constexpr int n = 2; };

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;\n" ::: "memory");
}

__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }

// alpha*acc (+ beta*y) with the reference's separate roundings.
template <typename T>
__device__ __forceinline__ T epilogue(T acc, T alpha, const T* y, T beta, int64_t i) {
  T r = mul_rn(alpha, acc);
  if (y != nullptr) r = add_rn(r, mul_rn(beta, y[i]));
  return r;
}

// Copies elements [s0, e) of `src` (s0 aligned down to a 16-byte chunk) into
// `dst`, where dst[0] corresponds to src[s0]. Uses 16-byte cp.async for every
// chunk that lies inside [0, total); the ragged tail is copied with plain loads.
template <typename E>
__device__ __forceinline__ void stage_span(E* dst, const E* __restrict__ src, int64_t s0, int64_t e,
                                           int64_t total, bool vec_ok) {
  constexpr int V = 16 / sizeof(E);
  if (vec_ok) {
    const int64_t nchunks = (e - s0 + V - 1) / V;
    for (int64_t c = threadIdx.x; c < nchunks; c += blockDim.x) {
      const int64_t g = s0 + c * V;
      if (g + V <= total) {
        cp_async16(dst + c * V, src + g);
      } else {
        for (int t = 0; t < V && g + t < total; ++t) dst[c * V + t] = src[g + t];
      }
    }
  } else {
    for (int64_t c = threadIdx.x; c < e - s0; c += blockDim.x) dst[c] = src[s0 + c];
  }
}

struct Stage {
  int64_t s, e;   // absolute nnz range of the CTA's rows
  int dv, dc;     // offset of element s inside the staged value / column arrays
  bool fits;
};

// Loads the CTA's row pointers (relative to s) and, if the slice fits `cap`,
// its values and column indices into shared memory.
template <typename I, typename T>
__device__ __forceinline__ Stage stage_rows(unsigned char* smem, int cap, const I* __restrict__ rp,
                                            const I* __restrict__ ci, const T* __restrict__ v,
                                            int64_t nnz, int64_t r0, int nrows, bool vec_ok,
                                            int** rps_out, T** vs_out, I** cs_out) {
  int* rps = reinterpret_cast<int*>(smem);
  const int rp_words = (nrows + 1 + 3) & ~3;
  T* vs = reinterpret_cast<T*>(smem + sizeof(int) * rp_words);
  // keep 16-byte alignment of the value and column regions
  const size_t vbytes = ((size_t)(cap + 16) * sizeof(T) + 15) & ~(size_t)15;
  I* cs = reinterpret_cast<I*>(reinterpret_cast<unsigned char*>(vs) + vbytes);
  *rps_out = rps;
  *vs_out = vs;
  *cs_out = cs;

  Stage st;
  st.s = static_cast<int64_t>(rp[r0]);
  st.e = static_cast<int64_t>(rp[r0 + nrows]);
  st.fits = (st.e - st.s) <= cap;
  if (st.fits) {
    constexpr int VT = 16 / sizeof(T);
    constexpr int VC = 16 / sizeof(I);
    const int64_t s0v = vec_ok ? (st.s & ~(int64_t)(VT - 1)) : st.s;
    const int64_t s0c = vec_ok ? (st.s & ~(int64_t)(VC - 1)) : st.s;
    st.dv = static_cast<int>(st.s - s0v);
    st.dc = static_cast<int>(st.s - s0c);
    for (int r = threadIdx.x; r <= nrows; r += blockDim.x)
      rps[r] = static_cast<int>(static_cast<int64_t>(rp[r0 + r]) - st.s);
    stage_span<T>(vs, v, s0v, st.e, nnz, vec_ok);
    stage_span<I>(cs, ci, s0c, st.e, nnz, vec_ok);
    cp_async_wait_all();
  } else {
    st.dv = st.dc = 0;
  }
  __syncthreads();
  return st;
}

template <typename I, typename T>
__global__ void __launch_bounds__(kThreads)
csr_spmv_kernel(int64_t m, int64_t nnz, const I* __restrict__ rp, const I* __restrict__ ci,
                const T* __restrict__ v, const T* __restrict__ x, T alpha, const T* __restrict__ y,
                T beta, T* __restrict__ out, int rows_per_cta, int cap, bool vec_ok) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_cta;
  const int nrows = static_cast<int>((m - r0 < (int64_t)rows_per_cta ? m - r0 : (int64_t)rows_per_cta));
  int* rps;
  T* vs;
  I* cs;
  const Stage st = stage_rows<I, T>(smem, cap, rp, ci, v, nnz, r0, nrows, vec_ok, &rps, &vs, &cs);

  if (st.fits) {
    const T* vrow = vs + st.dv;
    const I* crow = cs + st.dc;
    for (int r = threadIdx.x; r < nrows; r += blockDim.x) {
      const int a = rps[r], b = rps[r + 1];
      T acc = T(0);
      for (int j = a; j < b; ++j) acc += vrow[j] * __ldg(x + static_cast<int64_t>(crow[j]));
      out[r0 + r] = epilogue<T>(acc, alpha, y, beta, r0 + r);
    }
  } else {
    // warp-per-row straight from global memory
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int r = warp; r < nrows; r += kThreads / 32) {
      const int64_t a = static_cast<int64_t>(rp[r0 + r]), b = static_cast<int64_t>(rp[r0 + r + 1]);
      T acc = T(0);
      for (int64_t j = a + lane; j < b; j += 32) acc += __ldg(v + j) * __ldg(x + static_cast<int64_t>(__ldg(ci + j)));
      acc = warp_sum(acc);
      if (lane == 0) out[r0 + r] = epilogue<T>(acc, alpha, y, beta, r0 + r);
    }
  }
}

// SpMM: a group of G lanes owns one row; each lane owns VEC-wide column
// chunks c = lane_in_group + G*t of the k output columns.
template <typename I, typename T, int VEC>
__global__ void __launch_bounds__(kThreads)
csr_spmm_kernel(int64_t m, int64_t k, int64_t nnz, const I* __restrict__ rp, const I* __restrict__ ci,
                const T* __restrict__ v, const T* __restrict__ B, int64_t ldb, T alpha,
                const T* __restrict__ C, int64_t ldc, T beta, T* __restrict__ out, int64_t ldo,
                int rows_per_cta, int cap, bool vec_ok, int G) {
  extern __shared__ __align__(16) unsigned char smem[];
  using VT = typename Vec16<T>::type;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_cta;
  const int nrows = static_cast<int>((m - r0 < (int64_t)rows_per_cta ? m - r0 : (int64_t)rows_per_cta));
  int* rps;
  T* vs;
  I* cs;
  const Stage st = stage_rows<I, T>(smem, cap, rp, ci, v, nnz, r0, nrows, vec_ok, &rps, &vs, &cs);

  const int g = threadIdx.x % G;
  const int grp = threadIdx.x / G;
  const int ngrp = kThreads / G;
  const int64_t nchunk = k / VEC;
  for (int r = grp; r < nrows; r += ngrp) {
    int64_t a, b;
    if (st.fits) { a = rps[r]; b = rps[r + 1]; }
    else { a = static_cast<int64_t>(rp[r0 + r]) - st.s; b = static_cast<int64_t>(rp[r0 + r + 1]) - st.s; }
    const int64_t row = r0 + r;
    for (int64_t c = g; c < nchunk; c += G) {
      if constexpr (VEC == 1) {
        T acc = T(0);
        for (int64_t j = a; j < b; ++j) {
          T val; int64_t col;
          if (st.fits) { val = vs[st.dv + j]; col = static_cast<int64_t>(cs[st.dc + j]); }
          else { val = __ldg(v + st.s + j); col = static_cast<int64_t>(__ldg(ci + st.s + j)); }
          acc += val * __ldg(B + col * ldb + c);
        }
        out[row * ldo + c] = epilogue<T>(acc, alpha, C ? C + row * ldc : nullptr, beta, c);
      } else {
        T acc[VEC];
#pragma unroll
        for (int q = 0; q < VEC; ++q) acc[q] = T(0);
        for (int64_t j = a; j < b; ++j) {
          T val; int64_t col;
          if (st.fits) { val = vs[st.dv + j]; col = static_cast<int64_t>(cs[st.dc + j]); }
          else { val = __ldg(v + st.s + j); col = static_cast<int64_t>(__ldg(ci + st.s + j)); }
          const VT bv = __ldg(reinterpret_cast<const VT*>(B + col * ldb) + c);
          const T* bp = reinterpret_cast<const T*>(&bv);
#pragma unroll
          for (int q = 0; q < VEC; ++q) acc[q] += val * bp[q];
        }
        VT o;
        T* op = reinterpret_cast<T*>(&o);
        const T* crow = C ? C + row * ldc + c * VEC : nullptr;
#pragma unroll
        for (int q = 0; q < VEC; ++q) op[q] = epilogue<T>(acc[q], alpha, crow, beta, q);
        reinterpret_cast<VT*>(out + row * ldo)[c] = o;
      }
    }
  }
}

// Rows per CTA so that a CTA stages about `target` stored entries.
inline int pick_rows(int64_t m, int64_t nnz, int target) {
  double avg = m > 0 ? static_cast<double>(nnz) / static_cast<double>(m) : 1.0;
  if (avg < 0.25) avg = 0.25;
  int rows = 64;
  while (rows < 8192 && rows * 2 * avg <= target) rows *= 2;
  return rows;
}

template <typename I, typename T>
size_t smem_bytes(int rows, int cap) {
  const size_t rp_words = (rows + 1 + 3) & ~3;
  const size_t vbytes = ((size_t)(cap + 16) * sizeof(T) + 15) & ~(size_t)15;
  return sizeof(int) * rp_words + vbytes + (size_t)(cap + 16) * sizeof(I);
}

template <typename I, typename T>
int launch_spmv(int64_t m, int64_t nnz, const void* rp, const void* ci, const void* v, const void* x,
                double alpha, const void* y, double beta, void* out, cudaStream_t st) {
  const int rows = pick_rows(m, nnz, 4096);
  const double avg = m > 0 ? static_cast<double>(nnz) / m : 0.0;
  int cap = static_cast<int>(rows * avg * 1.25) + 256;
  if (cap > 8192) cap = 8192;
  const bool vec_ok = aligned16(v) && aligned16(ci);
  const size_t sm = smem_bytes<I, T>(rows, cap);
  auto kern = csr_spmv_kernel<I, T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return cuda_status(e, "csr_spmv: set smem");
  const int64_t grid = (m + rows - 1) / rows;
  if (grid > 0x7fffffff) return fail(TRNSPARSE_ERR_ARG, "csr_spmv: m=%lld too large", (long long)m);
  kern<<<(unsigned)grid, kThreads, sm, st>>>(m, nnz, (const I*)rp, (const I*)ci, (const T*)v, (const T*)x,
                                             (T)alpha, (const T*)y, (T)beta, (T*)out, rows, cap, vec_ok);
  TSB_CHECK_LAUNCH("csr_spmv launch");
  return TRNSPARSE_OK;
}

template <typename I, typename T>
int launch_spmm(int64_t m, int64_t k, int64_t nnz, const void* rp, const void* ci, const void* v,
                const void* B, int64_t ldb, double alpha, const void* C, int64_t ldc, double beta,
                void* out, int64_t ldo, cudaStream_t st) {
  constexpr int V = Vec16<T>::n;
  const bool vec_cols = (k % V == 0) && (ldb % V == 0) && (ldo % V == 0) && aligned16(B) &&
                        aligned16(out) && (C == nullptr || ((ldc % V == 0) && aligned16(C)));
  const int64_t nchunk = vec_cols ? k / V : k;
  int G = 1;
  while (G < 32 && G < nchunk) G *= 2;
  // rows per CTA: enough row-groups to fill the CTA, and a slice that fits
  const int rows = pick_rows(m, nnz, 2048);
  const double avg = m > 0 ? static_cast<double>(nnz) / m : 0.0;
  int cap = static_cast<int>(rows * avg * 1.25) + 256;
  if (cap > 8192) cap = 8192;
  const bool vec_ok = aligned16(v) && aligned16(ci);
  const size_t sm = smem_bytes<I, T>(rows, cap);
  const int64_t grid = (m + rows - 1) / rows;
  if (grid > 0x7fffffff) return fail(TRNSPARSE_ERR_ARG, "csr_spmm: m=%lld too large", (long long)m);
  if (vec_cols) {
    auto kern = csr_spmm_kernel<I, T, V>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return cuda_status(e, "csr_spmm: set smem");
    kern<<<(unsigned)grid, kThreads, sm, st>>>(m, k, nnz, (const I*)rp, (const I*)ci, (const T*)v,
                                               (const T*)B, ldb, (T)alpha, (const T*)C, ldc, (T)beta,
                                               (T*)out, ldo, rows, cap, vec_ok, G);
  } else {
    auto kern = csr_spmm_kernel<I, T, 1>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return cuda_status(e, "csr_spmm: set smem");
    kern<<<(unsigned)grid, kThreads, sm, st>>>(m, k, nnz, (const I*)rp, (const I*)ci, (const T*)v,
                                               (const T*)B, ldb, (T)alpha, (const T*)C, ldc, (T)beta,
                                               (T*)out, ldo, rows, cap, vec_ok, G);
  }
  TSB_CHECK_LAUNCH("csr_spmm launch");
  return TRNSPARSE_OK;
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" int trnsparse_csr_spmv(int64_t m, int64_t n, int64_t nnz, int index_type, int dtype,
                                  const void* row_ptrs, const void* col_indices, const void* values,
                                  const void* x, double alpha, const void* y, double beta, void* out,
                                  void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && nnz >= 0, "csr_spmv: negative size (m=%lld n=%lld nnz=%lld)",
              (long long)m, (long long)n, (long long)nnz);
  if (m == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(row_ptrs && out, "csr_spmv: null row_ptrs/out");
  TSB_REQUIRE(nnz == 0 || (col_indices && values && x), "csr_spmv: null col_indices/values/x");
  if (y != nullptr && beta == 0.0) y = nullptr;
  cudaStream_t st = as_stream(stream);
  if (dtype == TRNSPARSE_F32) {
    if (index_type == TRNSPARSE_I32) return launch_spmv<int32_t, float>(m, nnz, row_ptrs, col_indices, values, x, alpha, y, beta, out, st);
    if (index_type == TRNSPARSE_I64) return launch_spmv<int64_t, float>(m, nnz, row_ptrs, col_indices, values, x, alpha, y, beta, out, st);
  } else if (dtype == TRNSPARSE_F64) {
    if (index_type == TRNSPARSE_I32) return launch_spmv<int32_t, double>(m, nnz, row_ptrs, col_indices, values, x, alpha, y, beta, out, st);
    if (index_type == TRNSPARSE_I64) return launch_spmv<int64_t, double>(m, nnz, row_ptrs, col_indices, values, x, alpha, y, beta, out, st);
  } else {
    return fail(TRNSPARSE_ERR_DTYPE, "csr_spmv: dtype %d not supported (F32, F64)", dtype);
  }
  return fail(TRNSPARSE_ERR_DTYPE, "csr_spmv: index type %d not supported (I32, I64)", index_type);
}

extern "C" int trnsparse_csr_spmm(int64_t m, int64_t n, int64_t k, int64_t nnz, int index_type, int dtype,
                                  const void* row_ptrs, const void* col_indices, const void* values,
                                  const void* B, int64_t ldb, double alpha, const void* C, int64_t ldc,
                                  double beta, void* out, int64_t ldo, void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && k >= 0 && nnz >= 0, "csr_spmm: negative size");
  if (m == 0 || k == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(row_ptrs && out, "csr_spmm: null row_ptrs/out");
  TSB_REQUIRE(nnz == 0 || (col_indices && values && B), "csr_spmm: null col_indices/values/B");
  TSB_REQUIRE(ldb >= k && ldo >= k, "csr_spmm: ldb=%lld / ldo=%lld smaller than k=%lld", (long long)ldb,
              (long long)ldo, (long long)k);
  if (C != nullptr && beta == 0.0) C = nullptr;
  TSB_REQUIRE(C == nullptr || ldc >= k, "csr_spmm: ldc smaller than k");
  cudaStream_t st = as_stream(stream);
  if (dtype == TRNSPARSE_F32) {
    if (index_type == TRNSPARSE_I32) return launch_spmm<int32_t, float>(m, k, nnz, row_ptrs, col_indices, values, B, ldb, alpha, C, ldc, beta, out, ldo, st);
    if (index_type == TRNSPARSE_I64) return launch_spmm<int64_t, float>(m, k, nnz, row_ptrs, col_indices, values, B, ldb, alpha, C, ldc, beta, out, ldo, st);
  } else if (dtype == TRNSPARSE_F64) {
    if (index_type == TRNSPARSE_I32) return launch_spmm<int32_t, double>(m, k, nnz, row_ptrs, col_indices, values, B, ldb, alpha, C, ldc, beta, out, ldo, st);
    if (index_type == TRNSPARSE_I64) return launch_spmm<int64_t, double>(m, k, nnz, row_ptrs, col_indices, values, B, ldb, alpha, C, ldc, beta, out, ldo, st);
  } else {
    return fail(TRNSPARSE_ERR_DTYPE, "csr_spmm: dtype %d not supported (F32, F64)", dtype);
  }
  return fail(TRNSPARSE_ERR_DTYPE, "csr_spmm: index type %d not supported (I32, I64)", index_type);
}
