// Device-side sparse format construction: the reference's host-side
// BSRMatrix.from_dense (trnsparse/formats.py:184-221), CSR from_dense
// (formats.py:269-278) and COOMatrix.to_csr (formats.py:104-124), with the
// same results bit for bit.
//
//   BSR from dense   a CTA per 128x128 (b x b) block screens max |v| (a NaN
//                    in the block drops it, as torch.amax propagates NaN) and
//                    writes a 0/1 count; one exclusive scan over the block
//                    grid in row-major order gives every kept block its slot
//                    (the reference's nonzero() order) and the block-row
//                    pointers; a second pass copies the kept blocks, padded
//                    with zeros past the matrix edge.
//   CSR from dense   a warp per row counts |v| > threshold, a scan gives the
//                    row pointers, and a second pass compacts each row in
//                    column order with warp ballots.
//   COO -> CSR       row histogram (atomics) and scan, an atomic-cursor
//                    scatter of (col << 32 | entry index) keys into their row,
//                    then a sort of each row's keys: the entry index breaks
//                    ties, so the result is the stable (row, col) order of
//                    torch.argsort(rows * n + cols, stable=True). Rows of up to
//                    32 entries sort in a warp (shuffle bitonic), longer rows in a
//                    CTA (shared-memory bitonic over 2048-key chunks, then
//                    merge passes through a second key buffer).
// Thresholds compare in the matrix's dtype: the caller passes the threshold
// already rounded to it (torch rounds a Python scalar to the tensor's dtype).
#include <cuda_bf16.h>

#include "common.cuh"
#include "ptx.cuh"

namespace tsb {
namespace {

constexpr int kScanThreads = 1024;
constexpr int kScanItems = 4;
constexpr int kScanTile = kScanThreads * kScanItems;

template <typename T> __device__ __forceinline__ float fm_abs(T v);
template <> __device__ __forceinline__ float fm_abs<float>(float v) { return fabsf(v); }
template <> __device__ __forceinline__ float fm_abs<__nv_bfloat16>(__nv_bfloat16 v) {
  return fabsf(__bfloat162float(v));
}

// Inclusive block scan of one value per thread (kScanThreads threads); returns the
// thread's inclusive prefix and leaves the block total in *total.
__device__ __forceinline__ long long block_scan_incl(long long v, long long* warp_tot, long long* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long y = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += y;
  }
  if (lane == 31) warp_tot[w] = v;
  __syncthreads();
  if (w == 0) {
    long long t = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    warp_tot[lane] = t;  // inclusive over warps
  }
  __syncthreads();
  const long long off = w > 0 ? warp_tot[w - 1] : 0;
  if (total) *total = warp_tot[(blockDim.x >> 5) - 1];
  return v + off;
}

// ---------------------------------------------------------------- exclusive scan (in place)
// v[1..n] hold counts; afterwards v[0..n] hold their exclusive prefix (v[0] = 0).
__global__ void __launch_bounds__(kScanThreads) scan_tile_sums(const long long* __restrict__ v, int64_t n,
                                                               long long* __restrict__ part) {
  __shared__ long long wt[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile + threadIdx.x * kScanItems;
  long long s = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k)
    if (base + k < n) s += v[1 + base + k];
  long long tot;
  block_scan_incl(s, wt, &tot);
  if (threadIdx.x == 0) part[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(kScanThreads) scan_partials(long long* __restrict__ part, int64_t n_tiles) {
  __shared__ long long wt[32];
  long long carry = 0;
  for (int64_t b0 = 0; b0 < n_tiles; b0 += kScanThreads) {
    const int64_t i = b0 + threadIdx.x;
    const long long x = i < n_tiles ? part[i] : 0;
    long long tot;
    const long long inc = block_scan_incl(x, wt, &tot);
    if (i < n_tiles) part[i] = carry + inc - x;  // exclusive
    carry += tot;
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kScanThreads) scan_apply(long long* __restrict__ v, int64_t n,
                                                           const long long* __restrict__ part) {
  __shared__ long long wt[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile + threadIdx.x * kScanItems;
  long long x[kScanItems];
  long long s = 0;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    x[k] = base + k < n ? v[1 + base + k] : 0;
    s += x[k];
  }
  const long long inc = block_scan_incl(s, wt, nullptr);
  long long run = part[blockIdx.x] + inc - s;
#pragma unroll
  for (int k = 0; k < kScanItems; ++k) {
    run += x[k];
    if (base + k < n) v[1 + base + k] = run;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) v[0] = 0;
}

size_t scan_ws_bytes(int64_t n) { return sizeof(long long) * (size_t)((n + kScanTile - 1) / kScanTile + 1); }

int exclusive_scan(long long* v, int64_t n, long long* part, cudaStream_t st) {
  const int64_t tiles = (n + kScanTile - 1) / kScanTile;
  if (tiles == 0) return cuda_status(cudaMemsetAsync(v, 0, sizeof(long long), st), "scan: zero");
  scan_tile_sums<<<(unsigned)tiles, kScanThreads, 0, st>>>(v, n, part);
  scan_partials<<<1, kScanThreads, 0, st>>>(part, tiles);
  scan_apply<<<(unsigned)tiles, kScanThreads, 0, st>>>(v, n, part);
  TSB_CHECK_LAUNCH("exclusive scan");
  return TRNSPARSE_OK;
}

// ---------------------------------------------------------------- BSR from dense
// grid (block column, block row); writes pos[1 + i * nbc + j] = keep ? 1 : 0
template <typename T>
__global__ void __launch_bounds__(256) bsr_screen_kernel(int64_t m, int64_t n, const T* __restrict__ A, int64_t lda,
                                                         int b, float thr, int64_t nbc, long long* __restrict__ pos) {
  __shared__ float smax[8];
  __shared__ int snan[8];
  const int64_t j = blockIdx.x, i = blockIdx.y;
  float mx = 0.f;
  int nan = 0;
  const int64_t bb = static_cast<int64_t>(b) * b;
  for (int64_t e = threadIdx.x; e < bb; e += blockDim.x) {
    const int64_t r = i * b + e / b, c = j * b + e % b;
    if (r < m && c < n) {
      const float a = fm_abs<T>(A[r * lda + c]);
      nan |= a != a;
      mx = fmaxf(mx, a);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    nan |= __shfl_xor_sync(0xffffffffu, nan, o);
  }
  if ((threadIdx.x & 31) == 0) {
    smax[threadIdx.x >> 5] = mx;
    snan[threadIdx.x >> 5] = nan;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
      mx = fmaxf(mx, smax[w]);
      nan |= snan[w];
    }
    // padding zeros take part in the max, as in the reference's padded grid
    pos[1 + i * nbc + j] = (!nan && mx > thr) ? 1 : 0;
  }
}

__global__ void bsr_row_ptr_kernel(int64_t mb, int64_t nbc, const long long* __restrict__ pos,
                                   long long* __restrict__ row_ptr) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i <= mb;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    row_ptr[i] = pos[i * nbc];
}

// grid (block column, block row): copy a kept block to its slot
template <typename T>
__global__ void __launch_bounds__(256) bsr_fill_kernel(int64_t m, int64_t n, const T* __restrict__ A, int64_t lda,
                                                       int b, int64_t nbc, const long long* __restrict__ pos,
                                                       T* __restrict__ blocks, long long* __restrict__ col_idx) {
  const int64_t j = blockIdx.x, i = blockIdx.y;
  const int64_t k = i * nbc + j;
  const long long slot = pos[k];
  if (pos[k + 1] == slot) return;  // dropped
  if (threadIdx.x == 0) col_idx[slot] = j;
  const int64_t bb = static_cast<int64_t>(b) * b;
  T* dst = blocks + slot * bb;
  for (int64_t e = threadIdx.x; e < bb; e += blockDim.x) {
    const int64_t r = i * b + e / b, c = j * b + e % b;
    dst[e] = (r < m && c < n) ? A[r * lda + c] : T(0.f);
  }
}

// ---------------------------------------------------------------- CSR from dense
template <typename T>
__global__ void csr_count_kernel(int64_t m, int64_t n, const T* __restrict__ A, int64_t lda, float thr,
                                 long long* __restrict__ v) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m; r += warps) {
    const T* row = A + r * lda;
    long long c = 0;
    for (int64_t j = lane; j < n; j += 32) c += fm_abs<T>(row[j]) > thr ? 1 : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == 0) v[1 + r] = c;
  }
}

template <typename T>
__global__ void csr_fill_kernel(int64_t m, int64_t n, const T* __restrict__ A, int64_t lda, float thr,
                                const long long* __restrict__ row_ptr, T* __restrict__ vals,
                                long long* __restrict__ cols) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m; r += warps) {
    const T* row = A + r * lda;
    long long o = row_ptr[r];
    for (int64_t j0 = 0; j0 < n; j0 += 32) {
      const int64_t j = j0 + lane;
      T x = T(0.f);
      bool keep = false;
      if (j < n) {
        x = row[j];
        keep = fm_abs<T>(x) > thr;
      }
      const unsigned ball = __ballot_sync(0xffffffffu, keep);
      if (keep) {
        const long long p = o + __popc(ball & ((1u << lane) - 1u));
        vals[p] = x;
        cols[p] = j;
      }
      o += __popc(ball);
    }
  }
}

// ---------------------------------------------------------------- COO -> CSR
__global__ void coo_count_kernel(int64_t nnz, int64_t m, int64_t n, const long long* __restrict__ rows,
                                 const long long* __restrict__ cols, unsigned long long* __restrict__ v,
                                 int* __restrict__ bad) {
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < nnz;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const long long r = rows[e], c = cols[e];
    if (r < 0 || r >= m || c < 0 || c >= n) {
      atomicExch(bad, 1);
      continue;
    }
    atomicAdd(v + 1 + r, 1ull);
  }
}

__global__ void coo_scatter_kernel(int64_t nnz, int64_t m, int64_t n, const long long* __restrict__ rows,
                                   const long long* __restrict__ cols, unsigned long long* __restrict__ cursor,
                                   unsigned long long* __restrict__ keys) {
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < nnz;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const long long r = rows[e], c = cols[e];
    if (r < 0 || r >= m || c < 0 || c >= n) continue;
    const unsigned long long p = atomicAdd(cursor + r, 1ull);
    keys[p] = (static_cast<unsigned long long>(c) << 32) | static_cast<unsigned long long>(e);
  }
}

// entry of a sorted key: column and source index -> outputs
__device__ __forceinline__ void coo_emit(unsigned long long key, long long p, const uint8_t* __restrict__ vals_in,
                                         int esz, long long* __restrict__ cols_out, uint8_t* __restrict__ vals_out) {
  cols_out[p] = static_cast<long long>(key >> 32);
  const long long src = static_cast<long long>(key & 0xffffffffull);
  if (esz == 4)
    reinterpret_cast<uint32_t*>(vals_out)[p] = reinterpret_cast<const uint32_t*>(vals_in)[src];
  else if (esz == 2)
    reinterpret_cast<uint16_t*>(vals_out)[p] = reinterpret_cast<const uint16_t*>(vals_in)[src];
  else
    reinterpret_cast<uint64_t*>(vals_out)[p] = reinterpret_cast<const uint64_t*>(vals_in)[src];
}

// rows of at most 32 entries: a warp each, bitonic sort through shuffles
__global__ void coo_sort_short_kernel(int64_t m, const long long* __restrict__ row_ptr,
                                      const unsigned long long* __restrict__ keys, const uint8_t* __restrict__ vals_in,
                                      int esz, long long* __restrict__ cols_out, uint8_t* __restrict__ vals_out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m; r += warps) {
    const long long b0 = row_ptr[r], len = row_ptr[r + 1] - b0;
    if (len == 0 || len > 32) continue;
    unsigned long long k = lane < len ? keys[b0 + lane] : ~0ull;
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, stride);
        const bool up = (lane & size) == 0;          // ascending half of this bitonic stage
        const bool lower = (lane & stride) == 0;     // this lane keeps the smaller key when ascending
        const bool take_min = (up == lower);
        k = take_min ? (o < k ? o : k) : (o > k ? o : k);
      }
    }
    if (lane < len) coo_emit(k, b0 + lane, vals_in, esz, cols_out, vals_out);
  }
}

constexpr int kSortThreads = 256;
constexpr int kSortChunk = 2048;

// shared-memory bitonic sort of kSortChunk keys (ascending)
__device__ void smem_bitonic(unsigned long long* s) {
  for (int size = 2; size <= kSortChunk; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int t = threadIdx.x; t < kSortChunk / 2; t += blockDim.x) {
        const int lo = 2 * t - (t & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const unsigned long long a = s[lo], c = s[hi];
        if ((a > c) == up) {
          s[lo] = c;
          s[hi] = a;
        }
      }
    }
  }
  __syncthreads();
}

// number of keys in sorted [p, p + len) below x (keys are unique)
__device__ __forceinline__ long long lower_bound_u64(const unsigned long long* p, long long len, unsigned long long x) {
  long long lo = 0, hi = len;
  while (lo < hi) {
    const long long mid = (lo + hi) >> 1;
    if (p[mid] < x) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// rows of more than 32 entries: a CTA each (grid-stride over the rows)
__global__ void __launch_bounds__(kSortThreads) coo_sort_long_kernel(
    int64_t m, const long long* __restrict__ row_ptr, unsigned long long* __restrict__ keys,
    unsigned long long* __restrict__ keys2, const uint8_t* __restrict__ vals_in, int esz,
    long long* __restrict__ cols_out, uint8_t* __restrict__ vals_out) {
  __shared__ unsigned long long s[kSortChunk];
  for (int64_t r = blockIdx.x; r < m; r += gridDim.x) {
    const long long b0 = row_ptr[r], len = row_ptr[r + 1] - b0;
    if (len <= 32) continue;
    unsigned long long* src = keys + b0;
    unsigned long long* dst = keys2 + b0;
    // sort each chunk in shared memory
    for (long long c0 = 0; c0 < len; c0 += kSortChunk) {
      const long long cl = min((long long)kSortChunk, len - c0);
      __syncthreads();
      for (int t = threadIdx.x; t < kSortChunk; t += blockDim.x) s[t] = t < cl ? src[c0 + t] : ~0ull;
      smem_bitonic(s);
      for (int t = threadIdx.x; t < cl; t += blockDim.x) src[c0 + t] = s[t];
    }
    __syncthreads();
    // merge runs pairwise: an element's output index is its index in its own run plus
    // the number of keys of the partner run below it (keys are unique)
    for (long long run = kSortChunk; run < len; run <<= 1) {
      for (long long t = threadIdx.x; t < len; t += blockDim.x) {
        const long long pair0 = (t / (2 * run)) * (2 * run);
        const bool second = t - pair0 >= run;
        const long long own0 = second ? pair0 + run : pair0;
        const long long oth0 = second ? pair0 : pair0 + run;
        const long long oth_len = max(0ll, min(run, len - oth0));
        const long long rank = lower_bound_u64(src + oth0, oth_len, src[t]);
        dst[pair0 + (t - own0) + rank] = src[t];
      }
      __syncthreads();
      unsigned long long* tmp = src;
      src = dst;
      dst = tmp;
    }
    for (long long t = threadIdx.x; t < len; t += blockDim.x) coo_emit(src[t], b0 + t, vals_in, esz, cols_out, vals_out);
  }
}

int esize(int dtype) {
  switch (dtype) {
    case TRNSPARSE_F32: return 4;
    case TRNSPARSE_F64: return 8;
    case TRNSPARSE_BF16:
    case TRNSPARSE_F16: return 2;
    default: return 0;
  }
}

unsigned grid_for(int64_t items, int per_cta) {
  int64_t g = (items + per_cta - 1) / per_cta;
  const int64_t cap = 32ll * sm_count();
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace tsb

using namespace tsb;

// ---------------------------------------------------------------- BSR from dense
extern "C" size_t trnsparse_bsr_from_dense_workspace_size(int64_t m, int64_t n, int block_size) {
  if (m < 0 || n < 0 || block_size <= 0) return 0;
  const int64_t mb = (m + block_size - 1) / block_size, nbc = (n + block_size - 1) / block_size;
  return sizeof(long long) * (size_t)(mb * nbc + 1) + scan_ws_bytes(mb * nbc);
}

extern "C" int trnsparse_bsr_from_dense_count(int64_t m, int64_t n, const void* A, int64_t lda, int dtype,
                                              int block_size, float threshold, long long* block_row_ptr, void* ws,
                                              size_t ws_bytes, void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && block_size > 0 && lda >= n, "bsr_from_dense: bad sizes");
  TSB_REQUIRE(dtype == TRNSPARSE_F32 || dtype == TRNSPARSE_BF16, "bsr_from_dense: dtype must be F32 or BF16");
  TSB_REQUIRE(block_row_ptr && ws && (A || m * n == 0), "bsr_from_dense: null pointer");
  TSB_REQUIRE(ws_bytes >= trnsparse_bsr_from_dense_workspace_size(m, n, block_size), "bsr_from_dense: workspace too small");
  const int64_t mb = (m + block_size - 1) / block_size, nbc = (n + block_size - 1) / block_size;
  TSB_REQUIRE(mb < 65536 || nbc == 0, "bsr_from_dense: more than 65535 block-rows");
  TSB_REQUIRE(nbc < (1ll << 31), "bsr_from_dense: too many block columns");
  cudaStream_t st = as_stream(stream);
  long long* pos = static_cast<long long*>(ws);
  long long* part = pos + mb * nbc + 1;
  if (mb * nbc > 0) {
    dim3 g((unsigned)nbc, (unsigned)mb);
    if (dtype == TRNSPARSE_F32)
      bsr_screen_kernel<float><<<g, 256, 0, st>>>(m, n, (const float*)A, lda, block_size, threshold, nbc, pos);
    else
      bsr_screen_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(m, n, (const __nv_bfloat16*)A, lda, block_size, threshold,
                                                          nbc, pos);
    TSB_CHECK_LAUNCH("bsr_from_dense: screen");
  }
  int rc = exclusive_scan(pos, mb * nbc, part, st);
  if (rc) return rc;
  bsr_row_ptr_kernel<<<grid_for(mb + 1, 256), 256, 0, st>>>(mb, nbc, pos, block_row_ptr);
  TSB_CHECK_LAUNCH("bsr_from_dense: row pointers");
  return TRNSPARSE_OK;
}

extern "C" int trnsparse_bsr_from_dense_fill(int64_t m, int64_t n, const void* A, int64_t lda, int dtype,
                                             int block_size, void* blocks, long long* block_col_idx, const void* ws,
                                             void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && block_size > 0 && lda >= n, "bsr_from_dense: bad sizes");
  TSB_REQUIRE(dtype == TRNSPARSE_F32 || dtype == TRNSPARSE_BF16, "bsr_from_dense: dtype must be F32 or BF16");
  TSB_REQUIRE(ws, "bsr_from_dense: null workspace");
  const int64_t mb = (m + block_size - 1) / block_size, nbc = (n + block_size - 1) / block_size;
  if (mb * nbc == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(A && blocks && block_col_idx, "bsr_from_dense: null pointer");
  cudaStream_t st = as_stream(stream);
  const long long* pos = static_cast<const long long*>(ws);
  dim3 g((unsigned)nbc, (unsigned)mb);
  if (dtype == TRNSPARSE_F32)
    bsr_fill_kernel<float><<<g, 256, 0, st>>>(m, n, (const float*)A, lda, block_size, nbc, pos, (float*)blocks,
                                              block_col_idx);
  else
    bsr_fill_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(m, n, (const __nv_bfloat16*)A, lda, block_size, nbc, pos,
                                                      (__nv_bfloat16*)blocks, block_col_idx);
  TSB_CHECK_LAUNCH("bsr_from_dense: fill");
  return TRNSPARSE_OK;
}

// ---------------------------------------------------------------- CSR from dense
extern "C" size_t trnsparse_csr_from_dense_workspace_size(int64_t m) {
  return m < 0 ? 0 : scan_ws_bytes(m);
}

extern "C" int trnsparse_csr_from_dense_count(int64_t m, int64_t n, const void* A, int64_t lda, int dtype,
                                              float threshold, long long* row_ptr, void* ws, size_t ws_bytes,
                                              void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && lda >= n, "csr_from_dense: bad sizes");
  TSB_REQUIRE(dtype == TRNSPARSE_F32 || dtype == TRNSPARSE_BF16, "csr_from_dense: dtype must be F32 or BF16");
  TSB_REQUIRE(row_ptr && ws && (A || m * n == 0), "csr_from_dense: null pointer");
  TSB_REQUIRE(ws_bytes >= trnsparse_csr_from_dense_workspace_size(m), "csr_from_dense: workspace too small");
  cudaStream_t st = as_stream(stream);
  if (m > 0) {
    if (n == 0) {
      cudaError_t e = cudaMemsetAsync(row_ptr, 0, sizeof(long long) * (m + 1), st);
      return cuda_status(e, "csr_from_dense: empty rows");
    }
    if (dtype == TRNSPARSE_F32)
      csr_count_kernel<float><<<grid_for(m, 8), 256, 0, st>>>(m, n, (const float*)A, lda, threshold, row_ptr);
    else
      csr_count_kernel<__nv_bfloat16><<<grid_for(m, 8), 256, 0, st>>>(m, n, (const __nv_bfloat16*)A, lda, threshold,
                                                                    row_ptr);
    TSB_CHECK_LAUNCH("csr_from_dense: count");
  }
  return exclusive_scan(row_ptr, m, static_cast<long long*>(ws), st);
}

extern "C" int trnsparse_csr_from_dense_fill(int64_t m, int64_t n, const void* A, int64_t lda, int dtype,
                                             float threshold, const long long* row_ptr, void* values,
                                             long long* col_idx, void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && lda >= n, "csr_from_dense: bad sizes");
  TSB_REQUIRE(dtype == TRNSPARSE_F32 || dtype == TRNSPARSE_BF16, "csr_from_dense: dtype must be F32 or BF16");
  if (m == 0 || n == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(A && row_ptr && values && col_idx, "csr_from_dense: null pointer");
  cudaStream_t st = as_stream(stream);
  if (dtype == TRNSPARSE_F32)
    csr_fill_kernel<float><<<grid_for(m, 8), 256, 0, st>>>(m, n, (const float*)A, lda, threshold, row_ptr,
                                                          (float*)values, col_idx);
  else
    csr_fill_kernel<__nv_bfloat16><<<grid_for(m, 8), 256, 0, st>>>(m, n, (const __nv_bfloat16*)A, lda, threshold,
                                                                  row_ptr, (__nv_bfloat16*)values, col_idx);
  TSB_CHECK_LAUNCH("csr_from_dense: fill");
  return TRNSPARSE_OK;
}

// ---------------------------------------------------------------- COO -> CSR
extern "C" size_t trnsparse_coo_to_csr_workspace_size(int64_t m, int64_t nnz) {
  if (m < 0 || nnz < 0) return 0;
  return sizeof(unsigned long long) * (size_t)(2 * nnz + m + 1) + scan_ws_bytes(m) + 16;
}

extern "C" int trnsparse_coo_to_csr(int64_t m, int64_t n, int64_t nnz, const long long* rows, const long long* cols,
                                    const void* values, int dtype, long long* row_ptr, long long* cols_out,
                                    void* values_out, void* ws, size_t ws_bytes, void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && nnz >= 0, "coo_to_csr: bad sizes");
  TSB_REQUIRE(nnz < (1ll << 32) && n < (1ll << 31), "coo_to_csr: nnz must be < 2^32 and n < 2^31");
  const int esz = esize(dtype);
  TSB_REQUIRE(esz > 0, "coo_to_csr: unsupported dtype %d", dtype);
  TSB_REQUIRE(row_ptr && ws, "coo_to_csr: null pointer");
  TSB_REQUIRE(nnz == 0 || (rows && cols && values && cols_out && values_out), "coo_to_csr: null pointer");
  TSB_REQUIRE(ws_bytes >= trnsparse_coo_to_csr_workspace_size(m, nnz), "coo_to_csr: workspace too small");
  cudaStream_t st = as_stream(stream);
  unsigned long long* keys = static_cast<unsigned long long*>(ws);
  unsigned long long* keys2 = keys + nnz;
  unsigned long long* cursor = keys2 + nnz;  // m entries
  long long* part = reinterpret_cast<long long*>(cursor + m + 1);
  int* bad = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(part) + scan_ws_bytes(m));
  cudaError_t e = cudaMemsetAsync(row_ptr, 0, sizeof(long long) * (m + 1), st);
  if (e == cudaSuccess) e = cudaMemsetAsync(bad, 0, sizeof(int), st);
  if (e != cudaSuccess) return cuda_status(e, "coo_to_csr: clear");
  if (nnz > 0) {
    coo_count_kernel<<<grid_for(nnz, 256), 256, 0, st>>>(nnz, m, n, rows, cols,
                                                        reinterpret_cast<unsigned long long*>(row_ptr), bad);
    TSB_CHECK_LAUNCH("coo_to_csr: count");
  }
  int rc = exclusive_scan(row_ptr, m, part, st);
  if (rc) return rc;
  if (nnz == 0 || m == 0) return TRNSPARSE_OK;
  e = cudaMemcpyAsync(cursor, row_ptr, sizeof(long long) * m, cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return cuda_status(e, "coo_to_csr: cursors");
  coo_scatter_kernel<<<grid_for(nnz, 256), 256, 0, st>>>(nnz, m, n, rows, cols, cursor, keys);
  coo_sort_short_kernel<<<grid_for(m, 8), 256, 0, st>>>(m, row_ptr, keys, (const uint8_t*)values, esz, cols_out,
                                                       (uint8_t*)values_out);
  coo_sort_long_kernel<<<grid_for(m, 1), kSortThreads, 0, st>>>(m, row_ptr, keys, keys2, (const uint8_t*)values, esz,
                                                               cols_out, (uint8_t*)values_out);
  TSB_CHECK_LAUNCH("coo_to_csr: sort");
  // an out-of-range index is an argument error the caller sees on the host
  int hbad = 0;
  e = cudaMemcpyAsync(&hbad, bad, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_status(e, "coo_to_csr: status");
  TSB_REQUIRE(!hbad, "coo_to_csr: a row or column index is out of range");
  return TRNSPARSE_OK;
}
