// Device-side sparse format construction: the reference's host-side
// BSRMatrix.from_dense (trnsparse/formats.py:184-221), CSR from_dense
// (formats.py:269-278) and COOMatrix.to_csr (formats.py:104-124), with the
// same results bit for bit.
//
//   BSR from dense   a CTA per b x b block screens max |v| (a NaN
//                    in the block drops it, as torch.amax propagates NaN) and
//                    writes a 0/1 count; one exclusive scan over the block
//                    grid in row-major order gives every kept block its slot
//                    (the reference's nonzero() order) and the block-row
//                    pointers; a second pass copies the kept blocks, padded
//                    with zeros past the matrix edge.
//   CSR from dense   a warp per row counts |v| > threshold, a scan gives the
//                    row pointers, and a second pass compacts each row in
//                    column order (per-lane counts, a warp prefix sum).
// Dense rows are read in 16-byte pieces where the leading dimension and the
// base allow it.
//   COO -> CSR       row histogram (atomics) and scan, an atomic-cursor
//                    scatter of (col << 32 | entry index) keys into their row,
//                    then a sort of each row's keys: the entry index breaks
//                    ties, so the result is the stable (row, col) order of
//                    torch.argsort(rows * n + cols, stable=True). Rows of up to
//                    8 entries sort in one thread's registers, up to 32 in a warp
//                    (shuffle bitonic), longer ones in a CTA (shared-memory
//                    bitonic over 2048-key chunks, then merge passes through a
//                    second key buffer); the thread-per-row pass lists the others.
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
// VEC elements (16 bytes) per load when the rows allow it, else one
template <typename T, int VEC> struct Vec;
template <typename T> struct Vec<T, 1> {
  T v[1];
};
template <> struct alignas(16) Vec<float, 4> {
  float v[4];
};
template <> struct alignas(16) Vec<__nv_bfloat16, 8> {
  __nv_bfloat16 v[8];
};

// Warp w of the CTA walks rows w, w + 8, ... of the block; lanes cover the row in VEC-wide
// pieces. f(piece, k, valid) sees every element of the block that lies inside the matrix.
template <typename T, int VEC, typename F>
__device__ __forceinline__ void for_block_rows(int64_t m, int64_t n, const T* __restrict__ A, int64_t lda, int b,
                                               int64_t r0, int64_t c0, F&& f) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
  for (int r = warp; r < b; r += warps) {
    const int64_t gr = r0 + r;
    if (gr >= m) break;
    const T* row = A + gr * lda + c0;
    for (int c = lane * VEC; c < b; c += 32 * VEC) {
      if (c0 + c + VEC <= n) {
        f(r, c, *reinterpret_cast<const Vec<T, VEC>*>(row + c), VEC);
      } else {
        Vec<T, VEC> x;
        int cnt = 0;
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
          x.v[k] = T(0.f);
          if (c0 + c + k < n) {
            x.v[k] = row[c + k];
            cnt = k + 1;
          }
        }
        f(r, c, x, cnt);
      }
    }
  }
}

// grid (block column, block row); writes pos[1 + i * nbc + j] = keep ? 1 : 0
template <typename T, int VEC>
__global__ void __launch_bounds__(256) bsr_screen_kernel(int64_t m, int64_t n, const T* __restrict__ A, int64_t lda,
                                                         int b, float thr, int64_t nbc, long long* __restrict__ pos) {
  __shared__ float smax[8];
  __shared__ int snan[8];
  const int64_t j = blockIdx.x, i = blockIdx.y;
  float mx = 0.f;
  int nan = 0;
  for_block_rows<T, VEC>(m, n, A, lda, b, i * b, j * b, [&](int, int, const Vec<T, VEC>& x, int cnt) {
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      if (k < cnt) {
        const float a = fm_abs<T>(x.v[k]);
        nan |= a != a;
        mx = fmaxf(mx, a);
      }
    }
  });
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
    // padding zeros take part in the max (it starts at 0), as in the reference's padded grid
    pos[1 + i * nbc + j] = (!nan && mx > thr) ? 1 : 0;
  }
}

__global__ void bsr_row_ptr_kernel(int64_t mb, int64_t nbc, const long long* __restrict__ pos,
                                   long long* __restrict__ row_ptr) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i <= mb;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    row_ptr[i] = pos[i * nbc];
}

// grid (block column, block row): copy a kept block to its slot, zeros past the matrix edge
template <typename T, int VEC>
__global__ void __launch_bounds__(256) bsr_fill_kernel(int64_t m, int64_t n, const T* __restrict__ A, int64_t lda,
                                                       int b, int64_t nbc, const long long* __restrict__ pos,
                                                       T* __restrict__ blocks, long long* __restrict__ col_idx) {
  const int64_t j = blockIdx.x, i = blockIdx.y;
  const int64_t k = i * nbc + j;
  const long long slot = pos[k];
  if (pos[k + 1] == slot) return;  // dropped
  if (threadIdx.x == 0) col_idx[slot] = j;
  T* dst = blocks + slot * static_cast<int64_t>(b) * b;
  const bool ragged = (i + 1) * b > m || (j + 1) * b > n;
  if (ragged) {  // clear first: rows past the edge are skipped below
    for (int e = threadIdx.x; e < b * b; e += blockDim.x) dst[e] = T(0.f);
    __syncthreads();
  }
  for_block_rows<T, VEC>(m, n, A, lda, b, i * b, j * b, [&](int r, int c, const Vec<T, VEC>& x, int cnt) {
    if (cnt == VEC) {
      *reinterpret_cast<Vec<T, VEC>*>(dst + r * b + c) = x;
    } else {
#pragma unroll
      for (int q = 0; q < VEC; ++q)
        if (q < cnt) dst[r * b + c + q] = x.v[q];
    }
  });
}

// ---------------------------------------------------------------- CSR from dense
// a warp per row; lane l covers elements [j0 + VEC l, j0 + VEC l + VEC) of each 32 VEC piece
template <typename T, int VEC>
__device__ __forceinline__ Vec<T, VEC> load_piece(const T* row, int64_t j, int64_t n, int& cnt) {
  Vec<T, VEC> x;
  if (j + VEC <= n) {
    x = *reinterpret_cast<const Vec<T, VEC>*>(row + j);
    cnt = VEC;
  } else {
    cnt = 0;
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      x.v[k] = T(0.f);
      if (j + k < n) {
        x.v[k] = row[j + k];
        cnt = k + 1;
      }
    }
  }
  return x;
}

template <typename T, int VEC>
__global__ void csr_count_kernel(int64_t m, int64_t n, const T* __restrict__ A, int64_t lda, float thr,
                                 long long* __restrict__ v) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m; r += warps) {
    const T* row = A + r * lda;
    long long c = 0;
#pragma unroll 4
    for (int64_t j = lane * VEC; j < n; j += 32 * VEC) {
      int cnt;
      const Vec<T, VEC> x = load_piece<T, VEC>(row, j, n, cnt);
#pragma unroll
      for (int k = 0; k < VEC; ++k) c += (k < cnt && fm_abs<T>(x.v[k]) > thr) ? 1 : 0;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == 0) v[1 + r] = c;
  }
}

// The count pass that also writes a bit mask of the kept entries (bit c % 32 of word
// r * mw + c / 32 for entry (r, c)), so a fill can gather the kept values instead of
// reading the rows again. All lanes walk every piece together (the mask words are
// assembled across lanes).
template <typename T, int VEC>
__global__ void csr_count_mask_kernel(int64_t m, int64_t n, const T* __restrict__ A, int64_t lda, float thr,
                                      long long* __restrict__ v, uint32_t* __restrict__ mask, int64_t mw) {
  constexpr int L = 32 / VEC;  // lanes per 32-bit mask word
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m; r += warps) {
    const T* row = A + r * lda;
    uint32_t* mrow = mask + r * mw;
    long long c = 0;
    constexpr int kU = 4;  // pieces per batch: their loads are all in flight before any shuffle
    for (int64_t jb = 0; jb < n; jb += kU * 32 * VEC) {
      Vec<T, VEC> x[kU];
      int cnt[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t j = jb + u * 32 * VEC + lane * VEC;
        cnt[u] = 0;
        if (j < n) x[u] = load_piece<T, VEC>(row, j, n, cnt[u]);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t j0 = jb + u * 32 * VEC;
        if (j0 >= n) break;  // uniform across the warp
        unsigned bits = 0;
#pragma unroll
        for (int k = 0; k < VEC; ++k)
          if (k < cnt[u] && fm_abs<T>(x[u].v[k]) > thr) bits |= 1u << k;
        c += __popc(bits);
        unsigned word;
        if constexpr (VEC == 1) {
          word = __ballot_sync(0xffffffffu, bits != 0);
        } else {
          word = bits << ((lane % L) * VEC);
#pragma unroll
          for (int o = 1; o < L; o <<= 1) word |= __shfl_xor_sync(0xffffffffu, word, o);
        }
        const int64_t widx = j0 / 32 + lane / L;
        if (lane % L == 0 && widx < mw) mrow[widx] = word;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (lane == 0) v[1 + r] = c;
  }
}

// Fill from the mask: a warp per row, lane l takes mask word w0 + l, a warp prefix sum of
// the words' bit counts gives each lane its output offset, and the lane gathers its kept
// entries in column order.
template <typename T>
__global__ void csr_fill_masked_kernel(int64_t m, int64_t n, const T* __restrict__ A, int64_t lda,
                                       const long long* __restrict__ row_ptr, const uint32_t* __restrict__ mask,
                                       int64_t mw, T* __restrict__ vals, long long* __restrict__ cols) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m; r += warps) {
    const T* row = A + r * lda;
    const uint32_t* mrow = mask + r * mw;
    long long o = row_ptr[r];
    for (int64_t w0 = 0; w0 < mw; w0 += 32) {
      const int64_t w = w0 + lane;
      unsigned bits = w < mw ? mrow[w] : 0u;
      const int mine = __popc(bits);
      int inc = mine;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, d);
        if (lane >= d) inc += y;
      }
      long long p = o + inc - mine;
      while (bits) {
        const int b = __ffs(bits) - 1;
        bits &= bits - 1;
        const int64_t col = w * 32 + b;
        vals[p] = row[col];
        cols[p] = col;
        ++p;
      }
      o += __shfl_sync(0xffffffffu, inc, 31);
    }
  }
}

template <typename T, int VEC>
__global__ void csr_fill_kernel(int64_t m, int64_t n, const T* __restrict__ A, int64_t lda, float thr,
                                const long long* __restrict__ row_ptr, T* __restrict__ vals,
                                long long* __restrict__ cols) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m; r += warps) {
    const T* row = A + r * lda;
    long long o = row_ptr[r];
    for (int64_t j0 = 0; j0 < n; j0 += 32 * VEC) {
      const int64_t j = j0 + lane * VEC;
      int cnt = 0;
      Vec<T, VEC> x;
      if (j < n) x = load_piece<T, VEC>(row, j, n, cnt);
      unsigned keep = 0;
#pragma unroll
      for (int k = 0; k < VEC; ++k)
        if (k < cnt && fm_abs<T>(x.v[k]) > thr) keep |= 1u << k;
      if (!__any_sync(0xffffffffu, keep != 0)) continue;  // nothing kept in this piece of the row
      // exclusive prefix of the kept counts over the lanes: entries stay in column order
      const int mine = __popc(keep);
      int inc = mine;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, d);
        if (lane >= d) inc += y;
      }
      long long p = o + inc - mine;
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        if (keep & (1u << k)) {
          vals[p] = x.v[k];
          cols[p] = j + k;
          ++p;
        }
      }
      o += __shfl_sync(0xffffffffu, inc, 31);
    }
  }
}

// ---------------------------------------------------------------- COO -> CSR
// skip_negative: a row index of -1 marks an entry left out (the strict-triangle transpose)
__global__ void coo_count_kernel(int64_t nnz, int64_t m, int64_t n, const long long* __restrict__ rows,
                                 const long long* __restrict__ cols, unsigned long long* __restrict__ v,
                                 int* __restrict__ bad, int skip_negative = 0) {
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < nnz;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const long long r = rows[e], c = cols[e];
    if (skip_negative && r < 0) continue;
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
  // four entries per thread and sweep: four cursor atomics in flight at once
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t e0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e0 < nnz; e0 += 4 * stride) {
    long long r[4], c[4];
    unsigned long long p[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t e = e0 + u * stride;
      r[u] = -1;
      if (e < nnz) {
        r[u] = rows[e];
        c[u] = cols[e];
        if (r[u] >= m || c[u] < 0 || c[u] >= n) r[u] = -1;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (r[u] >= 0) p[u] = atomicAdd(cursor + r[u], 1ull);
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (r[u] >= 0)
        keys[p[u]] = (static_cast<unsigned long long>(c[u]) << 32) | static_cast<unsigned long long>(e0 + u * stride);
  }
}

// COO -> CSR for up to kBucketRows * kMaxBuckets rows, in buckets of kBucketRows
// consecutive rows, with no per-entry global atomic (a radix-partition scheme):
//   count      CTA c counts its chunk of entries per bucket in shared memory (and
//              flags out-of-range indices) and writes the counts to column c of a
//              bucket-major count matrix
//   scan       one exclusive scan of that matrix gives every (bucket, CTA) pair its
//              offset; bucket b's region starts at the offset of (b, 0)
//   partition  CTA c sorts its chunk by bucket in shared memory (counting sort,
//              ranks from shared-memory atomics) and writes it out bucket by bucket,
//              so each bucket receives one contiguous run per CTA: (row within the
//              bucket, col << 32 | entry index, value)
//   bucket     a CTA per bucket, all in shared memory: row histogram and scan (the
//              row pointers), the entries of rows of up to kTiny entries placed by
//              row, each such row sorted by key in one thread's registers with its
//              values, and the sorted bucket written out in order; entries of longer
//              rows go to their row's place in a key buffer for the warp / CTA sorts
// Entry order inside a row is arbitrary before the per-row sort of the
// (col << 32 | entry index) keys, which gives the stable (row, col) order.
#ifndef TSB_COO_BUCKET_ROWS
#define TSB_COO_BUCKET_ROWS 2048
#endif
#ifndef TSB_COO_BUCKET_KB
#define TSB_COO_BUCKET_KB 200
#endif
constexpr int kBucketRows = TSB_COO_BUCKET_ROWS;
constexpr int kMaxBuckets = 4096;              // rows up to 2^23 take this path
#ifndef TSB_COO_PART_CHUNK
#define TSB_COO_PART_CHUNK 8192
#endif
#ifndef TSB_COO_PART_THREADS
#define TSB_COO_PART_THREADS 1024
#endif
constexpr int kPartChunk = TSB_COO_PART_CHUNK;  // entries per CTA in the count / partition passes
constexpr int64_t kMaxCountCells = 1ll << 24;  // cells of the count matrix (the chunk grows past it)
constexpr int kTiny = 8;                       // rows of up to kTiny entries sort in one thread's registers
constexpr int kPartThreads = TSB_COO_PART_THREADS;
#ifndef TSB_COO_BUCKET_THREADS
#define TSB_COO_BUCKET_THREADS 1024
#endif
constexpr int kBucketThreads = TSB_COO_BUCKET_THREADS;
constexpr int kMaxSub = 64;  // sub-ranges per bucket: kBucketRows * kTiny / (cap - kTiny) at most

__host__ __device__ inline int64_t coo_chunk(int64_t nnz, int nb) {
  const int64_t per = kMaxCountCells / nb;  // CTAs the matrix can hold
  const int64_t c = (nnz + per - 1) / per;
  return c > kPartChunk ? c : kPartChunk;
}

__device__ __forceinline__ bool coo_ok(long long r, long long c, int64_t m, int64_t n) {
  return r >= 0 && r < m && c >= 0 && c < n;
}

// value payload carried through the partition (ESZ 0: none; the emitted "value" is the
// entry index, which the key holds)
template <int ESZ> struct CooVal { using type = unsigned long long; };
template <> struct CooVal<4> { using type = uint32_t; };
template <> struct CooVal<2> { using type = uint16_t; };
template <> struct CooVal<0> { using type = uint8_t; };

__global__ void __launch_bounds__(256) coo_bucket_count_kernel(int64_t nnz, int64_t m, int64_t n, int nb,
                                                               int64_t chunk, const long long* __restrict__ rows,
                                                               const long long* __restrict__ cols,
                                                               long long* __restrict__ cm, int* __restrict__ bad) {
  __shared__ int cnt[kMaxBuckets];
  const int64_t G = gridDim.x, c = blockIdx.x;
  const int64_t c0 = c * chunk, c1 = c0 + chunk < nnz ? c0 + chunk : nnz;
  for (int b = threadIdx.x; b < nb; b += blockDim.x) cnt[b] = 0;
  __syncthreads();
  int flag = 0;
  for (int64_t e0 = c0 + threadIdx.x; e0 < c1; e0 += 4 * blockDim.x) {
    long long r[4], k[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t e = e0 + u * blockDim.x;
      r[u] = e < c1 ? rows[e] : 0;
      k[u] = e < c1 ? cols[e] : 0;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (e0 + u * blockDim.x >= c1) continue;
      if (coo_ok(r[u], k[u], m, n)) atomicAdd(&cnt[r[u] / kBucketRows], 1);
      else flag = 1;
    }
  }
  if (flag) atomicExch(bad, 1);
  __syncthreads();
  for (int b = threadIdx.x; b < nb; b += blockDim.x) cm[1 + b * G + c] = cnt[b];
}

// Exclusive scan of n <= per * blockDim.x ints in place (per consecutive values a thread).
template <int PER>
__device__ __forceinline__ void block_excl_scan_ints(unsigned* v, int n, long long* warp_tot) {
  unsigned loc[PER], t = 0;
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int i = threadIdx.x * PER + q;
    loc[q] = i < n ? v[i] : 0u;
    t += loc[q];
  }
  const long long inc = block_scan_incl(t, warp_tot, nullptr);
  unsigned off = static_cast<unsigned>(inc) - t;
#pragma unroll
  for (int q = 0; q < PER; ++q) {
    const int i = threadIdx.x * PER + q;
    if (i < n) v[i] = off;
    off += loc[q];
  }
}

__host__ __device__ inline int coo_nb_pad(int nb) { return (nb + 3) & ~3; }
size_t coo_partition_smem(int esz, int nb) {
  return 4 * sizeof(unsigned) * coo_nb_pad(nb) +
         static_cast<size_t>(kPartChunk) * (sizeof(unsigned long long) + (esz ? esz : 1) + 2 * sizeof(uint16_t));
}

// The CTA's chunk in sub-tiles of kPartChunk entries, kPartPer per thread held in
// registers (all loads of a thread in flight together): count per bucket, scan, place
// each entry at its bucket's place in shared memory, then write the sub-tile out in
// bucket order (each bucket's entries continue where the previous sub-tile's stopped).
template <int ESZ>
__global__ void __launch_bounds__(kPartThreads) coo_partition_kernel(
    int64_t nnz, int64_t m, int64_t n, int nb, int64_t chunk, const long long* __restrict__ rows,
    const long long* __restrict__ cols, const void* __restrict__ vals, const long long* __restrict__ cm,
    uint16_t* __restrict__ plrow, unsigned long long* __restrict__ pkey, void* __restrict__ pval) {
  using V = typename CooVal<ESZ>::type;
  constexpr int kPer = kPartChunk / kPartThreads;
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ long long warp_tot[32];
  const int nbp = coo_nb_pad(nb);
  unsigned* cnt = reinterpret_cast<unsigned*>(sm);  // per bucket: count in this sub-tile
  unsigned* lst = cnt + nbp;                        // its start in the staged sub-tile
  unsigned* cur = lst + nbp;                        // placement cursor
  unsigned* gb = cur + nbp;                         // next output position (nnz < 2^32)
  unsigned long long* skey = reinterpret_cast<unsigned long long*>(gb + nbp);
  uint16_t* slr = reinterpret_cast<uint16_t*>(skey + kPartChunk);
  uint16_t* sbk = slr + kPartChunk;
  V* sval = reinterpret_cast<V*>(sbk + kPartChunk);
  const V* vin = static_cast<const V*>(vals);
  V* vout = static_cast<V*>(pval);
  const int64_t G = gridDim.x, c = blockIdx.x;
  const int64_t c0 = c * chunk, c1 = c0 + chunk < nnz ? c0 + chunk : nnz;
  for (int b = threadIdx.x; b < nb; b += blockDim.x) gb[b] = static_cast<unsigned>(cm[b * G + c]);
  for (int64_t t0 = c0; t0 < c1; t0 += kPartChunk) {
    long long r[kPer], k[kPer];
    V v[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int64_t e = t0 + threadIdx.x + u * kPartThreads;
      r[u] = e < c1 ? rows[e] : -1;
      k[u] = e < c1 ? cols[e] : -1;
      if constexpr (ESZ > 0) v[u] = e < c1 ? vin[e] : V(0);
    }
    __syncthreads();
    for (int b = threadIdx.x; b < nb; b += blockDim.x) {
      cnt[b] = 0;
      cur[b] = 0;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < kPer; ++u)
      if (coo_ok(r[u], k[u], m, n)) atomicAdd(&cnt[r[u] / kBucketRows], 1u);
    __syncthreads();
    for (int b = threadIdx.x; b < nb; b += blockDim.x) lst[b] = cnt[b];
    __syncthreads();
    block_excl_scan_ints<(kMaxBuckets + kPartThreads - 1) / kPartThreads>(lst, nb, warp_tot);
    __syncthreads();
    const int np = static_cast<int>(lst[nb - 1] + cnt[nb - 1]);
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      if (!coo_ok(r[u], k[u], m, n)) continue;
      const int b = static_cast<int>(r[u] / kBucketRows);
      const unsigned slot = lst[b] + atomicAdd(&cur[b], 1u);
      skey[slot] = (static_cast<unsigned long long>(k[u]) << 32) |
                   static_cast<unsigned long long>(t0 + threadIdx.x + u * kPartThreads);
      slr[slot] = static_cast<uint16_t>(r[u] - static_cast<long long>(b) * kBucketRows);
      sbk[slot] = static_cast<uint16_t>(b);
      if constexpr (ESZ > 0) sval[slot] = v[u];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < np; i += blockDim.x) {
      const int b = sbk[i];
      const size_t pos = static_cast<size_t>(gb[b]) + (i - lst[b]);
      plrow[pos] = slr[i];
      pkey[pos] = skey[i];
      if constexpr (ESZ > 0) vout[pos] = sval[i];
    }
    __syncthreads();
    for (int b = threadIdx.x; b < nb; b += blockDim.x) gb[b] += cnt[b];
  }
}

size_t coo_bucket_smem_fixed() { return 5 * sizeof(int) * kBucketRows; }
int coo_bucket_entry_bytes(int esz) {
  return static_cast<int>(sizeof(unsigned long long) + sizeof(uint16_t) + (esz ? esz : 1));
}

// A CTA per bucket (persistent over buckets). cap: entries the staging area holds.
// Rows of up to kTiny entries are staged by row (in sub-ranges of at most cap - kTiny
// entries when the bucket's short rows hold more than that), sorted in registers,
// written back in place and then copied out in order; longer rows go to `keys` at
// their row's place and are listed for the warp / CTA sorts.
template <int ESZ>
__global__ void __launch_bounds__(kBucketThreads) coo_bucket_sort_kernel(
    int64_t m, int nb, int64_t G, int cap, const long long* __restrict__ cm, const uint16_t* __restrict__ plrow,
    const unsigned long long* __restrict__ pkey, const void* __restrict__ pval, long long* __restrict__ row_ptr,
    unsigned long long* __restrict__ keys, long long* __restrict__ cols_out, void* __restrict__ vals_out,
    long long* __restrict__ mid_rows, unsigned long long* __restrict__ n_mid, long long* __restrict__ long_rows,
    unsigned long long* __restrict__ n_long) {
  using V = typename CooVal<ESZ>::type;
  constexpr int kPer = kBucketRows / kBucketThreads;
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ long long warp_tot[32];
  __shared__ long long tiny_total;
  __shared__ int bnd[kMaxSub + 1];
  int* cnt = reinterpret_cast<int*>(sm);  // entries per row
  int* rst = cnt + kBucketRows;           // row start in the bucket (all rows)
  int* tst = rst + kBucketRows;           // start among the short rows' entries
  int* curT = tst + kBucketRows;
  int* curL = curT + kBucketRows;
  unsigned long long* skey = reinterpret_cast<unsigned long long*>(curL + kBucketRows);
  uint16_t* srow = reinterpret_cast<uint16_t*>(skey + cap);
  V* sval = reinterpret_cast<V*>(srow + cap);
  const V* vin = static_cast<const V*>(pval);
  const int capE = cap - kTiny;
  for (int b = blockIdx.x; b < nb; b += gridDim.x) {
    const int64_t r0 = static_cast<int64_t>(b) * kBucketRows;
    const int nr = static_cast<int>(m - r0 < kBucketRows ? m - r0 : kBucketRows);
    const long long s = cm[b * G], e = cm[(b + 1) * G];
    const int len = static_cast<int>(e - s);
    __syncthreads();
    for (int i = threadIdx.x; i < kBucketRows; i += blockDim.x) {
      cnt[i] = 0;
      curT[i] = 0;
      curL[i] = 0;
    }
    __syncthreads();
    for (int i0 = threadIdx.x; i0 < len; i0 += 4 * kBucketThreads) {
      int lr[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) lr[u] = i0 + u * kBucketThreads < len ? plrow[s + i0 + u * kBucketThreads] : -1;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (lr[u] >= 0) atomicAdd(&cnt[lr[u]], 1);
    }
    __syncthreads();
    // row starts (all rows) and starts among the short rows' entries
    int cv[kPer], ta = 0, tt = 0;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      cv[q] = cnt[threadIdx.x * kPer + q];
      ta += cv[q];
      tt += cv[q] <= kTiny ? cv[q] : 0;
    }
    const long long ia = block_scan_incl(ta, warp_tot, nullptr);
    __syncthreads();  // warp_tot is reused
    long long tt_total = 0;
    const long long it = block_scan_incl(tt, warp_tot, &tt_total);
    int oa = static_cast<int>(ia) - ta, ot = static_cast<int>(it) - tt;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int i = threadIdx.x * kPer + q;
      rst[i] = oa;
      tst[i] = ot;
      if (i < nr) {
        row_ptr[r0 + i] = s + oa;
        if (cv[q] > 32) long_rows[atomicAdd(n_long, 1ull)] = r0 + i;
        else if (cv[q] > kTiny) mid_rows[atomicAdd(n_mid, 1ull)] = r0 + i;
      }
      oa += cv[q];
      ot += cv[q] <= kTiny ? cv[q] : 0;
    }
    if (threadIdx.x == 0) tiny_total = tt_total;
    if (r0 + nr == m && threadIdx.x == 0) row_ptr[m] = e;
    __syncthreads();
    const int T = static_cast<int>(tiny_total);
    const int nsub = T > 0 ? (T + capE - 1) / capE : 1;
    auto sub_of = [&](int t) { return nsub == 1 ? 0 : t / capE; };
    // bnd[k]: the start (among the short rows' entries) of sub-range k's first row; every
    // window of capE >= kTiny entries holds a row start, so no sub-range is empty
    for (int k = threadIdx.x; k <= nsub; k += blockDim.x) bnd[k] = T;
    __syncthreads();
    for (int r = threadIdx.x; r < nr; r += blockDim.x)
      if (cnt[r] > 0 && cnt[r] <= kTiny) atomicMin(&bnd[sub_of(tst[r])], tst[r]);
    __syncthreads();
    for (int k = 0; k < nsub; ++k) {
      const int sb = k * capE;
      for (int i0 = threadIdx.x; i0 < len; i0 += 4 * kBucketThreads) {
        int lr[4];
        unsigned long long kk[4];
        V vv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = i0 + u * kBucketThreads;
          lr[u] = i < len ? plrow[s + i] : -1;
          kk[u] = i < len ? pkey[s + i] : 0ull;
          if constexpr (ESZ > 0) vv[u] = i < len ? vin[s + i] : V(0);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (lr[u] < 0) continue;
          const int cn = cnt[lr[u]];
          if (cn <= kTiny) {
            if (sub_of(tst[lr[u]]) != k) continue;
            const int slot = tst[lr[u]] - sb + atomicAdd(&curT[lr[u]], 1);
            skey[slot] = kk[u];
            srow[slot] = static_cast<uint16_t>(lr[u]);
            if constexpr (ESZ > 0) sval[slot] = vv[u];
          } else if (k == 0) {
            keys[s + rst[lr[u]] + atomicAdd(&curL[lr[u]], 1)] = kk[u];
          }
        }
      }
      __syncthreads();
      // sort each short row of this sub-range in registers (values follow their keys)
      for (int r = threadIdx.x; r < nr; r += blockDim.x) {
        const int cn = cnt[r];
        if (cn == 0 || cn > kTiny || sub_of(tst[r]) != k) continue;
        const int base = tst[r] - sb;
        unsigned long long kk[kTiny];
        V vv[kTiny];
#pragma unroll
        for (int i = 0; i < kTiny; ++i) {
          kk[i] = i < cn ? skey[base + i] : ~0ull;
          if constexpr (ESZ > 0) vv[i] = i < cn ? sval[base + i] : V(0);
        }
#pragma unroll
        for (int i = 0; i < kTiny - 1; ++i) {
#pragma unroll
          for (int j = 0; j < kTiny - 1 - i; ++j) {
            const bool sw = kk[j + 1] < kk[j];
            const unsigned long long a = kk[j], c2 = kk[j + 1];
            kk[j] = sw ? c2 : a;
            kk[j + 1] = sw ? a : c2;
            if constexpr (ESZ > 0) {
              const V va = vv[j], vc = vv[j + 1];
              vv[j] = sw ? vc : va;
              vv[j + 1] = sw ? va : vc;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < kTiny; ++i) {
          if (i < cn) {
            skey[base + i] = kk[i];
            if constexpr (ESZ > 0) sval[base + i] = vv[i];
          }
        }
      }
      __syncthreads();
      // copy the sorted sub-range out in order: its staged slots are contiguous, from its
      // first row's start to the next sub-range's first row's start
      const int lo = bnd[k] - sb, hi = bnd[k + 1] - sb;
      for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const int r = srow[i];
        const long long out = s + rst[r] + (i - (tst[r] - sb));
        const unsigned long long key = skey[i];
        cols_out[out] = static_cast<long long>(key >> 32);
        if constexpr (ESZ > 0)
          static_cast<V*>(vals_out)[out] = sval[i];
        else
          static_cast<long long*>(vals_out)[out] = static_cast<long long>(key & 0xffffffffull);
      }
      __syncthreads();
    }
  }
}

// entry of a sorted key: column and source index -> outputs
__device__ __forceinline__ void coo_emit(unsigned long long key, long long p, const uint8_t* __restrict__ vals_in,
                                         int esz, long long* __restrict__ cols_out, uint8_t* __restrict__ vals_out) {
  cols_out[p] = static_cast<long long>(key >> 32);
  const long long src = static_cast<long long>(key & 0xffffffffull);
  if (vals_in == nullptr)  // no values: emit the source entry index (a permutation)
    reinterpret_cast<long long*>(vals_out)[p] = src;
  else if (esz == 4)
    reinterpret_cast<uint32_t*>(vals_out)[p] = reinterpret_cast<const uint32_t*>(vals_in)[src];
  else if (esz == 2)
    reinterpret_cast<uint16_t*>(vals_out)[p] = reinterpret_cast<const uint16_t*>(vals_in)[src];
  else
    reinterpret_cast<uint64_t*>(vals_out)[p] = reinterpret_cast<const uint64_t*>(vals_in)[src];
}

// A thread per row: rows of at most kTiny entries are sorted in registers (an unrolled
// exchange network); longer rows are listed for the warp (<= 32) or CTA passes.
__global__ void coo_sort_tiny_kernel(int64_t m, const long long* __restrict__ row_ptr,
                                     const unsigned long long* __restrict__ keys, const uint8_t* __restrict__ vals_in,
                                     int esz, long long* __restrict__ cols_out, uint8_t* __restrict__ vals_out,
                                     long long* __restrict__ mid_rows, unsigned long long* __restrict__ n_mid,
                                     long long* __restrict__ long_rows, unsigned long long* __restrict__ n_long) {
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; r < m;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const long long b0 = row_ptr[r], len = row_ptr[r + 1] - b0;
    if (len > 32) {
      long_rows[atomicAdd(n_long, 1ull)] = r;
      continue;
    }
    if (len > kTiny) {
      mid_rows[atomicAdd(n_mid, 1ull)] = r;
      continue;
    }
    unsigned long long k[kTiny];
#pragma unroll
    for (int i = 0; i < kTiny; ++i) k[i] = i < len ? keys[b0 + i] : ~0ull;
#pragma unroll
    for (int i = 0; i < kTiny - 1; ++i) {
#pragma unroll
      for (int j = 0; j < kTiny - 1 - i; ++j) {
        const unsigned long long a = k[j], c = k[j + 1];
        k[j] = a < c ? a : c;
        k[j + 1] = a < c ? c : a;
      }
    }
#pragma unroll
    for (int i = 0; i < kTiny; ++i)
      if (i < len) coo_emit(k[i], b0 + i, vals_in, esz, cols_out, vals_out);
  }
}

// A warp per listed row of kTiny < len <= 32 entries: bitonic sort through shuffles.
__global__ void coo_sort_mid_kernel(const long long* __restrict__ row_ptr, const long long* __restrict__ mid_rows,
                                    const unsigned long long* __restrict__ n_mid,
                                    const unsigned long long* __restrict__ keys, const uint8_t* __restrict__ vals_in,
                                    int esz, long long* __restrict__ cols_out, uint8_t* __restrict__ vals_out) {
  const int lane = threadIdx.x & 31;
  const long long n_rows = static_cast<long long>(*n_mid);
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long q = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); q < n_rows;
       q += warps) {
    const long long r = mid_rows[q];
    const long long b0 = row_ptr[r], len = row_ptr[r + 1] - b0;
    unsigned long long k = lane < len ? keys[b0 + lane] : ~0ull;
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, stride);
        const bool up = (lane & size) == 0;        // ascending half of this bitonic stage
        const bool lower = (lane & stride) == 0;   // this lane keeps the smaller key when ascending
        k = (up == lower) ? (o < k ? o : k) : (o > k ? o : k);
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

// rows of more than 32 entries (listed by the tiny pass): a CTA each
__global__ void __launch_bounds__(kSortThreads) coo_sort_long_kernel(
    const long long* __restrict__ row_ptr, const long long* __restrict__ long_rows,
    const unsigned long long* __restrict__ n_long, unsigned long long* __restrict__ keys,
    unsigned long long* __restrict__ keys2, const uint8_t* __restrict__ vals_in, int esz,
    long long* __restrict__ cols_out, uint8_t* __restrict__ vals_out) {
  __shared__ unsigned long long s[kSortChunk];
  const long long n_rows = static_cast<long long>(*n_long);
  for (long long q = blockIdx.x; q < n_rows; q += gridDim.x) {
    const long long r = long_rows[q];
    const long long b0 = row_ptr[r], len = row_ptr[r + 1] - b0;
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

// CSR transpose, step 1: every entry's transposed coordinates (row = its column,
// column = its row; row -1 for a diagonal entry when only the strict triangle is kept).
// A warp per row.
template <typename I>
__global__ void csr_entry_coords_kernel(int64_t m, const I* __restrict__ row_ptr, const I* __restrict__ col_idx,
                                        int strict, long long* __restrict__ trow, long long* __restrict__ tcol) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m; r += warps) {
    const int64_t e0 = static_cast<int64_t>(row_ptr[r]), e1 = static_cast<int64_t>(row_ptr[r + 1]);
    for (int64_t e = e0 + lane; e < e1; e += 32) {
      const long long c = static_cast<long long>(col_idx[e]);
      trow[e] = (strict && c == r) ? -1 : c;
      tcol[e] = r;
    }
  }
}

// dst[p] = src[idx[p]] for elements of 2, 4 or 8 bytes
template <typename T>
__global__ void gather_kernel(int64_t count, const T* __restrict__ src, const long long* __restrict__ idx,
                              T* __restrict__ dst) {
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < count;
       p += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[p] = src[idx[p]];
}

// dst block p = (src block idx[p])^T for b x b blocks, through 32 x 33 shared-memory tiles:
// a CTA per (block, 32 x 32 tile), coalesced reads and writes.
template <typename T>
__global__ void block_transpose_gather_kernel(int b, const T* __restrict__ src, const long long* __restrict__ idx,
                                              T* __restrict__ dst) {
  __shared__ T tile[32][33];
  const int tiles = (b + 31) / 32;
  const int64_t p = blockIdx.y;
  const int ti = blockIdx.x / tiles, tj = blockIdx.x % tiles;  // source tile (row ti, column tj)
  const T* s = src + static_cast<int64_t>(idx[p]) * b * b;
  T* d = dst + p * static_cast<int64_t>(b) * b;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  for (int y = ty; y < 32; y += 8) {
    const int r = ti * 32 + y, c = tj * 32 + tx;
    if (r < b && c < b) tile[y][tx] = s[static_cast<int64_t>(r) * b + c];
  }
  __syncthreads();
  for (int y = ty; y < 32; y += 8) {
    const int r = tj * 32 + y, c = ti * 32 + tx;  // destination row = source column
    if (r < b && c < b) d[static_cast<int64_t>(r) * b + c] = tile[tx][y];
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

// Launch a kernel templated on <T, VEC> with 16-byte pieces when rows and bases allow.
bool vec_ok(const void* p, int64_t lda, int64_t b, int vec) {
  return aligned16(p) && lda % vec == 0 && b % vec == 0;
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
    if (dtype == TRNSPARSE_F32) {
      if (vec_ok(A, lda, block_size, 4))
        bsr_screen_kernel<float, 4><<<g, 256, 0, st>>>(m, n, (const float*)A, lda, block_size, threshold, nbc, pos);
      else
        bsr_screen_kernel<float, 1><<<g, 256, 0, st>>>(m, n, (const float*)A, lda, block_size, threshold, nbc, pos);
    } else {
      using B16 = __nv_bfloat16;
      if (vec_ok(A, lda, block_size, 8))
        bsr_screen_kernel<B16, 8><<<g, 256, 0, st>>>(m, n, (const B16*)A, lda, block_size, threshold, nbc, pos);
      else
        bsr_screen_kernel<B16, 1><<<g, 256, 0, st>>>(m, n, (const B16*)A, lda, block_size, threshold, nbc, pos);
    }
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
  if (dtype == TRNSPARSE_F32) {
    if (vec_ok(A, lda, block_size, 4) && aligned16(blocks))
      bsr_fill_kernel<float, 4><<<g, 256, 0, st>>>(m, n, (const float*)A, lda, block_size, nbc, pos, (float*)blocks,
                                                   block_col_idx);
    else
      bsr_fill_kernel<float, 1><<<g, 256, 0, st>>>(m, n, (const float*)A, lda, block_size, nbc, pos, (float*)blocks,
                                                   block_col_idx);
  } else {
    using B16 = __nv_bfloat16;
    if (vec_ok(A, lda, block_size, 8) && aligned16(blocks))
      bsr_fill_kernel<B16, 8><<<g, 256, 0, st>>>(m, n, (const B16*)A, lda, block_size, nbc, pos, (B16*)blocks,
                                                 block_col_idx);
    else
      bsr_fill_kernel<B16, 1><<<g, 256, 0, st>>>(m, n, (const B16*)A, lda, block_size, nbc, pos, (B16*)blocks,
                                                 block_col_idx);
  }
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
    const unsigned gr = grid_for(m, 8);
    if (dtype == TRNSPARSE_F32) {
      if (vec_ok(A, lda, 4, 4))
        csr_count_kernel<float, 4><<<gr, 256, 0, st>>>(m, n, (const float*)A, lda, threshold, row_ptr);
      else
        csr_count_kernel<float, 1><<<gr, 256, 0, st>>>(m, n, (const float*)A, lda, threshold, row_ptr);
    } else {
      using B16 = __nv_bfloat16;
      if (vec_ok(A, lda, 8, 8))
        csr_count_kernel<B16, 8><<<gr, 256, 0, st>>>(m, n, (const B16*)A, lda, threshold, row_ptr);
      else
        csr_count_kernel<B16, 1><<<gr, 256, 0, st>>>(m, n, (const B16*)A, lda, threshold, row_ptr);
    }
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
  const unsigned gr = grid_for(m, 8);
  if (dtype == TRNSPARSE_F32) {
    if (vec_ok(A, lda, 4, 4))
      csr_fill_kernel<float, 4><<<gr, 256, 0, st>>>(m, n, (const float*)A, lda, threshold, row_ptr, (float*)values,
                                                    col_idx);
    else
      csr_fill_kernel<float, 1><<<gr, 256, 0, st>>>(m, n, (const float*)A, lda, threshold, row_ptr, (float*)values,
                                                    col_idx);
  } else {
    using B16 = __nv_bfloat16;
    if (vec_ok(A, lda, 8, 8))
      csr_fill_kernel<B16, 8><<<gr, 256, 0, st>>>(m, n, (const B16*)A, lda, threshold, row_ptr, (B16*)values, col_idx);
    else
      csr_fill_kernel<B16, 1><<<gr, 256, 0, st>>>(m, n, (const B16*)A, lda, threshold, row_ptr, (B16*)values, col_idx);
  }
  TSB_CHECK_LAUNCH("csr_from_dense: fill");
  return TRNSPARSE_OK;
}

extern "C" size_t trnsparse_csr_from_dense_mask_bytes(int64_t m, int64_t n) {
  return (m < 0 || n < 0) ? 0 : sizeof(uint32_t) * static_cast<size_t>(m) * static_cast<size_t>((n + 31) / 32);
}

extern "C" int trnsparse_csr_from_dense_count_mask(int64_t m, int64_t n, const void* A, int64_t lda, int dtype,
                                                   float threshold, long long* row_ptr, uint32_t* mask, void* ws,
                                                   size_t ws_bytes, void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && lda >= n, "csr_from_dense: bad sizes");
  TSB_REQUIRE(dtype == TRNSPARSE_F32 || dtype == TRNSPARSE_BF16, "csr_from_dense: dtype must be F32 or BF16");
  TSB_REQUIRE(row_ptr && ws && (A || m * n == 0) && (mask || m * n == 0), "csr_from_dense: null pointer");
  TSB_REQUIRE(ws_bytes >= trnsparse_csr_from_dense_workspace_size(m), "csr_from_dense: workspace too small");
  cudaStream_t st = as_stream(stream);
  if (m > 0) {
    if (n == 0) {
      cudaError_t e = cudaMemsetAsync(row_ptr, 0, sizeof(long long) * (m + 1), st);
      return cuda_status(e, "csr_from_dense: empty rows");
    }
    const int64_t mw = (n + 31) / 32;
    const unsigned gr = grid_for(m, 8);
    if (dtype == TRNSPARSE_F32) {
      if (vec_ok(A, lda, 4, 4))
        csr_count_mask_kernel<float, 4><<<gr, 256, 0, st>>>(m, n, (const float*)A, lda, threshold, row_ptr, mask, mw);
      else
        csr_count_mask_kernel<float, 1><<<gr, 256, 0, st>>>(m, n, (const float*)A, lda, threshold, row_ptr, mask, mw);
    } else {
      using B16 = __nv_bfloat16;
      if (vec_ok(A, lda, 8, 8))
        csr_count_mask_kernel<B16, 8><<<gr, 256, 0, st>>>(m, n, (const B16*)A, lda, threshold, row_ptr, mask, mw);
      else
        csr_count_mask_kernel<B16, 1><<<gr, 256, 0, st>>>(m, n, (const B16*)A, lda, threshold, row_ptr, mask, mw);
    }
    TSB_CHECK_LAUNCH("csr_from_dense: count + mask");
  }
  return exclusive_scan(row_ptr, m, static_cast<long long*>(ws), st);
}

extern "C" int trnsparse_csr_from_dense_fill_masked(int64_t m, int64_t n, const void* A, int64_t lda, int dtype,
                                                    const long long* row_ptr, const uint32_t* mask, void* values,
                                                    long long* col_idx, void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && lda >= n, "csr_from_dense: bad sizes");
  TSB_REQUIRE(dtype == TRNSPARSE_F32 || dtype == TRNSPARSE_BF16, "csr_from_dense: dtype must be F32 or BF16");
  if (m == 0 || n == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(A && row_ptr && mask && values && col_idx, "csr_from_dense: null pointer");
  cudaStream_t st = as_stream(stream);
  const unsigned gr = grid_for(m, 8);
  const int64_t mw = (n + 31) / 32;
  if (dtype == TRNSPARSE_F32)
    csr_fill_masked_kernel<float><<<gr, 256, 0, st>>>(m, n, (const float*)A, lda, row_ptr, mask, mw, (float*)values,
                                                      col_idx);
  else
    csr_fill_masked_kernel<__nv_bfloat16><<<gr, 256, 0, st>>>(m, n, (const __nv_bfloat16*)A, lda, row_ptr, mask, mw,
                                                              (__nv_bfloat16*)values, col_idx);
  TSB_CHECK_LAUNCH("csr_from_dense: masked fill");
  return TRNSPARSE_OK;
}

// ---------------------------------------------------------------- COO -> CSR
namespace tsb {
namespace {
template <int ESZ>
int coo_bucketed_launch(int64_t m, int64_t n, int64_t nnz, int nb, int64_t chunk, int64_t G, const long long* rows,
                        const long long* cols, const void* values, const long long* cm, uint16_t* plrow,
                        unsigned long long* pkey, void* pval, long long* row_ptr, unsigned long long* keys,
                        long long* cols_out, void* values_out, long long* mid_rows, unsigned long long* n_mid,
                        long long* long_rows, unsigned long long* n_long, cudaStream_t st) {
  if (nnz > 0) {
    auto pk = coo_partition_kernel<ESZ>;
    const size_t psm = coo_partition_smem(ESZ, nb);
    cudaError_t e = cudaFuncSetAttribute(pk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)psm);
    if (e != cudaSuccess) return cuda_status(e, "coo_to_csr: partition smem");
    pk<<<(unsigned)G, kPartThreads, psm, st>>>(nnz, m, n, nb, chunk, rows, cols, values, cm, plrow, pkey, pval);
    TSB_CHECK_LAUNCH("coo_to_csr: partition");
  }
  auto bk = coo_bucket_sort_kernel<ESZ>;
  const size_t budget = TSB_COO_BUCKET_KB * 1024;
  const int cap = static_cast<int>((budget - coo_bucket_smem_fixed()) / coo_bucket_entry_bytes(ESZ)) & ~7;
  // a bucket's short rows hold at most kBucketRows * kTiny entries: that many sub-ranges of
  // cap - kTiny must fit the kernel's boundary table
  TSB_REQUIRE(cap > 2 * kTiny && (kBucketRows * kTiny + cap - kTiny - 1) / (cap - kTiny) <= kMaxSub,
              "coo_to_csr: bucket staging area too small (%d entries)", cap);
  const size_t bsm = coo_bucket_smem_fixed() + static_cast<size_t>(cap) * coo_bucket_entry_bytes(ESZ) + 16;
  cudaError_t e = cudaFuncSetAttribute(bk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bsm);
  if (e != cudaSuccess) return cuda_status(e, "coo_to_csr: bucket smem");
  const int grid = nb < sm_count() ? nb : sm_count();
  bk<<<grid, kBucketThreads, bsm, st>>>(m, nb, G, cap, cm, plrow, pkey, pval, row_ptr, keys, cols_out, values_out,
                                        mid_rows, n_mid, long_rows, n_long);
  TSB_CHECK_LAUNCH("coo_to_csr: bucket sort");
  return TRNSPARSE_OK;
}

// esz: value bytes (2, 4 or 8), or 0 with values == nullptr (emit the entry index)
int coo_bucketed_sort(int esz, int64_t m, int64_t n, int64_t nnz, int nb, int64_t chunk, int64_t G,
                      const long long* rows, const long long* cols, const void* values, const long long* cm,
                      uint16_t* plrow, unsigned long long* pkey, void* pval, long long* row_ptr,
                      unsigned long long* keys, long long* cols_out, void* values_out, long long* mid_rows,
                      unsigned long long* n_mid, long long* long_rows, unsigned long long* n_long, cudaStream_t st) {
  if (values == nullptr) esz = 0;
  switch (esz) {
    case 0:
      return coo_bucketed_launch<0>(m, n, nnz, nb, chunk, G, rows, cols, values, cm, plrow, pkey, pval, row_ptr,
                                    keys, cols_out, values_out, mid_rows, n_mid, long_rows, n_long, st);
    case 2:
      return coo_bucketed_launch<2>(m, n, nnz, nb, chunk, G, rows, cols, values, cm, plrow, pkey, pval, row_ptr,
                                    keys, cols_out, values_out, mid_rows, n_mid, long_rows, n_long, st);
    case 4:
      return coo_bucketed_launch<4>(m, n, nnz, nb, chunk, G, rows, cols, values, cm, plrow, pkey, pval, row_ptr,
                                    keys, cols_out, values_out, mid_rows, n_mid, long_rows, n_long, st);
    default:
      return coo_bucketed_launch<8>(m, n, nnz, nb, chunk, G, rows, cols, values, cm, plrow, pkey, pval, row_ptr,
                                    keys, cols_out, values_out, mid_rows, n_mid, long_rows, n_long, st);
  }
}

// The bucketed COO -> CSR on a workspace laid out as trnsparse_coo_to_csr's (entries with
// an out-of-range index are left out and flag `bad`): count, scan, partition, per-bucket
// sort, then the warp / CTA sorts of the longer rows. values may be null (then the entry
// index is emitted as an int64 per entry).
int coo_to_csr_bucketed(int64_t m, int64_t n, int64_t nnz, const long long* rows, const long long* cols,
                        const void* values, int esz, long long* row_ptr, long long* cols_out, void* values_out,
                        void* ws, cudaStream_t st) {
  unsigned long long* keys = static_cast<unsigned long long*>(ws);
  unsigned long long* keys2 = keys + nnz;
  unsigned long long* cursor = keys2 + nnz;  // m entries
  long long* part = reinterpret_cast<long long*>(cursor + m + 1);
  long long* mid_rows = reinterpret_cast<long long*>(reinterpret_cast<uint8_t*>(part) + scan_ws_bytes(m));
  long long* long_rows = mid_rows + m;
  unsigned long long* n_mid = reinterpret_cast<unsigned long long*>(long_rows + m);
  unsigned long long* n_long = n_mid + 1;
  int* bad = reinterpret_cast<int*>(n_long + 1);
  cudaError_t e = cudaMemsetAsync(n_mid, 0, 24, st);  // n_mid, n_long and bad
  if (e != cudaSuccess) return cuda_status(e, "coo_to_csr: clear");
  const int nb = static_cast<int>((m + kBucketRows - 1) / kBucketRows);
  const int64_t chunk = coo_chunk(nnz, nb);
  const int64_t G = nnz > 0 ? (nnz + chunk - 1) / chunk : 1;
  uint8_t* pval = reinterpret_cast<uint8_t*>(n_mid) + 32;  // past n_mid, n_long, bad (8 bytes per entry)
  uint16_t* plrow = reinterpret_cast<uint16_t*>(pval + 8 * (size_t)nnz);
  long long* cm = reinterpret_cast<long long*>(
      (reinterpret_cast<uintptr_t>(plrow + nnz) + 15) & ~static_cast<uintptr_t>(15));  // nb * G + 1 cells
  long long* cpart = cm + nb * G + 1;                                                   // its scan partials
  if (nnz > 0) {
    coo_bucket_count_kernel<<<(unsigned)G, 256, 0, st>>>(nnz, m, n, nb, chunk, rows, cols, cm, bad);
    TSB_CHECK_LAUNCH("coo_to_csr: bucket count");
  } else {
    e = cudaMemsetAsync(cm, 0, sizeof(long long) * (nb * G + 1), st);
    if (e != cudaSuccess) return cuda_status(e, "coo_to_csr: clear counts");
  }
  int rc = exclusive_scan(cm, nb * G, cpart, st);
  if (rc) return rc;
  rc = coo_bucketed_sort(esz, m, n, nnz, nb, chunk, G, rows, cols, values, cm, plrow, keys2, pval, row_ptr, keys,
                         cols_out, values_out, mid_rows, n_mid, long_rows, n_long, st);
  if (rc || nnz == 0) return rc;
  // the rows of more than kTiny entries (listed by the bucket pass)
  const uint8_t* vin = static_cast<const uint8_t*>(values);
  const int vesz = values ? esz : 8;
  coo_sort_mid_kernel<<<grid_for(m, 8), 256, 0, st>>>(row_ptr, mid_rows, n_mid, keys, vin, vesz, cols_out,
                                                     (uint8_t*)values_out);
  coo_sort_long_kernel<<<grid_for(m, 1), kSortThreads, 0, st>>>(row_ptr, long_rows, n_long, keys, keys2, vin, vesz,
                                                               cols_out, (uint8_t*)values_out);
  TSB_CHECK_LAUNCH("coo_to_csr: sort");
  return TRNSPARSE_OK;
}
}  // namespace
}  // namespace tsb

extern "C" size_t trnsparse_coo_to_csr_workspace_size(int64_t m, int64_t nnz) {
  if (m < 0 || nnz < 0) return 0;
  // keys, keys2, cursors, scan partials, row lists, counters; then, for the bucketed
  // path, the partitioned values (up to 8 bytes each), the local rows (16 bits per
  // entry), the count matrix and its scan partials
  size_t extra = 0;
  if (m > 0 && m <= static_cast<int64_t>(kBucketRows) * kMaxBuckets) {
    const int nb = static_cast<int>((m + kBucketRows - 1) / kBucketRows);
    const int64_t chunk = coo_chunk(nnz, nb);
    const int64_t G = nnz > 0 ? (nnz + chunk - 1) / chunk : 1;
    extra = 8 * (size_t)nnz + ((sizeof(uint16_t) * (size_t)nnz + 255) & ~(size_t)255) + 16 + sizeof(long long) * (size_t)(nb * G + 1) +
            scan_ws_bytes(nb * G);
  }
  return sizeof(unsigned long long) * (size_t)(2 * nnz + 3 * m + 1) + scan_ws_bytes(m) + 32 + extra;
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
  long long* mid_rows = reinterpret_cast<long long*>(reinterpret_cast<uint8_t*>(part) + scan_ws_bytes(m));
  long long* long_rows = mid_rows + m;
  unsigned long long* n_mid = reinterpret_cast<unsigned long long*>(long_rows + m);
  unsigned long long* n_long = n_mid + 1;
  int* bad = reinterpret_cast<int*>(n_long + 1);
  cudaError_t e = cudaSuccess;
  if (m > 0 && m <= static_cast<int64_t>(kBucketRows) * kMaxBuckets) {
    // bucketed path: no per-entry global atomic (see coo_bucket_*_kernel)
    int rc = coo_to_csr_bucketed(m, n, nnz, rows, cols, values, esz, row_ptr, cols_out, values_out, ws, st);
    if (rc) return rc;
    if (nnz == 0) return TRNSPARSE_OK;
  } else {
    e = cudaMemsetAsync(n_mid, 0, 24, st);  // n_mid, n_long and bad
    if (e == cudaSuccess) e = cudaMemsetAsync(row_ptr, 0, sizeof(long long) * (m + 1), st);
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
    coo_sort_tiny_kernel<<<grid_for(m, 256), 256, 0, st>>>(m, row_ptr, keys, (const uint8_t*)values, esz, cols_out,
                                                          (uint8_t*)values_out, mid_rows, n_mid, long_rows, n_long);
    coo_sort_mid_kernel<<<grid_for(m, 8), 256, 0, st>>>(row_ptr, mid_rows, n_mid, keys, (const uint8_t*)values, esz,
                                                       cols_out, (uint8_t*)values_out);
    coo_sort_long_kernel<<<grid_for(m, 1), kSortThreads, 0, st>>>(row_ptr, long_rows, n_long, keys, keys2,
                                                                 (const uint8_t*)values, esz, cols_out,
                                                                 (uint8_t*)values_out);
    TSB_CHECK_LAUNCH("coo_to_csr: sort");
  }
  // an out-of-range index is an argument error the caller sees on the host
  int hbad = 0;
  e = cudaMemcpyAsync(&hbad, bad, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_status(e, "coo_to_csr: status");
  TSB_REQUIRE(!hbad, "coo_to_csr: a row or column index is out of range");
  return TRNSPARSE_OK;
}

// ---------------------------------------------------------------- transposes
extern "C" size_t trnsparse_csr_transpose_workspace_size(int64_t m, int64_t n, int64_t nnz) {
  if (m < 0 || n < 0 || nnz < 0) return 0;
  return trnsparse_coo_to_csr_workspace_size(n, nnz) + 2 * sizeof(long long) * (size_t)nnz + 256;
}

extern "C" int trnsparse_csr_transpose(int64_t m, int64_t n, int64_t nnz, int index_type, const void* row_ptr,
                                       const void* col_idx, int strict, long long* row_ptr_t, long long* col_t,
                                       long long* perm, void* ws, size_t ws_bytes, void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && nnz >= 0, "csr_transpose: bad sizes");
  TSB_REQUIRE(nnz < (1ll << 32) && m < (1ll << 31), "csr_transpose: nnz must be < 2^32 and m < 2^31");
  TSB_REQUIRE(index_type == TRNSPARSE_I32 || index_type == TRNSPARSE_I64, "csr_transpose: bad index type");
  TSB_REQUIRE(!strict || m == n, "csr_transpose: the strict triangle needs a square matrix");
  TSB_REQUIRE(row_ptr && row_ptr_t && ws, "csr_transpose: null pointer");
  TSB_REQUIRE(nnz == 0 || (col_idx && col_t && perm), "csr_transpose: null pointer");
  TSB_REQUIRE(ws_bytes >= trnsparse_csr_transpose_workspace_size(m, n, nnz), "csr_transpose: workspace too small");
  cudaStream_t st = as_stream(stream);
  long long* trow = static_cast<long long*>(ws);
  long long* tcol = trow + nnz;
  uint8_t* cws = reinterpret_cast<uint8_t*>(tcol + nnz);
  unsigned long long* keys = reinterpret_cast<unsigned long long*>(cws);
  unsigned long long* keys2 = keys + nnz;
  unsigned long long* cursor = keys2 + nnz;
  long long* part = reinterpret_cast<long long*>(cursor + n + 1);
  long long* mid_rows = reinterpret_cast<long long*>(reinterpret_cast<uint8_t*>(part) + scan_ws_bytes(n));
  long long* long_rows = mid_rows + n;
  unsigned long long* n_mid = reinterpret_cast<unsigned long long*>(long_rows + n);
  unsigned long long* n_long = n_mid + 1;
  int* bad = reinterpret_cast<int*>(n_long + 1);
  cudaError_t e = cudaMemsetAsync(row_ptr_t, 0, sizeof(long long) * (n + 1), st);
  if (e == cudaSuccess) e = cudaMemsetAsync(n_mid, 0, 24, st);
  if (e != cudaSuccess) return cuda_status(e, "csr_transpose: clear");
  if (nnz > 0 && m > 0) {
    if (index_type == TRNSPARSE_I32)
      csr_entry_coords_kernel<int><<<grid_for(m, 8), 256, 0, st>>>(m, static_cast<const int*>(row_ptr),
                                                                   static_cast<const int*>(col_idx), strict, trow, tcol);
    else
      csr_entry_coords_kernel<long long><<<grid_for(m, 8), 256, 0, st>>>(
          m, static_cast<const long long*>(row_ptr), static_cast<const long long*>(col_idx), strict, trow, tcol);
    TSB_CHECK_LAUNCH("csr_transpose: coordinates");
  }
  if (n > 0 && n <= static_cast<int64_t>(kBucketRows) * kMaxBuckets) {
    // the entries as a COO of A^T (diagonal entries left out of the strict triangle carry
    // row -1, which the bucketed sort skips); the emitted "values" are the entry indices
    return coo_to_csr_bucketed(n, m, m > 0 ? nnz : 0, trow, tcol, nullptr, 0, row_ptr_t, col_t, perm, cws, st);
  }
  if (nnz > 0 && m > 0) {
    coo_count_kernel<<<grid_for(nnz, 256), 256, 0, st>>>(nnz, n, m, trow, tcol,
                                                        reinterpret_cast<unsigned long long*>(row_ptr_t), bad, 1);
    TSB_CHECK_LAUNCH("csr_transpose: count");
  }
  int rc = exclusive_scan(row_ptr_t, n, part, st);
  if (rc) return rc;
  if (nnz == 0 || n == 0 || m == 0) return TRNSPARSE_OK;
  e = cudaMemcpyAsync(cursor, row_ptr_t, sizeof(long long) * n, cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return cuda_status(e, "csr_transpose: cursors");
  coo_scatter_kernel<<<grid_for(nnz, 256), 256, 0, st>>>(nnz, n, m, trow, tcol, cursor, keys);
  coo_sort_tiny_kernel<<<grid_for(n, 256), 256, 0, st>>>(n, row_ptr_t, keys, nullptr, 8, col_t, (uint8_t*)perm,
                                                        mid_rows, n_mid, long_rows, n_long);
  coo_sort_mid_kernel<<<grid_for(n, 8), 256, 0, st>>>(row_ptr_t, mid_rows, n_mid, keys, nullptr, 8, col_t,
                                                     (uint8_t*)perm);
  coo_sort_long_kernel<<<grid_for(n, 1), kSortThreads, 0, st>>>(row_ptr_t, long_rows, n_long, keys, keys2, nullptr,
                                                               8, col_t, (uint8_t*)perm);
  TSB_CHECK_LAUNCH("csr_transpose: sort");
  return TRNSPARSE_OK;
}

extern "C" int trnsparse_gather(int64_t count, int elem_bytes, const void* src, const long long* idx, void* dst,
                                void* stream) {
  TSB_REQUIRE(count >= 0, "gather: bad count");
  TSB_REQUIRE(elem_bytes == 2 || elem_bytes == 4 || elem_bytes == 8, "gather: element size must be 2, 4 or 8");
  if (count == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(src && idx && dst, "gather: null pointer");
  cudaStream_t st = as_stream(stream);
  const int g = grid_for(count, 256);
  if (elem_bytes == 2)
    gather_kernel<uint16_t><<<g, 256, 0, st>>>(count, (const uint16_t*)src, idx, (uint16_t*)dst);
  else if (elem_bytes == 4)
    gather_kernel<uint32_t><<<g, 256, 0, st>>>(count, (const uint32_t*)src, idx, (uint32_t*)dst);
  else
    gather_kernel<uint64_t><<<g, 256, 0, st>>>(count, (const uint64_t*)src, idx, (uint64_t*)dst);
  TSB_CHECK_LAUNCH("gather");
  return TRNSPARSE_OK;
}

extern "C" int trnsparse_bsr_blocks_transpose(int64_t count, int b, int elem_bytes, const void* src,
                                              const long long* idx, void* dst, void* stream) {
  TSB_REQUIRE(count >= 0 && b > 0, "bsr_blocks_transpose: bad sizes");
  TSB_REQUIRE(count < 65536 * 1024ll, "bsr_blocks_transpose: too many blocks");
  TSB_REQUIRE(elem_bytes == 2 || elem_bytes == 4, "bsr_blocks_transpose: element size must be 2 or 4");
  if (count == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(src && idx && dst, "bsr_blocks_transpose: null pointer");
  cudaStream_t st = as_stream(stream);
  const int tiles = (b + 31) / 32;
  int rc = TRNSPARSE_OK;
  for (int64_t c0 = 0; c0 < count && rc == TRNSPARSE_OK; c0 += 65535) {  // grid.y is at most 65535
    const int64_t c = count - c0 < 65535 ? count - c0 : 65535;
    dim3 grid(tiles * tiles, static_cast<unsigned>(c));
    if (elem_bytes == 2)
      block_transpose_gather_kernel<uint16_t><<<grid, 256, 0, st>>>(b, (const uint16_t*)src, idx + c0,
                                                                     (uint16_t*)dst + c0 * b * b);
    else
      block_transpose_gather_kernel<uint32_t><<<grid, 256, 0, st>>>(b, (const uint32_t*)src, idx + c0,
                                                                     (uint32_t*)dst + c0 * b * b);
    TSB_CHECK_LAUNCH("bsr_blocks_transpose");
  }
  return rc;
}
