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
#include "ptx.cuh"

#include <stdlib.h>

#include <mutex>

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
    // products v[j] * x[col[j]] element-parallel (every x gather of the slice
    // is independent, so each thread keeps several in flight), in place
    T* vrow = vs + st.dv;
    const I* crow = cs + st.dc;
    const int span = static_cast<int>(st.e - st.s);
    int q = threadIdx.x;
    for (; q + 3 * kThreads < span; q += 4 * kThreads) {
      const int64_t c0 = crow[q], c1 = crow[q + kThreads], c2 = crow[q + 2 * kThreads], c3 = crow[q + 3 * kThreads];
      const T x0 = __ldg(x + c0), x1 = __ldg(x + c1), x2 = __ldg(x + c2), x3 = __ldg(x + c3);
      vrow[q] = mul_rn(vrow[q], x0);
      vrow[q + kThreads] = mul_rn(vrow[q + kThreads], x1);
      vrow[q + 2 * kThreads] = mul_rn(vrow[q + 2 * kThreads], x2);
      vrow[q + 3 * kThreads] = mul_rn(vrow[q + 3 * kThreads], x3);
    }
    for (; q < span; q += kThreads) vrow[q] = mul_rn(vrow[q], __ldg(x + static_cast<int64_t>(crow[q])));
    __syncthreads();
    for (int r = threadIdx.x; r < nrows; r += blockDim.x) {
      const int a = rps[r], b = rps[r + 1];
      T acc = T(0);
      for (int j = a; j < b; ++j) acc = add_rn(acc, vrow[j]);
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


// ---------------------------------------------------------------------------
// Pipelined SpMV: persistent CTAs, each walking its tiles (R rows each) with a
// kStages-deep ring of shared-memory stages filled by 1-D bulk (TMA) copies
// of the tile's row pointers, values and column indices, so several tiles'
// loads stay in flight while earlier tiles are computed. Tiles whose slice
// does not fit a stage (or the ragged last tile) are computed straight from
// global memory.
constexpr int kStages = 4;
constexpr int kMaxTilesPerCta = 128;

struct TileMeta {
  int64_t s, e;  // nnz range of the tile
  int dv, dc;    // offset of s inside the staged values / columns
  int regular;
  int pad;
};

template <typename I, typename T>
struct PipeLayout {
  int R, cap;
  size_t rps_bytes, vals_bytes, cols_bytes, stage_bytes;
  __host__ __device__ PipeLayout(int R_, int cap_) : R(R_), cap(cap_) {
    rps_bytes = ((size_t)R * sizeof(I) + 15) & ~(size_t)15;
    vals_bytes = ((size_t)(cap + 16) * sizeof(T) + 15) & ~(size_t)15;
    cols_bytes = ((size_t)(cap + 16) * sizeof(I) + 15) & ~(size_t)15;
    stage_bytes = rps_bytes + vals_bytes + cols_bytes;
  }
  static constexpr size_t head_bytes() {
    return 64 /* barriers */ + kStages * sizeof(TileMeta) + 2 * kMaxTilesPerCta * sizeof(int64_t);
  }
  __host__ __device__ size_t total() const { return head_bytes() + kStages * stage_bytes + vals_bytes; }
};

template <typename I, typename T>
__global__ void __launch_bounds__(kThreads)
csr_spmv_pipe_kernel(int64_t m, int64_t nnz, const I* __restrict__ rp, const I* __restrict__ ci,
                     const T* __restrict__ v, const T* __restrict__ x, T alpha, const T* __restrict__ y, T beta,
                     T* __restrict__ out, int R, int cap, int64_t ntiles) {
  extern __shared__ __align__(16) unsigned char smem[];
  const PipeLayout<I, T> L(R, cap);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  TileMeta* meta = reinterpret_cast<TileMeta*>(smem + 64);
  int64_t* bs = reinterpret_cast<int64_t*>(smem + 64 + kStages * sizeof(TileMeta));
  int64_t* be = bs + kMaxTilesPerCta;
  unsigned char* stages = smem + PipeLayout<I, T>::head_bytes();
  T* prod = reinterpret_cast<T*>(stages + kStages * L.stage_bytes);
  constexpr int VT = 16 / sizeof(T);
  constexpr int VC = 16 / sizeof(I);

  const int64_t G = gridDim.x;
  const int nt = static_cast<int>((ntiles - blockIdx.x + G - 1) / G);
  for (int i = threadIdx.x; i < nt; i += kThreads) {
    const int64_t r0 = (blockIdx.x + i * G) * R;
    bs[i] = static_cast<int64_t>(rp[r0]);
    be[i] = static_cast<int64_t>(rp[r0 + R < m ? r0 + R : m]);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  auto stage_rps = [&](int s) { return reinterpret_cast<I*>(stages + s * L.stage_bytes); };
  auto stage_vals = [&](int s) { return reinterpret_cast<T*>(stages + s * L.stage_bytes + L.rps_bytes); };
  auto stage_cols = [&](int s) {
    return reinterpret_cast<I*>(stages + s * L.stage_bytes + L.rps_bytes + L.vals_bytes);
  };

  // thread 0: start loading tile i into stage i % kStages
  auto fill = [&](int i) {
    const int s = i % kStages;
    const int64_t r0 = (blockIdx.x + i * G) * R;
    const int64_t S = bs[i], E = be[i];
    const int64_t s0v = S & ~(int64_t)(VT - 1), e1v = (E + VT - 1) & ~(int64_t)(VT - 1);
    const int64_t s0c = S & ~(int64_t)(VC - 1), e1c = (E + VC - 1) & ~(int64_t)(VC - 1);
    TileMeta mt;
    mt.s = S;
    mt.e = E;
    mt.dv = static_cast<int>(S - s0v);
    mt.dc = static_cast<int>(S - s0c);
    mt.regular = (r0 + R <= m) && (E > S) && (E - S <= cap) && (e1v <= nnz) && (e1c <= nnz);
    mt.pad = 0;
    meta[s] = mt;
    if (mt.regular) {
      const uint32_t bv = static_cast<uint32_t>((e1v - s0v) * sizeof(T));
      const uint32_t bc = static_cast<uint32_t>((e1c - s0c) * sizeof(I));
      const uint32_t br = static_cast<uint32_t>(R * sizeof(I));
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&bars[s], br + bv + bc);
      bulk_g2s(stage_rps(s), rp + r0, br, &bars[s]);
      bulk_g2s(stage_vals(s), v + s0v, bv, &bars[s]);
      bulk_g2s(stage_cols(s), ci + s0c, bc, &bars[s]);
    } else {
      mbar_arrive(&bars[s]);
    }
  };

  if (threadIdx.x == 0)
    for (int i = 0; i < nt && i < kStages; ++i) fill(i);

  for (int i = 0; i < nt; ++i) {
    const int s = i % kStages;
    if (!mbar_wait(&bars[s], (i / kStages) & 1)) return;
    const TileMeta mt = meta[s];
    const int64_t r0 = (blockIdx.x + i * G) * R;
    if (mt.regular) {
      const T* vals = stage_vals(s) + mt.dv;
      const I* cols = stage_cols(s) + mt.dc;
      const int span = static_cast<int>(mt.e - mt.s);
      int q = threadIdx.x;
      for (; q + 3 * kThreads < span; q += 4 * kThreads) {
        const int64_t c0 = cols[q], c1 = cols[q + kThreads], c2 = cols[q + 2 * kThreads], c3 = cols[q + 3 * kThreads];
        const T x0 = __ldg(x + c0), x1 = __ldg(x + c1), x2 = __ldg(x + c2), x3 = __ldg(x + c3);
        prod[q] = mul_rn(vals[q], x0);
        prod[q + kThreads] = mul_rn(vals[q + kThreads], x1);
        prod[q + 2 * kThreads] = mul_rn(vals[q + 2 * kThreads], x2);
        prod[q + 3 * kThreads] = mul_rn(vals[q + 3 * kThreads], x3);
      }
      for (; q < span; q += kThreads) prod[q] = mul_rn(vals[q], __ldg(x + static_cast<int64_t>(cols[q])));
      __syncthreads();
      const I* rps = stage_rps(s);
      for (int r = threadIdx.x; r < R; r += kThreads) {
        const int a = static_cast<int>(static_cast<int64_t>(rps[r]) - mt.s);
        const int b = static_cast<int>((r + 1 < R ? static_cast<int64_t>(rps[r + 1]) : mt.e) - mt.s);
        T acc = T(0);
        for (int j = a; j < b; ++j) acc = add_rn(acc, prod[j]);
        out[r0 + r] = epilogue<T>(acc, alpha, y, beta, r0 + r);
      }
    } else {
      const int nrows = static_cast<int>(m - r0 < R ? m - r0 : R);
      const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
      for (int r = warp; r < nrows; r += kThreads / 32) {
        const int64_t a = static_cast<int64_t>(rp[r0 + r]), b = static_cast<int64_t>(rp[r0 + r + 1]);
        T acc = T(0);
        for (int64_t j = a + lane; j < b; j += 32) acc += __ldg(v + j) * __ldg(x + static_cast<int64_t>(__ldg(ci + j)));
        acc = warp_sum(acc);
        if (lane == 0) out[r0 + r] = epilogue<T>(acc, alpha, y, beta, r0 + r);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0 && i + kStages < nt) fill(i + kStages);
  }
}


// ---------------------------------------------------------------------------
// Warp-chunk SpMV: each warp owns chunks of 32*RW consecutive rows. Lane l
// reads row_ptrs[r0 + l + 32 t] (coalesced loads), the warp loads the chunk's
// slice of values / column indices with 16-byte vector loads, every lane
// gathers x for its vector chunks (independent loads, all in flight
// together), products go to a warp-private shared-memory strip and lane l
// sums rows r0 + l + 32 t from it. There is no CTA-wide barrier: the 8 warps
// of a CTA run independent chains, and the next chunk's row pointers are
// prefetched before the current chunk is computed. A chunk whose slice
// exceeds the strip is done row by row by the whole warp.
template <typename I, typename T, int RW, int STRIP>
__global__ void __launch_bounds__(kThreads)
csr_spmv_warp_kernel(int64_t m, int64_t nnz, const I* __restrict__ rp, const I* __restrict__ ci,
                     const T* __restrict__ v, const T* __restrict__ x, T alpha, const T* __restrict__ y, T beta,
                     T* __restrict__ out) {
  constexpr int VT = 16 / sizeof(T);
  constexpr int ROWS = 32 * RW;
  __shared__ __align__(16) T strip_all[kThreads / 32][STRIP + 8];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  T* strip = strip_all[w];
  const int64_t nchunks = (m + ROWS - 1) / ROWS;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
  int64_t chunk = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) + w;
  // lane l holds rp[r0 + l + 32 t] in pa[t]; pe = rp[r0 + ROWS] (clamped to m)
  int64_t pa[RW], pe = 0;
  auto load_ptrs = [&](int64_t c) {
    const int64_t r0 = c * ROWS;
#pragma unroll
    for (int t = 0; t < RW; ++t) pa[t] = static_cast<int64_t>(__ldg(rp + min(r0 + lane + 32 * t, m)));
    pe = static_cast<int64_t>(__ldg(rp + min(r0 + ROWS, m)));
  };
  if (chunk < nchunks) load_ptrs(chunk);
  for (; chunk < nchunks; chunk += stride) {
    const int64_t r0 = chunk * ROWS;
    int64_t a[RW], b[RW];
#pragma unroll
    for (int t = 0; t < RW; ++t) a[t] = pa[t];
#pragma unroll
    for (int t = 0; t < RW; ++t) {
      b[t] = __shfl_down_sync(0xffffffffu, a[t], 1);
      const int64_t nextfirst = (t + 1 < RW) ? __shfl_sync(0xffffffffu, a[t + 1 < RW ? t + 1 : t], 0) : pe;
      if (lane == 31) b[t] = nextfirst;
    }
    const int64_t s = __shfl_sync(0xffffffffu, a[0], 0);
    const int64_t e = pe;
    const int64_t nxt = chunk + stride;
    if (nxt < nchunks) load_ptrs(nxt);
    const int64_t s0 = s & ~(int64_t)(VT - 1);
    if (e - s0 <= STRIP) {
      const int nv = static_cast<int>((e - s0 + VT - 1) / VT);
      constexpr int kPer = (STRIP / VT + 31) / 32;
      T vv[kPer][VT];
      I cc[kPer][VT];
#pragma unroll
      for (int t = 0; t < kPer; ++t) {
        const int c = lane + 32 * t;
        const int64_t g = s0 + static_cast<int64_t>(c) * VT;
        if (c < nv) {
          if (g + VT <= nnz) {
            typename Vec16<T>::type q = __ldcs(reinterpret_cast<const typename Vec16<T>::type*>(v + g));
            const T* qp = reinterpret_cast<const T*>(&q);
#pragma unroll
            for (int u = 0; u < VT; ++u) vv[t][u] = qp[u];
            if constexpr (sizeof(I) * VT == 16) {
              int4 ic = __ldcs(reinterpret_cast<const int4*>(ci + g));
              const I* ip = reinterpret_cast<const I*>(&ic);
#pragma unroll
              for (int u = 0; u < VT; ++u) cc[t][u] = ip[u];
            } else {
#pragma unroll
              for (int u = 0; u < VT; ++u) cc[t][u] = ci[g + u];
            }
          } else {
#pragma unroll
            for (int u = 0; u < VT; ++u) {
              vv[t][u] = (g + u < nnz) ? v[g + u] : T(0);
              cc[t][u] = (g + u < nnz) ? ci[g + u] : I(0);
            }
          }
        }
      }
      T xv[kPer][VT];
#pragma unroll
      for (int t = 0; t < kPer; ++t) {
        const int c = lane + 32 * t;
        const int64_t g = s0 + static_cast<int64_t>(c) * VT;
#pragma unroll
        for (int u = 0; u < VT; ++u)
          xv[t][u] = (c < nv && g + u >= s && g + u < e) ? __ldg(x + static_cast<int64_t>(cc[t][u])) : T(0);
      }
#pragma unroll
      for (int t = 0; t < kPer; ++t) {
        const int c = lane + 32 * t;
        if (c < nv) {
#pragma unroll
          for (int u = 0; u < VT; ++u) strip[c * VT + u] = mul_rn(vv[t][u], xv[t][u]);
        }
      }
      __syncwarp();
#pragma unroll
      for (int t = 0; t < RW; ++t) {
        const int64_t row = r0 + lane + 32 * t;
        if (row < m) {
          T acc = T(0);
          const int lo = static_cast<int>(a[t] - s0), hi = static_cast<int>(b[t] - s0);
          for (int j = lo; j < hi; ++j) acc = add_rn(acc, strip[j]);
          out[row] = epilogue<T>(acc, alpha, y, beta, row);
        }
      }
      __syncwarp();
    } else {
      const int nrows = static_cast<int>(m - r0 < ROWS ? m - r0 : ROWS);
      for (int r = 0; r < nrows; ++r) {
        int64_t ra = 0, rb = 0;
#pragma unroll
        for (int t = 0; t < RW; ++t) {
          const int64_t ta = __shfl_sync(0xffffffffu, a[t], r & 31);
          const int64_t tb = __shfl_sync(0xffffffffu, b[t], r & 31);
          if ((r >> 5) == t) { ra = ta; rb = tb; }
        }
        T acc = T(0);
        for (int64_t j = ra + lane; j < rb; j += 32) acc += __ldg(v + j) * __ldg(x + static_cast<int64_t>(__ldg(ci + j)));
        acc = warp_sum(acc);
        if (lane == 0) out[r0 + r] = epilogue<T>(acc, alpha, y, beta, r0 + r);
      }
    }
  }
}

// SpMM: a group of G lanes owns one row; each lane owns VEC-wide column
// chunks c = lane_in_group + G*t of the k output columns.
// Eight CTAs per SM (32 registers) for 32-bit indices and values: the kernel
// is memory-latency bound and occupancy is what keeps enough B-row loads in
// flight (config 2b: 0.39 ms at four CTAs per SM, 0.30 ms at eight); the wider
// instantiations would spill at 32 registers and keep four.
template <typename I, typename T, int VEC, bool SMALL = false>
__global__ void __launch_bounds__(kThreads, (sizeof(I) == 4 && sizeof(T) == 4 && VEC > 1) ? 8 : 4)
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
        const VT* bc = reinterpret_cast<const VT*>(B) + c;
        const int64_t ldv = ldb / VEC;
        // unrolled so several independent B-row loads are in flight per group
        if (st.fits) {
          const T* vv = vs + st.dv;
          const I* cc = cs + st.dc;
#pragma unroll 4
          for (int j = static_cast<int>(a); j < static_cast<int>(b); ++j) {
            // SMALL: B fits 2^31 vector units, so 32-bit row offsets (one multiply per row)
            const VT bv = SMALL ? __ldg(bc + static_cast<int>(cc[j]) * static_cast<int>(ldv))
                                : __ldg(bc + static_cast<int64_t>(cc[j]) * ldv);
            const T val = vv[j];
            const T* bp = reinterpret_cast<const T*>(&bv);
#pragma unroll
            for (int q = 0; q < VEC; ++q) acc[q] += val * bp[q];
          }
        } else {
#pragma unroll 4
          for (int64_t j = a; j < b; ++j) {
            const VT bv = __ldg(bc + static_cast<int64_t>(__ldg(ci + st.s + j)) * ldv);
            const T val = __ldg(v + st.s + j);
            const T* bp = reinterpret_cast<const T*>(&bv);
#pragma unroll
            for (int q = 0; q < VEC; ++q) acc[q] += val * bp[q];
          }
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

inline int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
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
  static const int target = env_int("TRNSPARSE_SPMV_TILE", 640);  // tile holds target..2*target entries
  const bool vec_ok = aligned16(v) && aligned16(ci) && aligned16(rp);
  const double avg = m > 0 ? static_cast<double>(nnz) / m : 0.0;
  static const int variant = env_int("TRNSPARSE_SPMV_VARIANT", 2);  // 0 staged, 1 pipelined, 2 warp-chunk
  if (vec_ok && variant >= 2) {
    auto kern = variant == 2 ? csr_spmv_warp_kernel<I, T, 2, 384> : csr_spmv_warp_kernel<I, T, 1, 192>;
    constexpr int kRowsPer = 64;
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, 0);
    if (e != cudaSuccess) return cuda_status(e, "csr_spmv: occupancy");
    const int64_t nchunks = (m + (variant == 2 ? kRowsPer : 32) - 1) / (variant == 2 ? kRowsPer : 32);
    int64_t grid = static_cast<int64_t>(sm_count()) * (per_sm < 1 ? 1 : per_sm);
    const int64_t need = (nchunks + kThreads / 32 - 1) / (kThreads / 32);
    if (grid > need) grid = need;
    kern<<<(unsigned)grid, kThreads, 0, st>>>(m, nnz, (const I*)rp, (const I*)ci, (const T*)v, (const T*)x,
                                              (T)alpha, (const T*)y, (T)beta, (T*)out);
    TSB_CHECK_LAUNCH("csr_spmv launch");
    return TRNSPARSE_OK;
  }
  if (vec_ok && variant == 1) {
    int R = pick_rows(m, nnz, 2 * target);  // pick_rows halves: ~target entries per tile
    int cap = static_cast<int>(R * avg * 1.25) + 64;
    const PipeLayout<I, T> L(R, cap);
    const size_t sm = L.total();
    auto kern = csr_spmv_pipe_kernel<I, T>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    if (e != cudaSuccess) return cuda_status(e, "csr_spmv: set smem");
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, sm);
    if (e != cudaSuccess) return cuda_status(e, "csr_spmv: occupancy");
    if (per_sm < 1) per_sm = 1;
    const int64_t ntiles = (m + R - 1) / R;
    int64_t grid = static_cast<int64_t>(sm_count()) * per_sm;
    if (grid > ntiles) grid = ntiles;
    if (grid * kMaxTilesPerCta < ntiles) grid = (ntiles + kMaxTilesPerCta - 1) / kMaxTilesPerCta;
    if (grid > 0x7fffffff) return fail(TRNSPARSE_ERR_ARG, "csr_spmv: m=%lld too large", (long long)m);
    kern<<<(unsigned)grid, kThreads, sm, st>>>(m, nnz, (const I*)rp, (const I*)ci, (const T*)v, (const T*)x,
                                               (T)alpha, (const T*)y, (T)beta, (T*)out, R, cap, ntiles);
    TSB_CHECK_LAUNCH("csr_spmv launch");
    return TRNSPARSE_OK;
  }
  const int rows = pick_rows(m, nnz, 4096);
  int cap = static_cast<int>(rows * avg * 1.25) + 256;
  if (cap > 8192) cap = 8192;
  const size_t sm = smem_bytes<I, T>(rows, cap);
  auto kern = csr_spmv_kernel<I, T>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return cuda_status(e, "csr_spmv: set smem");
  const int64_t grid = (m + rows - 1) / rows;
  if (grid > 0x7fffffff) return fail(TRNSPARSE_ERR_ARG, "csr_spmv: m=%lld too large", (long long)m);
  kern<<<(unsigned)grid, kThreads, sm, st>>>(m, nnz, (const I*)rp, (const I*)ci, (const T*)v, (const T*)x,
                                             (T)alpha, (const T*)y, (T)beta, (T*)out, rows, cap, aligned16(v) && aligned16(ci));
  TSB_CHECK_LAUNCH("csr_spmv launch");
  return TRNSPARSE_OK;
}

template <typename I, typename T>
int launch_spmm(int64_t m, int64_t n, int64_t k, int64_t nnz, const void* rp, const void* ci, const void* v,
                const void* B, int64_t ldb, double alpha, const void* C, int64_t ldc, double beta,
                void* out, int64_t ldo, cudaStream_t st) {
  constexpr int V = Vec16<T>::n;
  const bool vec_cols = (k % V == 0) && (ldb % V == 0) && (ldo % V == 0) && aligned16(B) &&
                        aligned16(out) && (C == nullptr || ((ldc % V == 0) && aligned16(C)));
  const int64_t nchunk = vec_cols ? k / V : k;
  int G = 1;
  while (G < 32 && G < nchunk) G *= 2;
  // rows per CTA: enough row-groups to fill the CTA, and a slice that fits
  static const int target = env_int("TRNSPARSE_SPMM_TILE", 2048);  // stored entries staged per CTA
  const int rows = pick_rows(m, nnz, target);
  const double avg = m > 0 ? static_cast<double>(nnz) / m : 0.0;
  int cap = static_cast<int>(rows * avg * 1.25) + 256;
  if (cap > 8192) cap = 8192;
  const bool vec_ok = aligned16(v) && aligned16(ci);
  const size_t sm = smem_bytes<I, T>(rows, cap);
  const int64_t grid = (m + rows - 1) / rows;
  if (grid > 0x7fffffff) return fail(TRNSPARSE_ERR_ARG, "csr_spmm: m=%lld too large", (long long)m);
  // every gathered B row offset (in vector units) fits 31 bits
  const bool small_idx = vec_cols && n * (ldb / V) + nchunk < (1ll << 31);
  if (vec_cols) {
    auto kern = small_idx ? csr_spmm_kernel<I, T, V, true> : csr_spmm_kernel<I, T, V, false>;
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

// ---------------------------------------------------------------- SDDMM (value gradient)
// out[e] = alpha * <G[row_e, :k], X[col_e, :k]> for every stored entry e: the
// adjoint of alpha * A @ X with respect to A's values, projected on A's pattern.
// A warp per row. Short k: lanes take entries (each a full dot product, the
// G row read once per warp from L1); long k: lanes split the dot product and
// reduce by shuffles. Accumulates in the value type.
template <typename I, typename T>
__global__ void __launch_bounds__(256)
csr_sddmm_kernel(int64_t m, int64_t k, const I* __restrict__ row_ptrs, const I* __restrict__ col_indices,
                 const T* __restrict__ G, int64_t ldg, const T* __restrict__ X, int64_t ldx, T alpha,
                 T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < m; r += warps) {
    const int64_t e0 = static_cast<int64_t>(row_ptrs[r]), e1 = static_cast<int64_t>(row_ptrs[r + 1]);
    const T* g = G + r * ldg;
    if (k < 16) {
      for (int64_t e = e0 + lane; e < e1; e += 32) {
        const T* x = X + static_cast<int64_t>(col_indices[e]) * ldx;
        T acc = T(0);
        for (int64_t t = 0; t < k; ++t) acc += g[t] * x[t];
        out[e] = alpha * acc;
      }
    } else {
      for (int64_t e = e0; e < e1; ++e) {
        const T* x = X + static_cast<int64_t>(col_indices[e]) * ldx;
        T acc = T(0);
        for (int64_t t = lane; t < k; t += 32) acc += g[t] * x[t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) out[e] = alpha * acc;
      }
    }
  }
}

template <typename I, typename T>
int launch_sddmm(int64_t m, int64_t k, const void* rp, const void* ci, const void* G, int64_t ldg, const void* X,
                 int64_t ldx, double alpha, void* out, cudaStream_t st) {
  const int64_t blocks = (m + 7) / 8;
  const int grid = static_cast<int>(blocks < 148 * 64 ? blocks : 148 * 64);
  csr_sddmm_kernel<I, T><<<grid, 256, 0, st>>>(m, k, static_cast<const I*>(rp), static_cast<const I*>(ci),
                                               static_cast<const T*>(G), ldg, static_cast<const T*>(X), ldx,
                                               static_cast<T>(alpha), static_cast<T*>(out));
  TSB_CHECK_LAUNCH("csr_sddmm");
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

namespace {
// Per-device copy streams and events of the host-buffer SpMV pipeline (created on first use).
constexpr int kPipeMax = 64;
struct PipeCtx {
  bool ready = false;
  cudaStream_t s_in = nullptr, s_out = nullptr;
  cudaEvent_t start = nullptr, end = nullptr, in[kPipeMax] = {}, done[kPipeMax] = {};
};
PipeCtx g_pipe[64];
std::mutex g_pipe_mu;

int pipe_ctx(PipeCtx** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "csr_spmv_host: device");
  if (dev < 0 || dev >= 64) return fail(TRNSPARSE_ERR_UNSUPPORTED, "csr_spmv_host: device %d", dev);
  PipeCtx& c = g_pipe[dev];  // the caller holds g_pipe_mu
  if (!c.ready) {
    e = cudaStreamCreateWithFlags(&c.s_in, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c.s_out, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c.start, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c.end, cudaEventDisableTiming);
    for (int i = 0; i < kPipeMax && e == cudaSuccess; ++i) {
      e = cudaEventCreateWithFlags(&c.in[i], cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c.done[i], cudaEventDisableTiming);
    }
    if (e != cudaSuccess) return cuda_status(e, "csr_spmv_host: streams");
    c.ready = true;
  }
  *out = &c;
  return TRNSPARSE_OK;
}
}  // namespace

// y = alpha A x with x and y in pinned host memory: x goes up in prefix pieces on one copy
// stream, row chunk i runs once the first x_need[i] entries of x have arrived, and its rows
// go back on a second copy stream while later chunks compute (or, with out_dev == out_host,
// the kernels store them into the pinned host buffer themselves); the caller's stream waits
// for the last copy, so synchronising it (or any later work on it) sees y complete.
extern "C" int trnsparse_csr_spmv_host(int64_t m, int64_t n, int64_t nnz, int index_type, int dtype,
                                       const void* row_ptrs, const void* col_indices, const void* values,
                                       const void* x_host, double alpha, void* out_host, void* x_dev, void* out_dev,
                                       int n_chunks, const int64_t* row_splits, const int64_t* x_need,
                                       void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && nnz >= 0, "csr_spmv_host: negative size");
  if (m == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(n_chunks > 0 && n_chunks <= kPipeMax, "csr_spmv_host: n_chunks must be 1..%d", kPipeMax);
  TSB_REQUIRE(row_ptrs && x_host && out_host && x_dev && out_dev && row_splits && x_need,
              "csr_spmv_host: null pointer");
  TSB_REQUIRE(dtype == TRNSPARSE_F32 || dtype == TRNSPARSE_F64, "csr_spmv_host: dtype %d (F32, F64)", dtype);
  TSB_REQUIRE(index_type == TRNSPARSE_I32 || index_type == TRNSPARSE_I64, "csr_spmv_host: index type %d",
              index_type);
  TSB_REQUIRE(row_splits[0] == 0 && row_splits[n_chunks] == m, "csr_spmv_host: row_splits must span [0, m)");
  for (int i = 0; i < n_chunks; ++i)
    TSB_REQUIRE(row_splits[i + 1] >= row_splits[i] && x_need[i] >= 0 && x_need[i] <= n &&
                    (i == 0 || x_need[i] >= x_need[i - 1]),
                "csr_spmv_host: row_splits ascending, x_need ascending within [0, n]");
  std::lock_guard<std::mutex> lk(g_pipe_mu);  // one issue sequence at a time: the events are shared
  PipeCtx* c = nullptr;
  int rc = pipe_ctx(&c);
  if (rc) return rc;
  cudaStream_t st = as_stream(stream);
  const size_t es = dtype == TRNSPARSE_F32 ? 4 : 8, is = index_type == TRNSPARSE_I32 ? 4 : 8;
  cudaError_t e = cudaEventRecord(c->start, st);  // the scratch buffers' earlier users come first
  if (e == cudaSuccess) e = cudaStreamWaitEvent(c->s_in, c->start, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(c->s_out, c->start, 0);
  // x pieces: one per distinct prefix length
  int64_t have = 0;
  int piece[kPipeMax];
  int np = 0;
  for (int i = 0; i < n_chunks && e == cudaSuccess; ++i) {
    if (x_need[i] > have) {
      e = cudaMemcpyAsync(static_cast<uint8_t*>(x_dev) + have * es, static_cast<const uint8_t*>(x_host) + have * es,
                          (x_need[i] - have) * es, cudaMemcpyHostToDevice, c->s_in);
      if (e == cudaSuccess) e = cudaEventRecord(c->in[np], c->s_in);
      have = x_need[i];
      ++np;
    }
    piece[i] = np - 1;
  }
  int waited = -1;
  for (int i = 0; i < n_chunks && e == cudaSuccess; ++i) {
    const int64_t a = row_splits[i], b = row_splits[i + 1];
    if (piece[i] > waited) {
      e = cudaStreamWaitEvent(st, c->in[piece[i]], 0);
      waited = piece[i];
      if (e != cudaSuccess) break;
    }
    if (b > a) {
      const void* rp = static_cast<const uint8_t*>(row_ptrs) + a * is;
      void* o = static_cast<uint8_t*>(out_dev) + a * es;
      if (dtype == TRNSPARSE_F32)
        rc = index_type == TRNSPARSE_I32
                 ? launch_spmv<int32_t, float>(b - a, nnz, rp, col_indices, values, x_dev, alpha, nullptr, 0.0, o, st)
                 : launch_spmv<int64_t, float>(b - a, nnz, rp, col_indices, values, x_dev, alpha, nullptr, 0.0, o, st);
      else
        rc = index_type == TRNSPARSE_I32
                 ? launch_spmv<int32_t, double>(b - a, nnz, rp, col_indices, values, x_dev, alpha, nullptr, 0.0, o, st)
                 : launch_spmv<int64_t, double>(b - a, nnz, rp, col_indices, values, x_dev, alpha, nullptr, 0.0, o,
                                                st);
      if (rc) return rc;
      if (out_dev != out_host) {  // otherwise the kernel has written the rows to host memory itself
        e = cudaEventRecord(c->done[i], st);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(c->s_out, c->done[i], 0);
        if (e == cudaSuccess)
          e = cudaMemcpyAsync(static_cast<uint8_t*>(out_host) + a * es, o, (b - a) * es, cudaMemcpyDeviceToHost,
                              c->s_out);
      }
    }
  }
  if (e == cudaSuccess) e = cudaEventRecord(c->end, c->s_out);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(st, c->end, 0);
  return cuda_status(e, "csr_spmv_host");
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
    if (index_type == TRNSPARSE_I32) return launch_spmm<int32_t, float>(m, n, k, nnz, row_ptrs, col_indices, values, B, ldb, alpha, C, ldc, beta, out, ldo, st);
    if (index_type == TRNSPARSE_I64) return launch_spmm<int64_t, float>(m, n, k, nnz, row_ptrs, col_indices, values, B, ldb, alpha, C, ldc, beta, out, ldo, st);
  } else if (dtype == TRNSPARSE_F64) {
    if (index_type == TRNSPARSE_I32) return launch_spmm<int32_t, double>(m, n, k, nnz, row_ptrs, col_indices, values, B, ldb, alpha, C, ldc, beta, out, ldo, st);
    if (index_type == TRNSPARSE_I64) return launch_spmm<int64_t, double>(m, n, k, nnz, row_ptrs, col_indices, values, B, ldb, alpha, C, ldc, beta, out, ldo, st);
  } else {
    return fail(TRNSPARSE_ERR_DTYPE, "csr_spmm: dtype %d not supported (F32, F64)", dtype);
  }
  return fail(TRNSPARSE_ERR_DTYPE, "csr_spmm: index type %d not supported (I32, I64)", index_type);
}

extern "C" int trnsparse_csr_sddmm(int64_t m, int64_t n, int64_t k, int64_t nnz, int index_type, int dtype,
                                   const void* row_ptrs, const void* col_indices, const void* G, int64_t ldg,
                                   const void* X, int64_t ldx, double alpha, void* out, void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && k >= 1 && nnz >= 0, "csr_sddmm: bad sizes");
  if (m == 0 || nnz == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(row_ptrs && col_indices && G && X && out, "csr_sddmm: null pointer");
  TSB_REQUIRE(ldg >= k && ldx >= k, "csr_sddmm: leading dimension smaller than k");
  cudaStream_t st = as_stream(stream);
  if (dtype == TRNSPARSE_F32) {
    if (index_type == TRNSPARSE_I32) return launch_sddmm<int32_t, float>(m, k, row_ptrs, col_indices, G, ldg, X, ldx, alpha, out, st);
    if (index_type == TRNSPARSE_I64) return launch_sddmm<int64_t, float>(m, k, row_ptrs, col_indices, G, ldg, X, ldx, alpha, out, st);
  } else if (dtype == TRNSPARSE_F64) {
    if (index_type == TRNSPARSE_I32) return launch_sddmm<int32_t, double>(m, k, row_ptrs, col_indices, G, ldg, X, ldx, alpha, out, st);
    if (index_type == TRNSPARSE_I64) return launch_sddmm<int64_t, double>(m, k, row_ptrs, col_indices, G, ldg, X, ldx, alpha, out, st);
  } else {
    return fail(TRNSPARSE_ERR_DTYPE, "csr_sddmm: dtype %d not supported (F32, F64)", dtype);
  }
  return fail(TRNSPARSE_ERR_DTYPE, "csr_sddmm: index type %d not supported (I32, I64)", index_type);
}
