// Block-sparse attention backward on CUDA cores: the reference's
// _block_sparse_attn_backward (trnsparse/ops.py:360-473; NKI counterparts
// _attn_bwd_dq_kernel / _attn_bwd_dkdv_kernel, trnsparse/nki/kernels.py:
// 295-524). Flash-delta identity: with D_i = dO_i . O_i and the softmax
// weights P = exp(s - rowmax) / rowsum recomputed from Q and K,
//   dS = P (dP - D),  dP = dO V^T,
//   dQ += dS K scale,  dK += dS^T Q scale,  dV += P^T dO,
// over the stored blocks only. Three launches:
//   attn_bwd_stats_kernel   per query row: rowmax, rowsum (clamped at 1e-12,
//                           as the reference) and D; one pass with an online
//                           max/sum over the row's stored blocks.
//   attn_bwd_dq_kernel      row-first: a CTA owns 32 query rows of a head and
//                           walks their stored key blocks.
//   attn_bwd_dkdv_kernel    column-first: a CTA owns 32 key rows of a head and
//                           walks (up to 8 of) the query blocks that store its
//                           key block (the mask's transposed pattern,
//                           col_ptr/row_idx); key blocks stored by more query
//                           blocks (global tokens) are split over several
//                           CTAs that add into fp32 accumulators.
// Rows of empty block-rows and rows past the last whole block get no
// gradient (the reference's loops skip them). 8 threads share a row: they
// split the 32 keys (or queries) of a chunk for the scores and the head
// dimension for the accumulators. fp32 arithmetic, fp32 or bf16 I/O.
#include <cuda_bf16.h>

#include "common.cuh"

namespace tsb {
namespace {

constexpr int kBwThreads = 256;
constexpr int kBwRows = 32;  // rows owned per CTA
constexpr int kBwKeys = 32;  // partner rows per chunk
constexpr int kBwPerPart = 8;  // query blocks per dK/dV CTA before a key block is split

template <typename T> __device__ __forceinline__ float bw_ld(const T* p);
template <> __device__ __forceinline__ float bw_ld<float>(const float* p) { return __ldg(p); }
template <> __device__ __forceinline__ float bw_ld<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <typename T> __device__ __forceinline__ void bw_st(T* p, float v);
template <> __device__ __forceinline__ void bw_st<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void bw_st<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}

// rows [r0, r0 + 32) of a (seq, hd) head slice into a padded shared tile (zeros outside [lo, hi))
template <typename T>
__device__ __forceinline__ void load_rows(float* dst, const T* src, int64_t r0, int64_t lo, int64_t hi, int hd) {
  const int hdp = hd + 1;
  for (int i = threadIdx.x; i < kBwRows * hd; i += kBwThreads) {
    const int rr = i / hd, d = i - rr * hd;
    const int64_t r = r0 + rr;
    dst[rr * hdp + d] = (r >= lo && r < hi) ? bw_ld<T>(src + r * hd + d) : 0.f;
  }
}

// out[jj] = a . b[(sub + 8 jj) * hdp ...], jj < 4: one load of a per four products
__device__ __forceinline__ void dot4(const float* a, const float* b, int sub, int hdp, int hd, float (&out)[4]) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  const float* b0 = b + sub * hdp;
  for (int d = 0; d < hd; ++d) {
    const float x = a[d];
    s0 = fmaf(x, b0[d], s0);
    s1 = fmaf(x, b0[8 * hdp + d], s1);
    s2 = fmaf(x, b0[16 * hdp + d], s2);
    s3 = fmaf(x, b0[24 * hdp + d], s3);
  }
  out[0] = s0;
  out[1] = s1;
  out[2] = s2;
  out[3] = s3;
}

// two rows against the same four partner rows of two tiles: (a . b_j, c . e_j)
__device__ __forceinline__ void dot4x2(const float* a, const float* b, const float* c, const float* e, int sub,
                                       int hdp, int hd, float (&ab)[4], float (&ce)[4]) {
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f, t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
  const float* b0 = b + sub * hdp;
  const float* e0 = e + sub * hdp;
  for (int d = 0; d < hd; ++d) {
    const float x = a[d], y = c[d];
    s0 = fmaf(x, b0[d], s0);
    s1 = fmaf(x, b0[8 * hdp + d], s1);
    s2 = fmaf(x, b0[16 * hdp + d], s2);
    s3 = fmaf(x, b0[24 * hdp + d], s3);
    t0 = fmaf(y, e0[d], t0);
    t1 = fmaf(y, e0[8 * hdp + d], t1);
    t2 = fmaf(y, e0[16 * hdp + d], t2);
    t3 = fmaf(y, e0[24 * hdp + d], t3);
  }
  ab[0] = s0;
  ab[1] = s1;
  ab[2] = s2;
  ab[3] = s3;
  ce[0] = t0;
  ce[1] = t1;
  ce[2] = t2;
  ce[3] = t3;
}

// ---------------------------------------------------------------- stats: rowmax, rowsum, D
template <typename T>
__global__ void __launch_bounds__(kBwThreads)
attn_bwd_stats_kernel(const T* __restrict__ Q, const T* __restrict__ K, const T* __restrict__ O,
                      const T* __restrict__ dO, const int* __restrict__ row_ptr, const int* __restrict__ col_idx,
                      int seq, int hd, int b, int m_tiles, float scale, float* __restrict__ st_max,
                      float* __restrict__ st_sum, float* __restrict__ st_d) {
  extern __shared__ __align__(16) float sm_bw[];
  const int hdp = hd + 1;
  float* Qs = sm_bw;
  float* Ks = Qs + kBwRows * hdp;
  const int slices = (b + kBwRows - 1) / kBwRows;
  const int brow = blockIdx.x / slices;
  const int64_t r0 = static_cast<int64_t>(brow) * b + (blockIdx.x % slices) * kBwRows;
  const int64_t rend = min(static_cast<int64_t>(brow) * b + b, static_cast<int64_t>(m_tiles) * b);
  const int64_t hoff = static_cast<int64_t>(blockIdx.y) * seq * hd;
  const int t = threadIdx.x, row = t >> 3, sub = t & 7;
  load_rows<T>(Qs, Q + hoff, r0, r0, rend, hd);
  float mrow = -INFINITY, lrow = 0.f;
  const int e0 = row_ptr[brow], e1 = row_ptr[brow + 1];
  for (int idx = e0; idx < e1; ++idx) {
    const int64_t c = col_idx[idx];
    for (int k0 = 0; k0 < b; k0 += kBwKeys) {
      const int nk = min(kBwKeys, b - k0);
      __syncthreads();
      load_rows<T>(Ks, K + hoff, c * b + k0, c * b + k0, min(c * b + k0 + nk, static_cast<int64_t>(seq)), hd);
      __syncthreads();
      float s[kBwKeys / 8];
      dot4(Qs + row * hdp, Ks, sub, hdp, hd, s);
      float cmax = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < kBwKeys / 8; ++jj) {
        const int j = sub + 8 * jj;
        s[jj] = j < nk ? s[jj] * scale : -INFINITY;
        cmax = fmaxf(cmax, s[jj]);
      }
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, o));
      const float mnew = fmaxf(mrow, cmax);
      float ps = 0.f;
#pragma unroll
      for (int jj = 0; jj < kBwKeys / 8; ++jj) ps += s[jj] == -INFINITY ? 0.f : expf(s[jj] - mnew);
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      lrow = (mrow == -INFINITY ? 0.f : lrow * expf(mrow - mnew)) + ps;
      mrow = mnew;
    }
  }
  // D = dO . O over the head dimension, split across the row's 8 threads
  const int64_t r = r0 + row;
  float dd = 0.f;
  if (r < rend)
    for (int d = sub; d < hd; d += 8) dd = fmaf(bw_ld<T>(dO + hoff + r * hd + d), bw_ld<T>(O + hoff + r * hd + d), dd);
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) dd += __shfl_xor_sync(0xffffffffu, dd, o);
  if (sub == 0 && r < rend) {
    const int64_t gi = static_cast<int64_t>(blockIdx.y) * seq + r;
    st_max[gi] = e1 > e0 ? mrow : 0.f;
    st_sum[gi] = fmaxf(lrow, 1e-12f);
    st_d[gi] = dd;
  }
}

// ---------------------------------------------------------------- dQ (row-first)
template <typename T, int DPT>
__global__ void __launch_bounds__(kBwThreads)
attn_bwd_dq_kernel(const T* __restrict__ Q, const T* __restrict__ K, const T* __restrict__ V,
                   const T* __restrict__ dO, const int* __restrict__ row_ptr, const int* __restrict__ col_idx,
                   int seq, int hd, int b, int m_tiles, float scale, const float* __restrict__ st_max,
                   const float* __restrict__ st_sum, const float* __restrict__ st_d, T* __restrict__ dQ) {
  extern __shared__ __align__(16) float sm_bw[];
  const int hdp = hd + 1;
  float* Qs = sm_bw;
  float* dOs = Qs + kBwRows * hdp;
  float* Ks = dOs + kBwRows * hdp;
  float* Vs = Ks + kBwKeys * hdp;
  float* dSs = Vs + kBwKeys * hdp;  // kBwRows x (kBwKeys + 1)
  const int slices = (b + kBwRows - 1) / kBwRows;
  const int brow = blockIdx.x / slices;
  const int64_t r0 = static_cast<int64_t>(brow) * b + (blockIdx.x % slices) * kBwRows;
  const int64_t rend = min(static_cast<int64_t>(brow) * b + b, static_cast<int64_t>(m_tiles) * b);
  const int64_t hoff = static_cast<int64_t>(blockIdx.y) * seq * hd;
  const int t = threadIdx.x, row = t >> 3, sub = t & 7;
  load_rows<T>(Qs, Q + hoff, r0, r0, rend, hd);
  load_rows<T>(dOs, dO + hoff, r0, r0, rend, hd);
  const int64_t r = r0 + row;
  const int64_t gi = static_cast<int64_t>(blockIdx.y) * seq + r;
  const bool live = r < rend;
  const float mr = live ? st_max[gi] : 0.f, lr = live ? st_sum[gi] : 1.f, dr = live ? st_d[gi] : 0.f;
  float acc[DPT];
#pragma unroll
  for (int i = 0; i < DPT; ++i) acc[i] = 0.f;
  const int e1 = row_ptr[brow + 1];
  for (int idx = row_ptr[brow]; idx < e1; ++idx) {
    const int64_t c = col_idx[idx];
    for (int k0 = 0; k0 < b; k0 += kBwKeys) {
      const int nk = min(kBwKeys, b - k0);
      const int64_t kend = min(c * b + k0 + nk, static_cast<int64_t>(seq));
      __syncthreads();
      load_rows<T>(Ks, K + hoff, c * b + k0, c * b + k0, kend, hd);
      load_rows<T>(Vs, V + hoff, c * b + k0, c * b + k0, kend, hd);
      __syncthreads();
      float sc[4], dp[4];
      dot4x2(Qs + row * hdp, Ks, dOs + row * hdp, Vs, sub, hdp, hd, sc, dp);
#pragma unroll
      for (int jj = 0; jj < kBwKeys / 8; ++jj) {
        const int j = sub + 8 * jj;
        float ds = 0.f;
        if (live && j < nk) {
          const float p = expf(sc[jj] * scale - mr) / lr;
          ds = p * (dp[jj] - dr);
        }
        dSs[row * (kBwKeys + 1) + j] = ds;
      }
      __syncwarp();
      // acc[i] += sum_j dS[row][j] K[j][sub + 8 i], j ascending
      for (int j = 0; j < nk; ++j) {
        const float ds = dSs[row * (kBwKeys + 1) + j];
        const float* kr = Ks + j * hdp + sub;
#pragma unroll
        for (int i = 0; i < DPT; ++i)
          if (sub + 8 * i < hd) acc[i] = fmaf(ds, kr[8 * i], acc[i]);
      }
    }
  }
  if (live) {
#pragma unroll
    for (int i = 0; i < DPT; ++i) {
      const int d = sub + 8 * i;
      if (d < hd) bw_st<T>(dQ + hoff + r * hd + d, acc[i] * scale);
    }
  }
}

// ---------------------------------------------------------------- dK, dV (column-first)
template <typename T, int DPT>
__global__ void __launch_bounds__(kBwThreads)
attn_bwd_dkdv_kernel(const T* __restrict__ Q, const T* __restrict__ K, const T* __restrict__ V,
                     const T* __restrict__ dO, const int* __restrict__ col_ptr, const int* __restrict__ row_idx,
                     int seq, int hd, int b, int m_tiles, int parts, int per_part, float scale,
                     const float* __restrict__ st_max, const float* __restrict__ st_sum,
                     const float* __restrict__ st_d, T* __restrict__ dK, T* __restrict__ dV,
                     float* __restrict__ dK32, float* __restrict__ dV32) {
  extern __shared__ __align__(16) float sm_bw[];
  __shared__ float qm[kBwKeys], ql[kBwKeys], qd[kBwKeys];
  const int hdp = hd + 1;
  float* Ks = sm_bw;
  float* Vs = Ks + kBwRows * hdp;
  float* Qs = Vs + kBwRows * hdp;
  float* dOs = Qs + kBwKeys * hdp;
  float* Ps = dOs + kBwKeys * hdp;          // kBwRows x (kBwKeys + 1)
  float* dSs = Ps + kBwRows * (kBwKeys + 1);
  // CTA = (key block, 32-row slice of it, part of the query blocks that store it): a key
  // block stored by many query blocks (a global-token column) is spread over several CTAs
  const int slices = (b + kBwRows - 1) / kBwRows;
  const int bcol = blockIdx.x / (slices * parts);
  const int rem = blockIdx.x - bcol * slices * parts;
  const int slice = rem / parts, part = rem - slice * parts;
  const int q_begin = col_ptr[bcol] + part * per_part;
  const int e1 = min(q_begin + per_part, col_ptr[bcol + 1]);
  if (q_begin >= e1) return;
  const int64_t k0row = static_cast<int64_t>(bcol) * b + slice * kBwRows;
  const int64_t kend = min(static_cast<int64_t>(bcol) * b + b, static_cast<int64_t>(seq));
  const int64_t hoff = static_cast<int64_t>(blockIdx.y) * seq * hd;
  const int t = threadIdx.x, krow = t >> 3, sub = t & 7;
  load_rows<T>(Ks, K + hoff, k0row, k0row, kend, hd);
  load_rows<T>(Vs, V + hoff, k0row, k0row, kend, hd);
  const bool live = k0row + krow < kend;
  float ak[DPT], av[DPT];
#pragma unroll
  for (int i = 0; i < DPT; ++i) ak[i] = av[i] = 0.f;
  for (int idx = q_begin; idx < e1; ++idx) {
    const int64_t m = row_idx[idx];  // a query block storing this key block
    if (m >= m_tiles) continue;
    for (int q0 = 0; q0 < b; q0 += kBwKeys) {
      const int nq = min(kBwKeys, b - q0);
      const int64_t qa = m * b + q0;
      __syncthreads();
      load_rows<T>(Qs, Q + hoff, qa, qa, qa + nq, hd);
      load_rows<T>(dOs, dO + hoff, qa, qa, qa + nq, hd);
      if (t < kBwKeys) {
        const int64_t gi = static_cast<int64_t>(blockIdx.y) * seq + qa + t;
        const bool ok = t < nq;
        qm[t] = ok ? st_max[gi] : 0.f;
        ql[t] = ok ? st_sum[gi] : 1.f;
        qd[t] = ok ? st_d[gi] : 0.f;
      }
      __syncthreads();
      float sc[4], dpv[4];
      dot4x2(Ks + krow * hdp, Qs, Vs + krow * hdp, dOs, sub, hdp, hd, sc, dpv);
#pragma unroll
      for (int jj = 0; jj < kBwKeys / 8; ++jj) {
        const int q = sub + 8 * jj;
        float p = 0.f, ds = 0.f;
        if (live && q < nq) {
          p = expf(sc[jj] * scale - qm[q]) / ql[q];
          ds = p * (dpv[jj] - qd[q]);
        }
        Ps[krow * (kBwKeys + 1) + q] = p;
        dSs[krow * (kBwKeys + 1) + q] = ds;
      }
      __syncwarp();
      // ak[i] += sum_q dS[k][q] Q[q][d_i], av[i] += sum_q P[k][q] dO[q][d_i], q ascending
      for (int q = 0; q < nq; ++q) {
        const float ds = dSs[krow * (kBwKeys + 1) + q], p = Ps[krow * (kBwKeys + 1) + q];
        const float* qr = Qs + q * hdp + sub;
        const float* orr = dOs + q * hdp + sub;
#pragma unroll
        for (int i = 0; i < DPT; ++i) {
          if (sub + 8 * i < hd) {
            ak[i] = fmaf(ds, qr[8 * i], ak[i]);
            av[i] = fmaf(p, orr[8 * i], av[i]);
          }
        }
      }
    }
  }
  if (live) {
    const int64_t r = k0row + krow;
#pragma unroll
    for (int i = 0; i < DPT; ++i) {
      const int d = sub + 8 * i;
      if (d < hd) {
        if (parts == 1) {
          bw_st<T>(dK + hoff + r * hd + d, ak[i] * scale);
          bw_st<T>(dV + hoff + r * hd + d, av[i]);
        } else {  // partial sums of a split key block: fp32 accumulators
          atomicAdd(dK32 + hoff + r * hd + d, ak[i] * scale);
          atomicAdd(dV32 + hoff + r * hd + d, av[i]);
        }
      }
    }
  }
}

template <typename T>
__global__ void attn_bwd_finish_kernel(int64_t n, const float* __restrict__ a32, const float* __restrict__ b32,
                                       T* __restrict__ a, T* __restrict__ b) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    bw_st<T>(a + i, a32[i]);
    bw_st<T>(b + i, b32[i]);
  }
}

template <typename T, int DPT>
int launch_attn_bwd(int heads, int seq, int hd, int b, const int* rp, const int* ci, const int* cp, const int* ri,
                    int parts, int per_part, const void* Q, const void* K, const void* V, const void* O,
                    const void* dO, void* dQ, void* dK, void* dV, float scale, float* ws, cudaStream_t st) {
  const int m_tiles = seq / b;
  const int n_kb = (seq + b - 1) / b;
  const int slices = (b + kBwRows - 1) / kBwRows;
  const size_t hdp = (size_t)hd + 1;
  float* smax = ws;
  float* ssum = ws + (size_t)heads * seq;
  float* sd = ws + 2 * (size_t)heads * seq;
  const size_t sm_stats = sizeof(float) * 2 * kBwRows * hdp;
  const size_t sm_dq = sizeof(float) * (4 * kBwRows * hdp + kBwRows * (kBwKeys + 1));
  const size_t sm_kv = sizeof(float) * (4 * kBwRows * hdp + 2 * kBwRows * (kBwKeys + 1));
  auto k_st = attn_bwd_stats_kernel<T>;
  auto k_dq = attn_bwd_dq_kernel<T, DPT>;
  auto k_kv = attn_bwd_dkdv_kernel<T, DPT>;
  cudaError_t e = cudaFuncSetAttribute(k_st, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_stats);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_dq, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_dq);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_kv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm_kv);
  if (e != cudaSuccess) return cuda_status(e, "attention_backward: set smem");
  if (m_tiles > 0) {
    dim3 g((unsigned)(m_tiles * slices), (unsigned)heads);
    k_st<<<g, kBwThreads, sm_stats, st>>>((const T*)Q, (const T*)K, (const T*)O, (const T*)dO, rp, ci, seq, hd, b,
                                          m_tiles, scale, smax, ssum, sd);
    TSB_CHECK_LAUNCH("attention_backward: stats");
    k_dq<<<g, kBwThreads, sm_dq, st>>>((const T*)Q, (const T*)K, (const T*)V, (const T*)dO, rp, ci, seq, hd, b,
                                       m_tiles, scale, smax, ssum, sd, (T*)dQ);
    TSB_CHECK_LAUNCH("attention_backward: dQ");
  }
  if (n_kb > 0) {
    const size_t n = (size_t)heads * seq * hd;
    // split key blocks accumulate in fp32: the outputs themselves for fp32, else workspace
    float* a32 = nullptr;
    float* b32 = nullptr;
    if (parts > 1) {
      if (sizeof(T) == 4) {
        a32 = static_cast<float*>(dK);
        b32 = static_cast<float*>(dV);
      } else {
        a32 = ws + 3 * (size_t)heads * seq;
        b32 = a32 + n;
        cudaError_t e2 = cudaMemsetAsync(a32, 0, 2 * n * sizeof(float), st);
        if (e2 != cudaSuccess) return cuda_status(e2, "attention_backward: zero accumulators");
      }
    }
    dim3 g((unsigned)(n_kb * slices * parts), (unsigned)heads);
    k_kv<<<g, kBwThreads, sm_kv, st>>>((const T*)Q, (const T*)K, (const T*)V, (const T*)dO, cp, ri, seq, hd, b,
                                       m_tiles, parts, per_part, scale, smax, ssum, sd, (T*)dK, (T*)dV, a32, b32);
    TSB_CHECK_LAUNCH("attention_backward: dK dV");
    if (parts > 1 && sizeof(T) != 4) {
      int64_t gr = (int64_t)(n + 255) / 256;
      if (gr > 8 * sm_count()) gr = 8 * sm_count();
      attn_bwd_finish_kernel<T><<<(unsigned)gr, 256, 0, st>>>((int64_t)n, a32, b32, (T*)dK, (T*)dV);
      TSB_CHECK_LAUNCH("attention_backward: finish");
    }
  }
  return TRNSPARSE_OK;
}

template <typename T>
int dispatch_attn_bwd(int heads, int seq, int hd, int b, const int* rp, const int* ci, const int* cp,
                      const int* ri, int parts, int per_part, const void* Q, const void* K, const void* V,
                      const void* O, const void* dO, void* dQ, void* dK, void* dV, float scale, float* ws,
                      cudaStream_t st) {
  if (hd <= 64)
    return launch_attn_bwd<T, 8>(heads, seq, hd, b, rp, ci, cp, ri, parts, per_part, Q, K, V, O, dO, dQ, dK, dV,
                                 scale, ws, st);
  if (hd <= 128)
    return launch_attn_bwd<T, 16>(heads, seq, hd, b, rp, ci, cp, ri, parts, per_part, Q, K, V, O, dO, dQ, dK, dV,
                                  scale, ws, st);
  return fail(TRNSPARSE_ERR_UNSUPPORTED, "attention_backward: head_dim %d > 128", hd);
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" size_t trnsparse_bsr_attention_backward_workspace_size(int64_t heads, int64_t seq, int64_t head_dim,
                                                                 int dtype, int max_col_blocks) {
  if (heads < 0 || seq < 0 || head_dim < 0) return 0;
  size_t bytes = 3 * sizeof(float) * (size_t)heads * (size_t)seq;
  if (dtype != TRNSPARSE_F32 && max_col_blocks > kBwPerPart)  // fp32 accumulators of split key blocks
    bytes += 2 * sizeof(float) * (size_t)heads * (size_t)seq * (size_t)head_dim;
  return bytes;
}

extern "C" int trnsparse_bsr_attention_backward(int64_t heads, int64_t seq, int64_t head_dim, int block_size,
                                                const int* block_row_ptr, const int* block_col_idx,
                                                const int* block_col_ptr, const int* block_row_idx,
                                                int max_col_blocks, const void* Q, const void* K, const void* V,
                                                const void* O, const void* dO, void* dQ, void* dK, void* dV,
                                                int dtype, double scale, void* ws, size_t ws_bytes, void* stream) {
  TSB_REQUIRE(heads >= 0 && seq >= 0 && head_dim > 0 && block_size > 0, "attention_backward: bad sizes");
  TSB_REQUIRE(seq < (1ll << 31) && heads < 65536, "attention_backward: sizes out of range");
  if (heads == 0 || seq == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(Q && K && V && O && dO && dQ && dK && dV && block_row_ptr && block_col_idx && block_col_ptr &&
                  block_row_idx && ws,
              "attention_backward: null pointer");
  TSB_REQUIRE(max_col_blocks >= 0, "attention_backward: bad max_col_blocks");
  TSB_REQUIRE(ws_bytes >= trnsparse_bsr_attention_backward_workspace_size(heads, seq, head_dim, dtype, max_col_blocks),
              "attention_backward: workspace too small");
  const int parts = max_col_blocks > kBwPerPart ? (max_col_blocks + kBwPerPart - 1) / kBwPerPart : 1;
  const int per_part = parts > 1 ? kBwPerPart : (max_col_blocks > 0 ? max_col_blocks : 1);
  cudaStream_t st = as_stream(stream);
  // rows that receive no gradient from the loops are zero (the reference's torch.zeros_like)
  const size_t es = dtype == TRNSPARSE_F32 ? 4 : 2;
  const size_t total = es * (size_t)heads * (size_t)seq * (size_t)head_dim;
  cudaError_t e = cudaMemsetAsync(dQ, 0, total, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(dK, 0, total, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(dV, 0, total, st);
  if (e != cudaSuccess) return cuda_status(e, "attention_backward: zero gradients");
  float* w = static_cast<float*>(ws);
  if (dtype == TRNSPARSE_F32)
    return dispatch_attn_bwd<float>((int)heads, (int)seq, (int)head_dim, block_size, block_row_ptr, block_col_idx,
                                    block_col_ptr, block_row_idx, parts, per_part, Q, K, V, O, dO, dQ, dK, dV,
                                    (float)scale, w, st);
  if (dtype == TRNSPARSE_BF16)
    return dispatch_attn_bwd<__nv_bfloat16>((int)heads, (int)seq, (int)head_dim, block_size, block_row_ptr,
                                            block_col_idx, block_col_ptr, block_row_idx, parts, per_part, Q, K, V, O,
                                            dO, dQ, dK, dV, (float)scale, w, st);
  return fail(TRNSPARSE_ERR_DTYPE, "attention_backward: dtype %d not supported (F32, BF16)", dtype);
}
