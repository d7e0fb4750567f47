// Block-sparse attention forward on CUDA cores (trnsparse/ops.py:549-625,
// `block_sparse_attention_tiled`; the reference's two-pass PyTorch form is
// ops.py:280-357, its NKI kernels trnsparse/nki/kernels.py:157-293).
//
// Single pass with an online softmax instead of the reference's two passes
// (row max, then exp-sum, then weighted sum): per query row the running max
// m and denominator l are rescaled as new key blocks arrive, so every stored
// block is read once and scores are computed once. The result equals the
// reference's exp(s - rowmax) / max(rowsum, 1e-12) @ V up to rounding; rows of
// an empty block-row are zero (the reference's row_max = 0 / zero-output
// case). Only the mask's pattern (block_row_ptrs, block_col_indices) is used.
//
// One CTA handles 32 query rows of one head; 8 threads share a row: they
// split the 32 keys of a key chunk for the scores and the head dimension for
// the output. Scores, softmax state and the output accumulate in float32;
// inputs and output are float32 or bfloat16.
#include <cuda_bf16.h>

#include "common.cuh"

namespace tsb {
namespace {

constexpr int kAttnThreads = 256;
constexpr int kRows = 32;  // query rows per CTA
constexpr int kKeys = 32;  // keys per chunk

template <typename T> __device__ __forceinline__ float ld(const T* p);
template <> __device__ __forceinline__ float ld<float>(const float* p) { return __ldg(p); }
template <> __device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <typename T> __device__ __forceinline__ void st(T* p, float v);
template <> __device__ __forceinline__ void st<float>(float* p, float v) { *p = v; }
template <> __device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <typename T, int DPT>  // DPT: head-dim elements per thread (hd <= 8 * DPT)
__global__ void __launch_bounds__(kAttnThreads)
attn_simt_kernel(const T* __restrict__ Q, const T* __restrict__ K, const T* __restrict__ V, T* __restrict__ O,
                 const int* __restrict__ row_ptr, const int* __restrict__ col_idx, int seq, int hd, int b,
                 int m_tiles, int64_t head_stride, float scale) {
  extern __shared__ __align__(16) float sm_attn[];
  const int hdp = hd + 1;  // padded row stride
  float* Qs = sm_attn;                  // kRows x hdp
  float* Ks = Qs + kRows * hdp;         // kKeys x hdp
  float* Vs = Ks + kKeys * hdp;         // kKeys x hdp
  float* Ps = Vs + kKeys * hdp;         // kRows x (kKeys + 1)

  const int slices = (b + kRows - 1) / kRows;
  const int brow = blockIdx.x / slices;
  const int r0 = brow * b + (blockIdx.x % slices) * kRows;
  const int rend = min(brow * b + b, m_tiles * b);
  const int64_t hoff = static_cast<int64_t>(blockIdx.y) * head_stride;
  const T* Qh = Q + hoff;
  const T* Kh = K + hoff;
  const T* Vh = V + hoff;
  T* Oh = O + hoff;

  const int t = threadIdx.x, row = t >> 3, sub = t & 7;
  for (int i = t; i < kRows * hd; i += kAttnThreads) {
    const int rr = i / hd, d = i - rr * hd;
    Qs[rr * hdp + d] = (r0 + rr < rend) ? ld<T>(Qh + static_cast<int64_t>(r0 + rr) * hd + d) : 0.f;
  }
  float acc[DPT];
#pragma unroll
  for (int i = 0; i < DPT; ++i) acc[i] = 0.f;
  float mrow = -INFINITY, lrow = 0.f;
  const int e = row_ptr[brow + 1];
  for (int idx = row_ptr[brow]; idx < e; ++idx) {
    const int c = col_idx[idx];
    for (int k0 = 0; k0 < b; k0 += kKeys) {
      const int nk = min(kKeys, b - k0);
      __syncthreads();
      for (int i = t; i < kKeys * hd; i += kAttnThreads) {
        const int kk = i / hd, d = i - kk * hd;
        const int64_t key = static_cast<int64_t>(c) * b + k0 + kk;
        const bool in = kk < nk && key < seq;
        Ks[kk * hdp + d] = in ? ld<T>(Kh + key * hd + d) : 0.f;
        Vs[kk * hdp + d] = in ? ld<T>(Vh + key * hd + d) : 0.f;
      }
      __syncthreads();
      // scores of this thread's 4 keys
      float s[kKeys / 8];
      float cmax = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < kKeys / 8; ++jj) {
        const int j = sub + 8 * jj;
        float dot = 0.f;
        const float* qp = Qs + row * hdp;
        const float* kp = Ks + j * hdp;
        for (int d = 0; d < hd; ++d) dot = fmaf(qp[d], kp[d], dot);
        s[jj] = j < nk ? dot * scale : -INFINITY;
        cmax = fmaxf(cmax, s[jj]);
      }
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, o));
      const float mnew = fmaxf(mrow, cmax);
      const float corr = (mrow == -INFINITY) ? 0.f : expf(mrow - mnew);
      float psum = 0.f;
#pragma unroll
      for (int jj = 0; jj < kKeys / 8; ++jj) {
        const int j = sub + 8 * jj;
        const float p = (s[jj] == -INFINITY) ? 0.f : expf(s[jj] - mnew);
        Ps[row * (kKeys + 1) + j] = p;
        psum += p;
      }
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
      lrow = lrow * corr + psum;
      mrow = mnew;
      __syncwarp();
#pragma unroll
      for (int i = 0; i < DPT; ++i) {
        const int d = sub + 8 * i;
        float a = acc[i] * corr;
        if (d < hd) {
          for (int j = 0; j < nk; ++j) a = fmaf(Ps[row * (kKeys + 1) + j], Vs[j * hdp + d], a);
        }
        acc[i] = a;
      }
    }
  }
  const int r = r0 + row;
  if (r < rend) {
    const float inv = (e > row_ptr[brow]) ? 1.f / fmaxf(lrow, 1e-12f) : 0.f;
#pragma unroll
    for (int i = 0; i < DPT; ++i) {
      const int d = sub + 8 * i;
      if (d < hd) st<T>(Oh + static_cast<int64_t>(r) * hd + d, (e > row_ptr[brow]) ? acc[i] * inv : 0.f);
    }
  }
}

template <typename T, int DPT>
int launch_attn(const void* Q, const void* K, const void* V, void* O, const int* rp, const int* ci, int seq, int hd,
                int b, int heads, int64_t head_stride, float scale, cudaStream_t st) {
  const int m_tiles = seq / b;
  const size_t smem = sizeof(float) * (size_t)((kRows + 2 * kKeys) * (hd + 1) + kRows * (kKeys + 1));
  auto kern = attn_simt_kernel<T, DPT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_status(e, "attention: set smem");
  const int slices = (b + kRows - 1) / kRows;
  dim3 grid((unsigned)(m_tiles * slices), (unsigned)heads);
  if (m_tiles > 0)
    kern<<<grid, kAttnThreads, smem, st>>>((const T*)Q, (const T*)K, (const T*)V, (T*)O, rp, ci, seq, hd, b, m_tiles,
                                           head_stride, scale);
  TSB_CHECK_LAUNCH("attention launch");
  return TRNSPARSE_OK;
}

template <typename T>
int dispatch_attn(const void* Q, const void* K, const void* V, void* O, const int* rp, const int* ci, int seq, int hd,
                  int b, int heads, int64_t hs, float scale, cudaStream_t st) {
  if (hd <= 64) return launch_attn<T, 8>(Q, K, V, O, rp, ci, seq, hd, b, heads, hs, scale, st);
  if (hd <= 128) return launch_attn<T, 16>(Q, K, V, O, rp, ci, seq, hd, b, heads, hs, scale, st);
  if (hd <= 256) return launch_attn<T, 32>(Q, K, V, O, rp, ci, seq, hd, b, heads, hs, scale, st);
  return fail(TRNSPARSE_ERR_UNSUPPORTED, "attention: head_dim %d > 256", hd);
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" int trnsparse_bsr_attention(int64_t heads, int64_t seq, int64_t head_dim, int block_size,
                                       const int* block_row_ptr, const int* block_col_idx, const void* Q,
                                       const void* K, const void* V, void* O, int dtype, double scale,
                                       void* stream) {
  TSB_REQUIRE(heads >= 0 && seq >= 0 && head_dim > 0 && block_size > 0, "attention: bad sizes");
  TSB_REQUIRE(seq < (1ll << 31) && heads < 65536, "attention: sizes out of range");
  if (heads == 0 || seq == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(Q && K && V && O && block_row_ptr && block_col_idx, "attention: null pointer");
  cudaStream_t st = as_stream(stream);
  const int64_t m_tiles = seq / block_size;
  if (seq % block_size) {
    // rows past the last whole block are not covered by the mask: zero, as in the reference
    const size_t es = dtype == TRNSPARSE_F32 ? 4 : 2;
    for (int64_t h = 0; h < heads; ++h) {
      char* base = static_cast<char*>(O) + es * (size_t)(h * seq * head_dim + m_tiles * block_size * head_dim);
      cudaError_t e = cudaMemsetAsync(base, 0, es * (size_t)((seq - m_tiles * block_size) * head_dim), st);
      if (e != cudaSuccess) return cuda_status(e, "attention: zero tail");
    }
  }
  const int64_t hs = seq * head_dim;
  if (dtype == TRNSPARSE_F32)
    return dispatch_attn<float>(Q, K, V, O, block_row_ptr, block_col_idx, (int)seq, (int)head_dim, block_size,
                                (int)heads, hs, (float)scale, st);
  if (dtype == TRNSPARSE_BF16)
    return dispatch_attn<__nv_bfloat16>(Q, K, V, O, block_row_ptr, block_col_idx, (int)seq, (int)head_dim,
                                        block_size, (int)heads, hs, (float)scale, st);
  return fail(TRNSPARSE_ERR_DTYPE, "attention: dtype %d not supported (F32, BF16)", dtype);
}
