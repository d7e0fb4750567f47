// Helpers shared by the tensor-core kernels (bsr_spmm_tc.cu, screened_tc.cu):
// fire-and-forget global reductions, the tf32 split, the B -> K-major B^T
// prep kernel, tensor-map encoding and an opt-in debug synchronisation.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <stdlib.h>

#include <utility>

#include "common.cuh"
#include "tc.cuh"

namespace tsb {
namespace {

// TRNSPARSE_DEBUG_SYNC=1: synchronise after each launch and name the step that failed.
inline int debug_sync(cudaStream_t st, const char* step) {
  static const int on = [] {
    const char* v = getenv("TRNSPARSE_DEBUG_SYNC");
    return (v && *v == '1') ? 1 : 0;
  }();
  if (!on) return TRNSPARSE_OK;
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cuda_status(e, step);
  return TRNSPARSE_OK;
}

// Fire-and-forget float adds into global memory (no returned value to wait on).
__device__ __forceinline__ void red_add_v4(float* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(p), "f"(__uint_as_float(a)),
               "f"(__uint_as_float(b)), "f"(__uint_as_float(c)), "f"(__uint_as_float(d))
               : "memory");
}
__device__ __forceinline__ void red_add(float* p, uint32_t a) {
  asm volatile("red.global.add.f32 [%0], %1;\n" ::"l"(p), "f"(__uint_as_float(a)) : "memory");
}

// Two floats -> one 32-bit word of bf16 (round to nearest even), a in the low half.
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// ---------------------------------------------------------------- prep kernels
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__global__ void split_tf32_kernel(int64_t n, const float* __restrict__ src, float* __restrict__ hi,
                                  float* __restrict__ lo) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float x = src[i];
    if (hi != nullptr) {
      const float h = tf32_rna(x);
      hi[i] = h;
      lo[i] = tf32_rna(x - h);
    } else {
      // src itself is the hi operand: a kind::tf32 MMA reads an fp32 operand's sign,
      // exponent and top 10 mantissa bits, so the part it drops is x minus x with its
      // low 13 bits cleared (exact in fp32)
      lo[i] = tf32_rna(x - __uint_as_float(__float_as_uint(x) & 0xffffe000u));
    }
  }
}

// Bt[kk][nn] = B[nn][kk] for nn < n, 0 for n <= nn < n_pad (32x32 smem tiles).
// SPLIT (fp32): writes the tf32 hi/lo split; otherwise a plain bf16 transpose.
template <bool SPLIT, typename E>
__global__ void transpose_b_kernel(int64_t n, int64_t k, const E* __restrict__ B, int64_t ldb, int64_t n_pad,
                                   E* __restrict__ hi, E* __restrict__ lo) {
  __shared__ float tile[32][33];
  grid_dep_launch();  // the tensor-core kernel after it may start its set-up now
  const int64_t nb = static_cast<int64_t>(blockIdx.x) * 32, kb = static_cast<int64_t>(blockIdx.y) * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t nn = nb + r, kk = kb + threadIdx.x;
    float v = 0.f;
    if (nn < n && kk < k) {
      if constexpr (sizeof(E) == 4) v = B[nn * ldb + kk];
      else v = __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(B + nn * ldb + kk));
    }
    tile[r][threadIdx.x] = v;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int64_t kk = kb + r, nn = nb + threadIdx.x;
    if (kk < k && nn < n_pad) {
      const float v = tile[threadIdx.x][r];
      if constexpr (SPLIT) {
        const float h = tf32_rna(v);
        hi[kk * n_pad + nn] = h;
        lo[kk * n_pad + nn] = tf32_rna(v - h);
      } else {
        *reinterpret_cast<__nv_bfloat16*>(hi + kk * n_pad + nn) = __float2bfloat16_rn(v);
      }
    }
  }
}

inline size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// Launches `kern` with programmatic stream serialization (the kernel calls
// grid_dep_wait() before touching memory the previous kernel writes), so its
// launch latency and set-up overlap the previous kernel's tail.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t cols, uint64_t rows,
                 uint64_t row_bytes, uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return fail(TRNSPARSE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (row_bytes & 15u))
    return fail(TRNSPARSE_ERR_ALIGN, "tensor map: base/stride not 16-byte aligned");
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TRNSPARSE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return TRNSPARSE_OK;
}

}  // namespace
}  // namespace tsb
