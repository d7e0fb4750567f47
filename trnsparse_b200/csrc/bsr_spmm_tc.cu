// BSR x dense on the 5th-generation tensor cores (tcgen05 + TMA + TMEM).
//
// Computes C = A @ B for a BSR A with 128x128 blocks (trnsparse/ops.py:162-210,
// the reference's `bsr_spmm`, accelerated there by nki_bsr_spmm,
// trnsparse/nki/dispatch.py:193-381). Each stored block is a dense
// 128x128 contraction against a 128-row slice of B.
//
// Work decomposition: a work unit is (block-row, contiguous run of that
// row's stored blocks); the grid is units x N-tiles of BN columns. A CTA
// (4 warps) streams its unit's blocks in 128-byte-wide K chunks: warp 0
// issues TMA loads of the A and B^T chunks into a ring of shared-memory
// stages, warp 1 issues tcgen05.mma into a 128 x BN fp32 accumulator in
// TMEM, and all four warps drain TMEM with tcgen05.ld and add the tile into
// C (red.global.add.v4 reductions; C is zeroed first, so units that split a block-row
// combine). No host-side gather or K_max padding of B (the reference's NKI
// path materialises B once per block).
//
// fp32 inputs use 3xTF32: every operand x is split into hi = tf32(x) and
// lo = tf32(x - hi) and the product accumulates hi*hi + hi*lo + lo*hi, which
// keeps the result within ~1e-6 relative error of fp32. A's split is done once
// per matrix (trnsparse_bsr_split_tf32, cached with the device layout); B's
// split and transpose to K-major B^T run per call into the workspace.
// bf16 inputs use kind::f16 with bf16 operands and fp32 accumulation.
//
// Dynamic shared memory is only guaranteed 16-byte alignment (on this part it
// starts 16 bytes into the window), so it is declared 16-byte aligned and the
// 1024-byte alignment the 128-byte-swizzled TMA tiles need is done by hand; an
// over-aligned declaration would let the compiler fold that round-up away.
#include "tc_common.cuh"

namespace tsb {
namespace {

constexpr int kTcThreads = 128;
constexpr int kSmemBudget = 200 * 1024;

#ifdef TSB_TC_TRACE
__device__ unsigned long long g_tc_trace[1024][8];
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
#define TC_TRACE(slot) g_tc_trace[(blockIdx.x + blockIdx.y * gridDim.x) & 1023][slot] = gtime()
#else
#define TC_TRACE(slot)
#endif

template <MmaKind KIND>
struct TcCfg {
  static constexpr int kElem = KIND == MmaKind::TF32 ? 4 : 2;
  static constexpr int kChunk = 128 / kElem;            // K elements per 128-byte chunk
  static constexpr int kChunksPerBlock = 128 / kChunk;  // chunks per 128-wide block
  static constexpr int kUmmaK = 32 / kElem;             // K per MMA instruction
  static constexpr int kSteps = kChunk / kUmmaK;        // MMAs per chunk per product
  static constexpr int kParts = KIND == MmaKind::TF32 ? 2 : 1;  // hi (+ lo) tiles per operand
};

template <MmaKind KIND, int BN>
struct TcLayout {
  static constexpr int kATile = 128 * 128;  // bytes
  static constexpr int kBTile = BN * 128;
  static constexpr int kStage = TcCfg<KIND>::kParts * (kATile + kBTile);
  static constexpr int kStages = kSmemBudget / kStage;
  static constexpr int kSmem = kStages * kStage + 1024;
  static_assert(kStages * kStage >= 128 * (BN + 4) * 4, "epilogue tile must fit in the operand ring");
};

template <MmaKind KIND, int BN>
__global__ void __launch_bounds__(kTcThreads, 1)
bsr_spmm_tc_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                   const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
                   const int* __restrict__ units, const int* __restrict__ col_idx, int64_t m, int64_t k,
                   float* __restrict__ C, int64_t ldc) {
  using Cfg = TcCfg<KIND>;
  using Lay = TcLayout<KIND, BN>;
  constexpr int S = Lay::kStages;
  extern __shared__ __align__(16) uint8_t dsmem_tc[];
  __shared__ __align__(8) uint64_t full_bar[S];
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const uint32_t raw = smem_u32(dsmem_tc);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const sbase = dsmem_tc + (base - raw);
  auto a_tile = [&](int s, int part) { return sbase + s * Lay::kStage + part * Lay::kATile; };
  auto b_tile = [&](int s, int part) {
    return sbase + s * Lay::kStage + Cfg::kParts * Lay::kATile + part * Lay::kBTile;
  };

  if (threadIdx.x == 0) TC_TRACE(0);
  const int warp = threadIdx.x >> 5;
  const int row_blk = units[3 * blockIdx.x + 0];
  const int blk0 = units[3 * blockIdx.x + 1];
  const int blk1 = units[3 * blockIdx.x + 2];
  const int n0 = blockIdx.y * BN;
  const int total = (blk1 - blk0) * Cfg::kChunksPerBlock;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&done_bar, 1);
    abort_flag = (base & 1023u) ? 1 : 0;  // self-check: never hand TMA a misaligned tile
    if (abort_flag) record_device_error(DEVERR_SELFCHECK_SMEM);
    fence_mbar_init();
    tma_prefetch_desc(&ta_hi);
    tma_prefetch_desc(&tb_hi);
    if (KIND == MmaKind::TF32) {
      tma_prefetch_desc(&ta_lo);
      tma_prefetch_desc(&tb_lo);
    }
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  if (threadIdx.x == 0) TC_TRACE(1);

  if (warp == 0 && elect_lane0()) {
    // ---------------- TMA producer
    int issued = 0;
    for (int it = 0; it < total; ++it) {
      const int s = it % S, use = it / S;
      if (use > 0 && !mbar_wait(&empty_bar[s], (use - 1) & 1)) {
        atomicExch(&abort_flag, 1);
        break;
      }
      if (*(volatile int*)&abort_flag) break;
      const int blk = blk0 + it / Cfg::kChunksPerBlock;
      const int c = it % Cfg::kChunksPerBlock;
      const int j = col_idx[blk];
      mbar_arrive_expect_tx(&full_bar[s], Lay::kStage);
      tma_load_2d(a_tile(s, 0), &ta_hi, c * Cfg::kChunk, blk * 128, &full_bar[s]);
      tma_load_2d(b_tile(s, 0), &tb_hi, j * 128 + c * Cfg::kChunk, n0, &full_bar[s]);
      if (KIND == MmaKind::TF32) {
        tma_load_2d(a_tile(s, 1), &ta_lo, c * Cfg::kChunk, blk * 128, &full_bar[s]);
        tma_load_2d(b_tile(s, 1), &tb_lo, j * 128 + c * Cfg::kChunk, n0, &full_bar[s]);
      }
      issued = it + 1;
      if (it == 0) TC_TRACE(2);
    }
    // never leave the CTA with copies in flight: on the abort path wait for
    // every issued fill the consumer has not waited for
    if (*(volatile int*)&abort_flag) {
      for (int it = (issued > S ? issued - S : 0); it < issued; ++it) mbar_wait(&full_bar[it % S], (it / S) & 1);
    }
  } else if (warp == 1 && elect_lane0()) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc = make_idesc(KIND, 128, BN);
    bool acc = false;
    for (int it = 0; it < total; ++it) {
      if (*(volatile int*)&abort_flag) break;
      const int s = it % S, use = it / S;
      if (!mbar_wait(&full_bar[s], use & 1)) {
        atomicExch(&abort_flag, 1);
        break;
      }
      tc_fence_after();
      if (it == 0) TC_TRACE(3);
      const uint32_t ah = smem_u32(a_tile(s, 0)), bh = smem_u32(b_tile(s, 0));
#pragma unroll
      for (int ks = 0; ks < Cfg::kSteps; ++ks) {
        const uint32_t off = ks * 32;
        umma<KIND>(tmem, smem_desc_sw128(ah + off), smem_desc_sw128(bh + off), idesc, acc);
        acc = true;
        if constexpr (KIND == MmaKind::TF32) {
          const uint32_t al = smem_u32(a_tile(s, 1)), bl = smem_u32(b_tile(s, 1));
          umma<KIND>(tmem, smem_desc_sw128(ah + off), smem_desc_sw128(bl + off), idesc, true);
          umma<KIND>(tmem, smem_desc_sw128(al + off), smem_desc_sw128(bh + off), idesc, true);
        }
      }
      umma_commit(&empty_bar[s]);
    }
    umma_commit(&done_bar);
    TC_TRACE(4);
  }
  __syncwarp();

  // ---------------- epilogue: TMEM -> registers -> C (all 4 warps)
  const bool ok = mbar_wait(&done_bar, 0);
  tc_fence_after();
  if (threadIdx.x == 0) TC_TRACE(5);
  // Each warp moves its 32 accumulator rows TMEM -> registers -> a padded
  // shared-memory tile (the operand ring is idle now); then the CTA adds the
  // tile into C with coalesced 16-byte reductions, a warp covering 512
  // contiguous bytes of a row per instruction.
  const bool run = ok && !*(volatile int*)&abort_flag && total > 0;
  constexpr int LDS = BN + 4;  // padded row stride (floats): conflict-free float4 stores
  float* stile = reinterpret_cast<float*>(sbase);
  if (run) {
    const int lane = threadIdx.x & 31;
    const int r_local = warp * 32 + lane;
#pragma unroll 1
    for (int cc = 0; cc < BN / 32; ++cc) {
      uint32_t r[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + cc * 32, r);
      tmem_wait_ld();
      float4* dst = reinterpret_cast<float4*>(stile + r_local * LDS + cc * 32);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        dst[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 2]),
                             __uint_as_float(r[4 * q + 3]));
    }
  }
  __syncthreads();
  if (run) {
    const int64_t row0 = static_cast<int64_t>(row_blk) * 128;
    const bool vec = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15u) == 0) && (n0 + BN <= k);
    if (vec) {
      constexpr int F4 = BN / 4;  // float4 per tile row
      for (int f = threadIdx.x; f < 128 * F4; f += kTcThreads) {
        const int rl = f / F4, c4 = f - rl * F4;
        const int64_t row = row0 + rl;
        if (row < m) {
          const float4 v = *reinterpret_cast<const float4*>(stile + rl * LDS + 4 * c4);
          red_add_v4(C + row * ldc + n0 + 4 * c4, __float_as_uint(v.x), __float_as_uint(v.y), __float_as_uint(v.z),
                     __float_as_uint(v.w));
        }
      }
    } else {
      for (int f = threadIdx.x; f < 128 * BN; f += kTcThreads) {
        const int rl = f / BN, c = f - rl * BN;
        const int64_t row = row0 + rl, col = n0 + c;
        if (row < m && col < k) red_add(C + row * ldc + col, __float_as_uint(stile[rl * LDS + c]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) TC_TRACE(6);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

template <MmaKind KIND, int BN>
int launch_tc(const CUtensorMap& ahi, const CUtensorMap& alo, const CUtensorMap& bhi, const CUtensorMap& blo,
              const int* units, int n_units, const int* col_idx, int64_t m, int64_t k, float* C, int64_t ldc,
              cudaStream_t st) {
  using Lay = TcLayout<KIND, BN>;
  auto kern = bsr_spmm_tc_kernel<KIND, BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kSmem);
  if (e != cudaSuccess) return cuda_status(e, "bsr_spmm_tc: set smem");
  dim3 grid((unsigned)n_units, (unsigned)((k + BN - 1) / BN));
  kern<<<grid, kTcThreads, Lay::kSmem, st>>>(ahi, alo, bhi, blo, units, col_idx, m, k, C, ldc);
  TSB_CHECK_LAUNCH("bsr_spmm_tc launch");
  return debug_sync(st, "bsr_spmm_tc: main kernel (sync)");
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" int trnsparse_bsr_split_tf32(int64_t count, const float* src, float* hi, float* lo, void* stream) {
  TSB_REQUIRE(count >= 0 && (count == 0 || (src && hi && lo)), "bsr_split_tf32: bad argument");
  if (count == 0) return TRNSPARSE_OK;
  int64_t g = (count + 255) / 256;
  if (g > 8 * sm_count()) g = 8 * sm_count();
  split_tf32_kernel<<<(unsigned)g, 256, 0, as_stream(stream)>>>(count, src, hi, lo);
  TSB_CHECK_LAUNCH("bsr_split_tf32");
  return debug_sync(as_stream(stream), "bsr_split_tf32 (sync)");
}

extern "C" size_t trnsparse_bsr_spmm_tc_workspace_size(int64_t n, int64_t k, int dtype) {
  const int64_t n_pad = (n + 127) / 128 * 128;
  const size_t es = dtype == TRNSPARSE_F32 ? 4 : 2;
  const size_t one = align256(es * (size_t)n_pad * (size_t)(k < 0 ? 0 : k));
  return dtype == TRNSPARSE_F32 ? 2 * one : one;
}

extern "C" int trnsparse_bsr_spmm_tc(int64_t m, int64_t n, int64_t n_blocks, const int* col_idx,
                                     const void* blocks_hi, const void* blocks_lo, int dtype, const int* units,
                                     int n_units, const void* B, int64_t k, int64_t ldb, float* C, int64_t ldc,
                                     int bn, void* ws, size_t ws_bytes, void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && k >= 0 && n_blocks >= 0 && n_units >= 0, "bsr_spmm_tc: negative size");
  TSB_REQUIRE(dtype == TRNSPARSE_F32 || dtype == TRNSPARSE_BF16, "bsr_spmm_tc: dtype must be F32 or BF16");
  TSB_REQUIRE(ldc >= k && ldb >= k, "bsr_spmm_tc: leading dimension smaller than k");
  TSB_REQUIRE(bn == 0 || bn == 128 || bn == 256, "bsr_spmm_tc: bn must be 0, 128 or 256");
  if (m == 0 || k == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(C && (n_units == 0 || (units && col_idx && blocks_hi && B)), "bsr_spmm_tc: null pointer");
  TSB_REQUIRE(dtype != TRNSPARSE_F32 || n_units == 0 || blocks_lo, "bsr_spmm_tc: F32 needs blocks_lo");
  const size_t need = trnsparse_bsr_spmm_tc_workspace_size(n, k, dtype);
  TSB_REQUIRE(ws && ws_bytes >= need, "bsr_spmm_tc: workspace too small (%zu < %zu)", ws_bytes, need);
  TSB_REQUIRE(k <= 65535 * 32, "bsr_spmm_tc: k too large");
  cudaStream_t st = as_stream(stream);
  cudaError_t e = cudaMemset2DAsync(C, sizeof(float) * (size_t)ldc, 0, sizeof(float) * (size_t)k, (size_t)m, st);
  if (e != cudaSuccess) return cuda_status(e, "bsr_spmm_tc: zero C");
  if (n_units == 0 || n_blocks == 0) return TRNSPARSE_OK;

  const int64_t n_pad = (n + 127) / 128 * 128;
  const bool f32 = dtype == TRNSPARSE_F32;
  const size_t es = f32 ? 4 : 2;
  uint8_t* bt_hi = static_cast<uint8_t*>(ws);
  uint8_t* bt_lo = bt_hi + align256(es * (size_t)n_pad * (size_t)k);
  dim3 tg((unsigned)(n_pad / 32), (unsigned)((k + 31) / 32));
  if (f32)
    transpose_b_kernel<true, float><<<tg, dim3(32, 8), 0, st>>>(n, k, (const float*)B, ldb, n_pad, (float*)bt_hi,
                                                               (float*)bt_lo);
  else
    transpose_b_kernel<false, uint16_t><<<tg, dim3(32, 8), 0, st>>>(n, k, (const uint16_t*)B, ldb, n_pad,
                                                                   (uint16_t*)bt_hi, nullptr);
  TSB_CHECK_LAUNCH("bsr_spmm_tc: transpose B");
  if (int drc = debug_sync(st, "bsr_spmm_tc: transpose B (sync)")) return drc;

  if (bn == 0) bn = k > 128 ? 256 : 128;
  const CUtensorMapDataType dt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t kch = f32 ? 32 : 64;
  CUtensorMap ahi, alo, bhi, blo;
  int rc = make_tmap_2d(&ahi, blocks_hi, dt, 128, (uint64_t)n_blocks * 128, 128 * es, kch, 128);
  if (rc) return rc;
  rc = make_tmap_2d(&bhi, bt_hi, dt, (uint64_t)n_pad, (uint64_t)k, n_pad * es, kch, (uint32_t)bn);
  if (rc) return rc;
  if (f32) {
    rc = make_tmap_2d(&alo, blocks_lo, dt, 128, (uint64_t)n_blocks * 128, 128 * es, kch, 128);
    if (rc) return rc;
    rc = make_tmap_2d(&blo, bt_lo, dt, (uint64_t)n_pad, (uint64_t)k, n_pad * es, kch, (uint32_t)bn);
    if (rc) return rc;
  } else {
    alo = ahi;
    blo = bhi;
  }
  if (f32)
    return bn == 128 ? launch_tc<MmaKind::TF32, 128>(ahi, alo, bhi, blo, units, n_units, col_idx, m, k, C, ldc, st)
                     : launch_tc<MmaKind::TF32, 256>(ahi, alo, bhi, blo, units, n_units, col_idx, m, k, C, ldc, st);
  return bn == 128 ? launch_tc<MmaKind::BF16, 128>(ahi, alo, bhi, blo, units, n_units, col_idx, m, k, C, ldc, st)
                   : launch_tc<MmaKind::BF16, 256>(ahi, alo, bhi, blo, units, n_units, col_idx, m, k, C, ldc, st);
}

#ifdef TSB_TC_TRACE
extern "C" __attribute__((visibility("default"))) int trnsparse_tc_trace_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, tsb::g_tc_trace, sizeof(tsb::g_tc_trace));
}
#endif
