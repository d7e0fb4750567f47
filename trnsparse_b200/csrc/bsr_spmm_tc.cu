// BSR x dense on the 5th-generation tensor cores (tcgen05 + TMA + TMEM).
//
// Computes C = A @ B for a BSR A with 128x128 blocks (trnsparse/ops.py:162-210,
// the reference's `bsr_spmm`, accelerated there by nki_bsr_spmm,
// trnsparse/nki/dispatch.py:193-381). Each stored block is a dense
// 128x128 contraction against a 128-row slice of B.
//
// Work: a unit is (block-row, contiguous run of its stored blocks, N tile of
// BN columns). A host-side plan (trnsparse_bsr_spmm_tc_plan) splits long
// block-rows into runs so there are a few units per SM and hands the units
// to persistent CTAs, longest first, each to the least-loaded CTA. A CTA
// (6 warps) runs its units back to back:
//   warp 0      TMA producer: per 128-byte K chunk, the A chunk and the B
//               chunk into a ring of shared-memory stages.
//   warp 1      TMEM owner and MMA issuer: tcgen05.mma into one of two
//               128 x BN fp32 accumulators in TMEM, alternating per unit, so
//               the next unit's MMAs overlap this unit's epilogue.
//   warps 2-5   epilogue: each owns 32 accumulator rows (its TMEM lane
//               quadrant), moves 32-column pieces TMEM -> registers -> a
//               128-byte-swizzled shared tile -> one TMA store into C (units
//               that cover their whole block-row) or TMA reduce-add (units
//               that share a block-row; C is zeroed first only then).
// Empty block-rows are units with no blocks whose epilogue stores zeros, so
// C needs no separate clearing unless a block-row is split.
//
// fp32 inputs use 3xTF32: every operand x is split into hi = tf32(x) and
// lo = tf32(x - hi) and the product accumulates hi*hi + hi*lo + lo*hi, which
// keeps the result within ~1e-6 relative error of fp32. A's split is done once
// per matrix (trnsparse_bsr_split_tf32, cached with the device layout); B's
// split and transpose to K-major B^T run per call into the workspace.
// bf16 inputs use kind::f16 with bf16 operands and fp32 accumulation; B is
// read in place as an MN-major operand (no transpose), or from a padded copy
// in the workspace when its rows are not 16-byte aligned.
//
// The kernel declares no static shared memory, so its dynamic window starts
// 1024-byte aligned as the swizzled tiles need; a misaligned base is caught
// by a self-check that aborts the CTA with an error record.
#include <algorithm>
#include <queue>
#include <vector>

#include "tc_common.cuh"

namespace tsb {
namespace {

constexpr int kSpThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kSmemMax = 232448;
constexpr int kUnitReduce = 1 << 30;  // flag in a unit's tile word: reduce-add into C

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
struct SpLayout {
  static constexpr int kA = 128 * 128;  // 128 rows x 128 bytes of K, per part
  static constexpr int kB = BN * 128;   // BN columns x 128 bytes of K, per part
  static constexpr int kStage = TcCfg<KIND>::kParts * (kA + kB);
  static constexpr int kEpi = 4 * 2 * 4096;  // per epilogue warp: two 32 x 32 fp32 staging tiles
  static constexpr int kBarBytes = 512;
  static constexpr int kStages = (kSmemMax - kEpi - kBarBytes) / kStage;
  static constexpr int kEpiOff = kStages * kStage;
  static constexpr int kBarOff = kEpiOff + kEpi;
  static constexpr int kSmem = kBarOff + kBarBytes;
  static_assert(kStages >= 2 && kStages <= 8, "operand ring");
};

struct SpBars {
  uint64_t full[8], empty[8], acc_full[2], acc_empty[2];
  uint32_t tmem_slot;
  int abort_flag;
};

// OUT_BF16: C is bf16 (whole-row units only, plain stores); otherwise fp32.
// plan: grid + 1 CTA offsets into the unit list (padded to a multiple of 4
// ints), then 4 ints per unit: block_row, first block, end block,
// N tile (| kUnitReduce).
__host__ __device__ inline int plan_head(int grid) { return (grid + 4) & ~3; }

template <MmaKind KIND, int BN, bool OUT_BF16>
__global__ void __launch_bounds__(kSpThreads, 1)
bsr_spmm_tc_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                   const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
                   const __grid_constant__ CUtensorMap tc, const int* __restrict__ plan, int grid,
                   const int* __restrict__ col_idx, int64_t m, int64_t k) {
  using Cfg = TcCfg<KIND>;
  using Lay = SpLayout<KIND, BN>;
  constexpr int S = Lay::kStages;
  extern __shared__ __align__(16) uint8_t sp_smem[];
  SpBars& B = *reinterpret_cast<SpBars*>(sp_smem + Lay::kBarOff);
  auto a_tile = [&](int s, int part) { return sp_smem + s * Lay::kStage + part * Lay::kA; };
  auto b_tile = [&](int s, int part) { return sp_smem + s * Lay::kStage + Cfg::kParts * Lay::kA + part * Lay::kB; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&B.full[s], 1);
      mbar_init(&B.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.acc_full[i], 1);
      mbar_init(&B.acc_empty[i], 128);
    }
    B.abort_flag = (smem_u32(sp_smem) & 1023u) ? 1 : 0;
    if (B.abort_flag) record_device_error(DEVERR_SELFCHECK_SMEM);
    fence_mbar_init();
    tma_prefetch_desc(&ta_hi);
    tma_prefetch_desc(&tb_hi);
    tma_prefetch_desc(&tc);
  }
  if (warp == 1) {
    tmem_alloc(&B.tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_wait();  // the set-up above overlapped the previous kernel (the B split, the C clearing)
  const uint32_t tmem = B.tmem_slot;
  volatile int* abort_flag = &B.abort_flag;
  const int u_begin = plan[blockIdx.x], u_end = plan[blockIdx.x + 1];
  const int4* units = reinterpret_cast<const int4*>(plan + plan_head(grid));

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0 && !*abort_flag) {
      int it = 0;
      bool ok = true;
      for (int u = u_begin; ok && u < u_end; ++u) {
        const int4 un = units[u];
        const int n0 = (un.w & ~kUnitReduce) * BN;
        for (int blk = un.y; ok && blk < un.z; ++blk) {
          const int j = col_idx[blk];
#pragma unroll 1
          for (int c = 0; c < Cfg::kChunksPerBlock; ++c, ++it) {
            const int s = it % S, use = it / S;
            if (use > 0 && !mbar_wait(&B.empty[s], (use - 1) & 1)) { ok = false; break; }
            if (*abort_flag) { ok = false; break; }
            mbar_arrive_expect_tx(&B.full[s], Lay::kStage);
            tma_load_2d(a_tile(s, 0), &ta_hi, c * Cfg::kChunk, blk * 128, &B.full[s]);
            if constexpr (KIND == MmaKind::TF32) {
              tma_load_2d(a_tile(s, 1), &ta_lo, c * Cfg::kChunk, blk * 128, &B.full[s]);
              tma_load_2d(b_tile(s, 0), &tb_hi, j * 128 + c * Cfg::kChunk, n0, &B.full[s]);
              tma_load_2d(b_tile(s, 1), &tb_lo, j * 128 + c * Cfg::kChunk, n0, &B.full[s]);
            } else {
              // MN-major B: BN / 64 boxes of 64 columns x 64 K rows
#pragma unroll
              for (int q = 0; q < BN / 64; ++q)
                tma_load_2d(b_tile(s, 0) + q * 8192, &tb_hi, n0 + q * 64, j * 128 + c * 64, &B.full[s]);
            }
          }
        }
      }
      if (!ok) {
        atomicExch(&B.abort_flag, 1);
        // never leave the CTA with copies in flight: wait for the fills nobody consumed
        for (int i = (it > S ? it - S : 0); i < it; ++i) mbar_wait(&B.full[i % S], (i / S) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(KIND, 128, BN) | (KIND == MmaKind::BF16 ? (1u << 16) : 0u);
      int it = 0, q = 0;
      bool ok = !*abort_flag;
      for (int u = u_begin; ok && u < u_end; ++u, ++q) {
        const int4 un = units[u];
        const int acc = q & 1;
        if (q >= 2 && !mbar_wait(&B.acc_empty[acc], ((q >> 1) - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        const int nch = (un.z - un.y) * Cfg::kChunksPerBlock;
        if (nch == 0) {  // empty block-row: nothing to accumulate, the epilogue stores zeros
          mbar_arrive(&B.acc_full[acc]);
          continue;
        }
        for (int ch = 0; ch < nch; ++ch, ++it) {
          const int s = it % S, use = it / S;
          if (*abort_flag || !mbar_wait(&B.full[s], use & 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t ah = smem_u32(a_tile(s, 0)), bh = smem_u32(b_tile(s, 0));
#pragma unroll
          for (int ks = 0; ks < Cfg::kSteps; ++ks) {
            const bool accum = ch > 0 || ks > 0;
            if constexpr (KIND == MmaKind::TF32) {
              const uint32_t off = ks * 32;
              const uint32_t al = smem_u32(a_tile(s, 1)), bl = smem_u32(b_tile(s, 1));
              umma<KIND>(d, smem_desc_sw128(ah + off), smem_desc_sw128(bh + off), idesc, accum);
              umma<KIND>(d, smem_desc_sw128(ah + off), smem_desc_sw128(bl + off), idesc, true);
              umma<KIND>(d, smem_desc_sw128(al + off), smem_desc_sw128(bh + off), idesc, true);
            } else {
              // A K-major (+32 bytes per 16 K); B MN-major (+16 K rows = 2048 bytes), 64-column
              // chunks 8192 bytes apart
              umma<KIND>(d, smem_desc_sw128(ah + ks * 32), smem_desc_sw128_mn(bh + ks * 2048, 8192), idesc, accum);
            }
          }
          umma_commit(&B.empty[s]);
        }
        if (!ok) break;
        umma_commit(&B.acc_full[acc]);
      }
      if (!ok) atomicExch(&B.abort_flag, 1);
    }
  } else {
    // ---------------- epilogue warps: TMEM lane quadrant = warp % 4
    const int quad = warp & 3;
    uint8_t* const stage0 = sp_smem + Lay::kEpiOff + (warp - 2) * 8192;
    int q = 0, pc = 0;
    bool ok = !*abort_flag;
    for (int u = u_begin; u < u_end; ++u, ++q) {
      const int4 un = units[u];
      const int acc = q & 1;
      const bool reduce = (un.w & kUnitReduce) != 0;
      const int n0 = (un.w & ~kUnitReduce) * BN;
      const int64_t row0 = static_cast<int64_t>(un.x) * 128 + quad * 32;
      ok = ok && mbar_wait(&B.acc_full[acc], (q >> 1) & 1) && !*abort_flag;
      tc_fence_after();
      const bool have = __all_sync(0xffffffffu, ok) && un.z > un.y;
      constexpr int PW = OUT_BF16 ? 64 : 32;  // columns per piece: one 128-byte staged row
      const uint32_t t_row = tmem + acc * BN + (static_cast<uint32_t>(quad * 32) << 16);
#pragma unroll 1
      for (int p = 0; p < BN / PW && n0 + p * PW < k; ++p, ++pc) {
        uint8_t* stage = stage0 + (pc & 1) * 4096;
        if (pc >= 2) {
          if (lane == 0) bulk_wait_read_1();  // the store issued two pieces ago has read its tile
          __syncwarp();
        }
        uint32_t w[32];  // the 128 bytes of row `lane` of this piece
        if (have) {
          if constexpr (OUT_BF16) {
            uint32_t v0[32], v1[32];
            tmem_ld32(t_row + p * 64, v0);
            tmem_ld32(t_row + p * 64 + 32, v1);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              w[i] = pack_bf16(__uint_as_float(v0[2 * i]), __uint_as_float(v0[2 * i + 1]));
              w[16 + i] = pack_bf16(__uint_as_float(v1[2 * i]), __uint_as_float(v1[2 * i + 1]));
            }
          } else {
            tmem_ld32(t_row + p * 32, w);
            tmem_wait_ld();
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = 0u;
        }
        // 8 16-byte units per row, 128-byte swizzle (the C tensor map's)
#pragma unroll
        for (int x = 0; x < 8; ++x)
          *reinterpret_cast<uint4*>(stage + lane * 128 + ((x ^ (lane & 7)) * 16)) =
              make_uint4(w[4 * x], w[4 * x + 1], w[4 * x + 2], w[4 * x + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && row0 < m && ok) {
          if (reduce)  // fp32 or bf16 adds, per the C tensor map's type
            tma_reduce_add_2d(&tc, stage, n0 + p * PW, static_cast<int>(row0));
          else
            tma_store_2d(&tc, stage, n0 + p * PW, static_cast<int>(row0));
          bulk_commit_group();
        }
      }
      tc_fence_before();
      mbar_arrive(&B.acc_empty[acc]);
    }
    if (lane == 0) bulk_wait_all();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
}

template <MmaKind KIND, int BN, bool OUT_BF16 = false>
int launch_sp(const CUtensorMap& ahi, const CUtensorMap& alo, const CUtensorMap& bhi, const CUtensorMap& blo,
              const CUtensorMap& cm, const int* plan, int grid, const int* col_idx, int64_t m, int64_t k,
              cudaStream_t st) {
  using Lay = SpLayout<KIND, BN>;
  auto kern = bsr_spmm_tc_kernel<KIND, BN, OUT_BF16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kSmem);
  if (e != cudaSuccess) return cuda_status(e, "bsr_spmm_tc: set smem");
  e = launch_pdl(kern, dim3(grid), dim3(kSpThreads), Lay::kSmem, st, ahi, alo, bhi, blo, cm, plan, grid, col_idx, m, k);
  if (e != cudaSuccess) return cuda_status(e, "bsr_spmm_tc launch");
  return debug_sync(st, "bsr_spmm_tc: main kernel (sync)");
}

inline int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

// Row stride (elements) of the padded bf16 copy of B used when B cannot be read in place.
inline int64_t bf16_pad_ld(int64_t k) { return std::max<int64_t>(64, round_up(k, 8)); }

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" int trnsparse_bsr_split_tf32(int64_t count, const float* src, float* hi, float* lo, void* stream) {
  TSB_REQUIRE(count >= 0 && (count == 0 || (src && lo)), "bsr_split_tf32: bad argument");
  if (count == 0) return TRNSPARSE_OK;
  int64_t g = (count + 255) / 256;
  if (g > 8 * sm_count()) g = 8 * sm_count();
  split_tf32_kernel<<<(unsigned)g, 256, 0, as_stream(stream)>>>(count, src, hi, lo);
  TSB_CHECK_LAUNCH("bsr_split_tf32");
  return debug_sync(as_stream(stream), "bsr_split_tf32 (sync)");
}

extern "C" int64_t trnsparse_bsr_spmm_tc_plan_capacity(int64_t n_block_rows, int64_t n_blocks, int64_t k, int bn,
                                                       int n_ctas) {
  if (n_block_rows < 0 || n_blocks < 0 || k < 0 || (bn != 128 && bn != 256) || n_ctas <= 0) return -1;
  const int64_t tiles = (k + bn - 1) / bn;
  return plan_head(n_ctas) + 4 * tiles * (n_block_rows + n_blocks);
}

extern "C" int trnsparse_bsr_spmm_tc_plan(int64_t n_block_rows, const int* row_ptr, int64_t k, int bn, int n_ctas,
                                          int* plan, int64_t capacity, int* n_units_out, int* grid_out,
                                          int* needs_zero_out) {
  TSB_REQUIRE(n_block_rows >= 0 && k > 0 && (bn == 128 || bn == 256) && n_ctas > 0 && row_ptr && plan &&
                  n_units_out && grid_out && needs_zero_out,
              "bsr_spmm_tc_plan: bad argument");
  TSB_REQUIRE(n_block_rows < (1 << 24) && k <= (1ll << 31) - 1, "bsr_spmm_tc_plan: sizes out of range");
  const int64_t n_blocks = row_ptr[n_block_rows] - row_ptr[0];
  TSB_REQUIRE(capacity >= trnsparse_bsr_spmm_tc_plan_capacity(n_block_rows, n_blocks, k, bn, n_ctas),
              "bsr_spmm_tc_plan: plan buffer too small");
  const int tiles = static_cast<int>((k + bn - 1) / bn);
  // Whole block-rows are units when they alone give every CTA work (no C clearing, no
  // reduce-adds); otherwise rows are cut into runs of at most G blocks, about `units_per_cta`
  // units per CTA (TRNSPARSE_SPMM_UNITS_PER_CTA, default 3; 0 = never cut a block-row).
  static const int units_per_cta = [] {
    const char* v = getenv("TRNSPARSE_SPMM_UNITS_PER_CTA");
    return v ? std::max(0, atoi(v)) : 3;
  }();
  const int64_t work = n_blocks * tiles;
  int64_t busy_rows = 0;
  for (int64_t i = 0; i < n_block_rows; ++i) busy_rows += row_ptr[i + 1] > row_ptr[i];
  const bool whole_rows = units_per_cta == 0 || busy_rows * tiles >= n_ctas;
  const int64_t G = whole_rows ? std::max<int64_t>(1, work)
                             : std::max<int64_t>(1, (work + units_per_cta * (int64_t)n_ctas - 1) /
                                                    (units_per_cta * (int64_t)n_ctas));
  struct Unit {
    int row, b0, b1, tile;
  };
  std::vector<Unit> units;
  bool split = false;
  for (int64_t i = 0; i < n_block_rows; ++i) {
    const int b0 = row_ptr[i], b1 = row_ptr[i + 1];
    TSB_REQUIRE(b1 >= b0, "bsr_spmm_tc_plan: row_ptr not monotone at %lld", (long long)i);
    const int64_t len = b1 - b0;
    const int64_t runs = std::max<int64_t>(1, (len + G - 1) / G);
    if (runs > 1) split = true;
    for (int64_t r = 0; r < runs; ++r) {
      const int s = b0 + static_cast<int>(len * r / runs), e = b0 + static_cast<int>(len * (r + 1) / runs);
      for (int t = 0; t < tiles; ++t)
        units.push_back({static_cast<int>(i), s, e, t | (runs > 1 ? kUnitReduce : 0)});
    }
  }
  const int n_units = static_cast<int>(units.size());
  const int grid = std::max(1, std::min(n_ctas, n_units));
  // longest-processing-time-first onto the least-loaded CTA; cost in K chunks, plus the epilogue
  std::vector<int> order(n_units);
  for (int i = 0; i < n_units; ++i) order[i] = i;
  auto cost = [&](const Unit& u) { return static_cast<int64_t>(u.b1 - u.b0) * 4 + 2; };
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return cost(units[a]) > cost(units[b]); });
  using Load = std::pair<int64_t, int>;
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
  for (int c = 0; c < grid; ++c) heap.push({0, c});
  std::vector<std::vector<int>> per(grid);
  for (int idx : order) {
    Load l = heap.top();
    heap.pop();
    per[l.second].push_back(idx);
    l.first += cost(units[idx]);
    heap.push(l);
  }
  int pos = 0;
  for (int c = 0; c < grid; ++c) {
    plan[c] = pos;
    for (int idx : per[c]) {
      int* w = plan + plan_head(grid) + 4 * pos;
      w[0] = units[idx].row;
      w[1] = units[idx].b0;
      w[2] = units[idx].b1;
      w[3] = units[idx].tile;
      ++pos;
    }
  }
  plan[grid] = pos;
  *n_units_out = n_units;
  *grid_out = grid;
  *needs_zero_out = split ? 1 : 0;
  return TRNSPARSE_OK;
}

extern "C" size_t trnsparse_bsr_spmm_tc_workspace_size(int64_t n, int64_t k, int dtype) {
  if (n < 0 || k < 0) return 0;
  if (dtype == TRNSPARSE_F32) {
    const int64_t n_pad = round_up(n, 128);
    return 2 * align256(4 * (size_t)n_pad * (size_t)k);
  }
  return align256(2 * (size_t)n * (size_t)bf16_pad_ld(k));
}

extern "C" int trnsparse_bsr_spmm_tc(int64_t m, int64_t n, int64_t n_blocks, const int* col_idx,
                                     const void* blocks_hi, const void* blocks_lo, int dtype, const int* plan,
                                     int grid, int needs_zero, const void* B, int64_t k, int64_t ldb, void* C,
                                     int64_t ldc, int c_dtype, int bn, void* ws, size_t ws_bytes, void* stream) {
  TSB_REQUIRE(m >= 0 && n >= 0 && k >= 0 && n_blocks >= 0 && grid >= 0, "bsr_spmm_tc: negative size");
  TSB_REQUIRE(dtype == TRNSPARSE_F32 || dtype == TRNSPARSE_BF16, "bsr_spmm_tc: dtype must be F32 or BF16");
  TSB_REQUIRE(ldc >= k && ldb >= k, "bsr_spmm_tc: leading dimension smaller than k");
  TSB_REQUIRE(bn == 128 || bn == 256, "bsr_spmm_tc: bn must be 128 or 256");
  if (m == 0 || k == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(C && plan && grid > 0, "bsr_spmm_tc: null pointer or empty plan");
  TSB_REQUIRE(c_dtype == TRNSPARSE_F32 || (c_dtype == TRNSPARSE_BF16 && dtype == TRNSPARSE_BF16),
              "bsr_spmm_tc: C is F32, or BF16 for BF16 inputs");
  const bool c_bf16 = c_dtype == TRNSPARSE_BF16;
  TSB_REQUIRE((ldc * (c_bf16 ? 2 : 4)) % 16 == 0 && (reinterpret_cast<uintptr_t>(C) & 15u) == 0,
              "bsr_spmm_tc: C must be 16-byte aligned with 16-byte rows");
  TSB_REQUIRE(n_blocks == 0 || (col_idx && blocks_hi && B), "bsr_spmm_tc: null pointer");
  TSB_REQUIRE(dtype != TRNSPARSE_F32 || n_blocks == 0 || blocks_lo, "bsr_spmm_tc: F32 needs blocks_lo");
  TSB_REQUIRE(m < (1ll << 31) && k < (1ll << 31) && n_blocks < (1ll << 24), "bsr_spmm_tc: sizes out of range");
  const size_t need = trnsparse_bsr_spmm_tc_workspace_size(n, k, dtype);
  TSB_REQUIRE(ws && ws_bytes >= need, "bsr_spmm_tc: workspace too small (%zu < %zu)", ws_bytes, need);
  cudaStream_t st = as_stream(stream);
  if (needs_zero) {
    const size_t es_c = c_dtype == TRNSPARSE_BF16 ? 2 : 4;
    cudaError_t e = cudaMemset2DAsync(C, es_c * (size_t)ldc, 0, es_c * (size_t)k, (size_t)m, st);
    if (e != cudaSuccess) return cuda_status(e, "bsr_spmm_tc: zero C");
  }
  const bool f32 = dtype == TRNSPARSE_F32;
  const CUtensorMapDataType dt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const size_t es = f32 ? 4 : 2;
  const uint64_t a_rows = (uint64_t)std::max<int64_t>(n_blocks, 1) * 128;
  CUtensorMap ahi, alo, bhi, blo, cm;
  int rc = c_bf16 ? make_tmap_2d(&cm, C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)k, (uint64_t)m, 2 * ldc, 64, 32)
                  : make_tmap_2d(&cm, C, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (uint64_t)k, (uint64_t)m, 4 * ldc, 32, 32);
  if (rc) return rc;
  const void* a_hi = n_blocks ? blocks_hi : ws;  // an empty A only ever runs zero-storing units
  rc = make_tmap_2d(&ahi, a_hi, dt, 128, a_rows, 128 * es, (uint32_t)(128 / es), 128);
  if (rc) return rc;
  if (n_blocks == 0) {  // no operand is ever loaded
    if (c_bf16) return launch_sp<MmaKind::BF16, 128, true>(ahi, ahi, ahi, ahi, cm, plan, grid, col_idx, m, k, st);
    return f32 ? launch_sp<MmaKind::TF32, 128>(ahi, ahi, ahi, ahi, cm, plan, grid, col_idx, m, k, st)
               : launch_sp<MmaKind::BF16, 128>(ahi, ahi, ahi, ahi, cm, plan, grid, col_idx, m, k, st);
  }
  if (f32) {
    const int64_t n_pad = round_up(n, 128);
    float* bt_hi = static_cast<float*>(ws);
    float* bt_lo = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + align256(4 * (size_t)n_pad * (size_t)k));
    dim3 tg((unsigned)(n_pad / 32), (unsigned)((k + 31) / 32));
    transpose_b_kernel<true, float><<<tg, dim3(32, 8), 0, st>>>(n, k, (const float*)B, ldb, n_pad, bt_hi, bt_lo);
    TSB_CHECK_LAUNCH("bsr_spmm_tc: split/transpose B");
    if (int drc = debug_sync(st, "bsr_spmm_tc: split/transpose B (sync)")) return drc;
    rc = make_tmap_2d(&alo, blocks_lo, dt, 128, a_rows, 512, 32, 128);
    if (!rc) rc = make_tmap_2d(&bhi, bt_hi, dt, (uint64_t)n_pad, (uint64_t)k, 4 * n_pad, 32, (uint32_t)bn);
    if (!rc) rc = make_tmap_2d(&blo, bt_lo, dt, (uint64_t)n_pad, (uint64_t)k, 4 * n_pad, 32, (uint32_t)bn);
    if (rc) return rc;
    return bn == 128 ? launch_sp<MmaKind::TF32, 128>(ahi, alo, bhi, blo, cm, plan, grid, col_idx, m, k, st)
                     : launch_sp<MmaKind::TF32, 256>(ahi, alo, bhi, blo, cm, plan, grid, col_idx, m, k, st);
  }
  // bf16: B (n x k, row-major) read in place as the MN-major operand when its rows are 16-byte
  // aligned and at least one 64-column box wide; otherwise from a zero-padded copy
  const void* bsrc = B;
  int64_t bld = ldb;
  const bool in_place = (k >= 64 && ldb % 8 == 0 && (reinterpret_cast<uintptr_t>(B) & 15u) == 0);
  if (!in_place) {
    bld = bf16_pad_ld(k);
    cudaError_t e = cudaMemsetAsync(ws, 0, 2 * (size_t)n * (size_t)bld, st);
    if (e == cudaSuccess)
      e = cudaMemcpy2DAsync(ws, 2 * (size_t)bld, B, 2 * (size_t)ldb, 2 * (size_t)k, (size_t)n,
                            cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_status(e, "bsr_spmm_tc: pad B");
    bsrc = ws;
  }
  const uint64_t b_cols = (uint64_t)(in_place ? k : bld);
  rc = make_tmap_2d(&bhi, bsrc, dt, b_cols, (uint64_t)std::max<int64_t>(n, 1), 2 * bld, 64, 64);
  if (rc) return rc;
  if (c_bf16)
    return bn == 128 ? launch_sp<MmaKind::BF16, 128, true>(ahi, ahi, bhi, bhi, cm, plan, grid, col_idx, m, k, st)
                     : launch_sp<MmaKind::BF16, 256, true>(ahi, ahi, bhi, bhi, cm, plan, grid, col_idx, m, k, st);
  return bn == 128 ? launch_sp<MmaKind::BF16, 128>(ahi, ahi, bhi, bhi, cm, plan, grid, col_idx, m, k, st)
                   : launch_sp<MmaKind::BF16, 256>(ahi, ahi, bhi, bhi, cm, plan, grid, col_idx, m, k, st);
}
