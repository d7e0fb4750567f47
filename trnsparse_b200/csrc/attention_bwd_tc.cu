// Block-sparse attention backward on the tensor cores (bf16 in/out, fp32
// accumulation), block size 128, head_dim 64 or 128: the reference's
// _block_sparse_attn_backward (trnsparse/ops.py:360-473) with the same
// Flash-delta identity as the CUDA-core kernels of attention_bwd.cu,
//   P = exp(s - lse) (lse = log-sum-exp of the row), dP = dO V^T,
//   dS = P (dP - D), D = rowsum(dO * O),
//   dQ = scale dS K,  dK = scale dS^T Q,  dV = P^T dO,
// over the stored 128x128 blocks only.
//
// One kernel template, two modes, each a persistent CTA per SM walking
// "units" (a fixed 128-row block and a run of at most `split` partner
// blocks; a host plan sorts them longest first):
//   row mode (dQ)     fixed Q, dO of a query block; streamed K, V of the key
//                     blocks it stores (block_col_idx).
//   column mode (dK, dV) fixed K, V of a key block; streamed Q, dO (and the
//                     lse / D of their rows) of the query blocks that store
//                     it (block_row_idx of the transposed pattern).
// Per partner block the MMA warp issues S = F1 X1^T, then dP = F2 X2^T
// (128x128, K = head_dim) into the same 128 TMEM columns; eight warps read
// them (one TMEM lane = one fixed row per thread, 64 columns per warp half),
// form P and dS in fp32 and write them as packed bf16 into two 64-column
// TMEM areas; the MMA warp adds dS X1 (and, in column mode, P X2) into the
// TMEM accumulators at column 256 (+ head_dim) with A taken from TMEM and
// the streamed tile as an MN-major B. The score columns are released as soon
// as they are read, so the next block's S runs on the tensor core while the
// warps compute this block's dS. At the end of a unit the same eight warps
// scale the accumulators and store them as bf16 rows; units of a block that
// was split over several CTAs add fp32 partial sums into a workspace slot
// instead, converted by a finishing kernel.
//
// Warps: 0-7 dS / epilogue, 8 TMA producer, 9 TMEM owner and MMA issuer.
// Every wait is bounded (ptx.cuh): a stalled partner ends in an error record.
#include <cuda_bf16.h>

#include <algorithm>
#include <vector>

#include "tc_common.cuh"

extern "C" int trnsparse_bsr_attention_tc_lse(int64_t heads, int64_t seq, int64_t head_dim,
                                              const int* block_row_ptr, const int* block_col_idx, const void* Q,
                                              const void* K, const void* V, void* O, float* lse, double scale,
                                              void* stream);

namespace tsb {
namespace {

#ifndef TSB_AB_X1_STAGES
#define TSB_AB_X1_STAGES 2
#endif

constexpr int kAbEpi = 256;               // dS / epilogue threads (warps 0-7)
constexpr int kAbThreads = kAbEpi + 64;   // + producer warp + MMA warp

template <int HD>
struct AbLayout {
  static constexpr int kChunks = HD / 64;       // 128-byte column chunks of a row
  static constexpr int kTile = 128 * HD * 2;    // one 128-row bf16 tile
  static constexpr int kF1 = 0, kF2 = kTile;    // fixed tiles
  // streamed tiles: X1 (used by S and by the dS product) and X2 (used by dP and, in column
  // mode, the P product; with the partner rows' lse[128], D[128]) in separate rings, released
  // at different times (a third X1 stage, which fits, measured no faster: the loads are bound
  // by the rate tiles arrive from L2, not by how early they are issued)
  static constexpr int kX1 = 2 * kTile, kX1Stages = TSB_AB_X1_STAGES;
  static constexpr int kX2 = kX1 + kX1Stages * kTile, kX2Stage = kTile + 1024, kX2Stages = 2;
  static constexpr int kBar = kX2 + kX2Stages * kX2Stage;
  static constexpr int kSmem = kBar + 256;
  // TMEM: S, then dP, in [0,128); P and dS as packed bf16 in [128,192) and [192,256);
  // accumulators at 256 (dQ, or dK) and 256 + HD (dV)
  static constexpr uint32_t kTmemA = 0, kTmemP = 128, kTmemDS = 192, kTmemAcc = 256;
  static constexpr int kTmemCols = 512;
};

struct AbBars {
  uint64_t f_full, f_empty, acc_full, acc_empty;
  uint64_t x1_full[TSB_AB_X1_STAGES], x1_empty[TSB_AB_X1_STAGES], x2_full[2], x2_empty[2];
  uint64_t a_full, a_empty, p_full, p_free, ds_full, ds_free;
  uint32_t tmem_slot;
  int abort_flag;
};

#ifdef TSB_TC_TRACE
__device__ unsigned long long g_ab_trace[2][10][64];
// (CTA 64 only) event ev of step i in mode m
#define AB_TRACE(ev, i)                                                                     \
  if (blockIdx.x == 64 && (i) < 64) {                                                       \
    unsigned long long tt_;                                                                 \
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(tt_));                                 \
    g_ab_trace[COL ? 1 : 0][ev][i] = tt_;                                                   \
  }
#else
#define AB_TRACE(ev, i)
#endif

__device__ __forceinline__ float ab_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// TMEM column of the packed A operand (P or dS) for partner rows 16 kk .. 16 kk + 15:
// warp half h packs partner columns 64 h .. 64 h + 63 into 32 columns.
__device__ __forceinline__ uint32_t ab_a_col(int kk) { return (kk >> 2) * 32 + (kk & 3) * 8; }

// units: {fixed block, first partner index, end partner index, workspace slot or -1}.
// Tile t covers unit t / heads of head t % heads (heads of a long unit run side by side).
//
// Per partner block j the MMA warp issues, in order: S_j = F1 X1^T into the score columns,
// the previous block's dS_{j-1} X1 product, dP_j = F2 X2^T into the same columns once S_j
// has been read, and (column mode) P_j X2 once P_j is written. The eight warps read S_j,
// release the columns, form P_j (fp32, kept in registers; packed into TMEM in column mode),
// read dP_j, release the columns and write dS_j = P_j (dP_j - D) packed. So the tensor
// core works on one block's scores while the warps work on the other's.
template <int HD, bool COL>
__global__ void __launch_bounds__(kAbThreads, 1)
attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tf1, const __grid_constant__ CUtensorMap tf2,
                   const __grid_constant__ CUtensorMap tx1, const __grid_constant__ CUtensorMap tx2,
                   const int4* __restrict__ units, const int* __restrict__ partner, int n_tiles, int heads,
                   int seq, const float* __restrict__ lse2, const float* __restrict__ delta,
                   __nv_bfloat16* __restrict__ out1, __nv_bfloat16* __restrict__ out2, float* __restrict__ slots,
                   float scale) {
  using Lay = AbLayout<HD>;
  extern __shared__ __align__(16) uint8_t sb[];  // no static smem: the window is 1024-byte aligned
  AbBars& B = *reinterpret_cast<AbBars*>(sb + Lay::kBar);
  const int warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    mbar_init(&B.f_full, 1);
    mbar_init(&B.f_empty, 1);
    mbar_init(&B.acc_full, 1);
    mbar_init(&B.acc_empty, kAbEpi);
    for (int i = 0; i < TSB_AB_X1_STAGES; ++i) {
      mbar_init(&B.x1_full[i], 1);
      mbar_init(&B.x1_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.x2_full[i], 1);
      mbar_init(&B.x2_empty[i], 1);
    }
    mbar_init(&B.a_full, 1);
    mbar_init(&B.a_empty, kAbEpi);
    mbar_init(&B.p_full, kAbEpi);
    mbar_init(&B.p_free, 1);
    mbar_init(&B.ds_full, kAbEpi);
    mbar_init(&B.ds_free, 1);
    B.abort_flag = (smem_u32(sb) & 1023u) ? 1 : 0;
    if (B.abort_flag) record_device_error(DEVERR_SELFCHECK_SMEM);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(&B.tmem_slot, Lay::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = B.tmem_slot;
  volatile int* abort_flag = &B.abort_flag;

  if (warp == 8) {
    // ---------------- TMA producers: lane 0 the fixed tiles and X1, lane 1 X2 (and the
    // partner rows' statistics); the two rings are released at different times
    const int lane = threadIdx.x & 31;
    if (lane < 2 && !*abort_flag) {
      int gs = 0, nt = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x, ++nt) {
        const int4 u = units[t / heads];
        const int row0 = (t % heads) * seq;
        if (lane == 0) {
          // the fixed tiles are free once the previous unit's last dP has run
          if (nt > 0 && !mbar_wait(&B.f_empty, (nt - 1) & 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&B.f_full, 2 * Lay::kTile);
          for (int c = 0; c < Lay::kChunks; ++c) {
            tma_load_2d(sb + Lay::kF1 + c * 16384, &tf1, c * 64, row0 + u.x * 128, &B.f_full);
            tma_load_2d(sb + Lay::kF2 + c * 16384, &tf2, c * 64, row0 + u.x * 128, &B.f_full);
          }
        }
        for (int e = u.y; e < u.z; ++e, ++gs) {
          const int pb = partner[e];
          const int xrow = row0 + pb * 128;
          if (lane == 0) {
            const int st = gs % TSB_AB_X1_STAGES, use = gs / TSB_AB_X1_STAGES;
            if (*abort_flag || (use > 0 && !mbar_wait(&B.x1_empty[st], (use - 1) & 1))) { ok = false; break; }
            AB_TRACE(0, gs);
            uint8_t* xs = sb + Lay::kX1 + st * Lay::kTile;
            mbar_arrive_expect_tx(&B.x1_full[st], Lay::kTile);
            for (int c = 0; c < Lay::kChunks; ++c) tma_load_2d(xs + c * 16384, &tx1, c * 64, xrow, &B.x1_full[st]);
          } else {
            const int st = gs & 1, use = gs >> 1;
            if (*abort_flag || (use > 0 && !mbar_wait(&B.x2_empty[st], (use - 1) & 1))) { ok = false; break; }
            uint8_t* xs = sb + Lay::kX2 + st * Lay::kX2Stage;
            mbar_arrive_expect_tx(&B.x2_full[st], Lay::kTile + (COL ? 1024 : 0));
            for (int c = 0; c < Lay::kChunks; ++c) tma_load_2d(xs + c * 16384, &tx2, c * 64, xrow, &B.x2_full[st]);
            if (COL) {
              const int vrow = (pb >= 0 && pb * 128 < seq) ? xrow : row0;  // never read past the statistics
              bulk_g2s(xs + Lay::kTile, lse2 + vrow, 512, &B.x2_full[st]);
              bulk_g2s(xs + Lay::kTile + 512, delta + vrow, 512, &B.x2_full[st]);
            }
          }
        }
      }
      if (!ok) atomicExch(&B.abort_flag, 1);
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer
    if (elect_lane0()) {
      constexpr uint32_t idesc_s = make_idesc(MmaKind::BF16, 128, 128);
      constexpr uint32_t idesc_a = make_idesc(MmaKind::BF16, 128, HD) | (1u << 16);  // B MN-major
      const uint32_t f1 = smem_u32(sb + Lay::kF1), f2 = smem_u32(sb + Lay::kF2);
      bool ok = !*abort_flag;
      // the dS X1 product of the previous partner block, issued after the next block's S
      bool pend = false, pfirst = false, plast = false;
      int pgs = 0, pnt = 0;
      auto issue_ds = [&]() -> bool {
        if (!mbar_wait(&B.ds_full, pgs & 1)) return false;
        if (!COL && pfirst && pnt > 0 && !mbar_wait(&B.acc_empty, (pnt - 1) & 1)) return false;
        tc_fence_after();
        const uint32_t x1 = smem_u32(sb + Lay::kX1 + (pgs % TSB_AB_X1_STAGES) * Lay::kTile);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // 128 partner rows, 16 per MMA
          umma_ts_f16(tmem + Lay::kTmemAcc, tmem + Lay::kTmemDS + ab_a_col(kk),
                      smem_desc_sw128_mn(x1 + kk * 2048, 16384), idesc_a, !pfirst || kk > 0);
        umma_commit(&B.ds_free);
        umma_commit(&B.x1_empty[pgs % TSB_AB_X1_STAGES]);
        if (COL) umma_commit(&B.x2_empty[pgs & 1]);  // dO, and D read by the dS warps
        if (plast) umma_commit(&B.acc_full);
        return true;
      };
      int gs = 0, nt = 0;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x, ++nt) {
        const int4 u = units[t / heads];
        // close the previous unit (its accumulators go to the epilogue) before waiting for new fixed tiles
        if (pend && !issue_ds()) { ok = false; break; }
        pend = false;
        if (!mbar_wait(&B.f_full, nt & 1)) { ok = false; break; }
        for (int e = u.y; e < u.z; ++e, ++gs) {
          const bool first = e == u.y, last = e == u.z - 1;
          if (*abort_flag || !mbar_wait(&B.x1_full[gs % TSB_AB_X1_STAGES], (gs / TSB_AB_X1_STAGES) & 1)) { ok = false; break; }
          AB_TRACE(1, gs);
          // score columns free: the previous block's dP has been read (a_empty completion 2 gs - 1)
          if (gs > 0 && !mbar_wait(&B.a_empty, 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t x1 = smem_u32(sb + Lay::kX1 + (gs % TSB_AB_X1_STAGES) * Lay::kTile);
          const uint32_t x2 = smem_u32(sb + Lay::kX2 + (gs & 1) * Lay::kX2Stage);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma<MmaKind::BF16>(tmem + Lay::kTmemA, smem_desc_sw128(f1 + off), smem_desc_sw128(x1 + off), idesc_s,
                                kk > 0);
          }
          umma_commit(&B.a_full);
          AB_TRACE(2, gs);
          if (pend && !issue_ds()) { ok = false; break; }
          AB_TRACE(3, gs);
          pend = false;
          // S read (a_empty completion 2 gs): dP into the same columns
          if (!mbar_wait(&B.a_empty, 0) || !mbar_wait(&B.x2_full[gs & 1], (gs >> 1) & 1)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma<MmaKind::BF16>(tmem + Lay::kTmemA, smem_desc_sw128(f2 + off), smem_desc_sw128(x2 + off), idesc_s,
                                kk > 0);
          }
          umma_commit(&B.a_full);
          if (!COL) umma_commit(&B.x2_empty[gs & 1]);  // V is read by dP only
          AB_TRACE(4, gs);
          if (last) umma_commit(&B.f_empty);  // the fixed tiles are read for the last time
          if (COL) {
            if (!mbar_wait(&B.p_full, gs & 1)) { ok = false; break; }
            if (first && nt > 0 && !mbar_wait(&B.acc_empty, (nt - 1) & 1)) { ok = false; break; }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_ts_f16(tmem + Lay::kTmemAcc + HD, tmem + Lay::kTmemP + ab_a_col(kk),
                          smem_desc_sw128_mn(x2 + kk * 2048, 16384), idesc_a, !first || kk > 0);
            umma_commit(&B.p_free);
          }
          pend = true;
          pgs = gs;
          pnt = nt;
          pfirst = first;
          plast = last;
        }
      }
      if (ok && pend && !issue_ds()) ok = false;
      if (!ok) atomicExch(&B.abort_flag, 1);
    }
  } else {
    // ---------------- P / dS and epilogue warps
    const int quad = warp & 3, half = warp >> 2, lr = threadIdx.x & 31;
    const int r = quad * 32 + lr;  // fixed row of this thread (TMEM lane)
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tl = tmem + lane_base;
    const float sl = scale * 1.4426950408889634f;
    int gs = 0, nt = 0;
    bool ok = !*abort_flag;
    for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++nt) {
      const int4 u = units[t / heads];
      const int head = t % heads;
      const int64_t frow = static_cast<int64_t>(head) * seq + u.x * 128 + r;
      float l_r = 0.f, d_r = 0.f;
      if (!COL && u.x * 128 < seq) {
        l_r = lse2[frow];
        d_r = delta[frow];
      }
      for (int e = u.y; e < u.z; ++e, ++gs) {
        const float4* vl4 =
            reinterpret_cast<const float4*>(sb + Lay::kX2 + (gs & 1) * Lay::kX2Stage + Lay::kTile) + half * 16;
        if (*abort_flag || (COL && !mbar_wait(&B.x2_full[gs & 1], (gs >> 1) & 1))) { ok = false; break; }
        // ---- S -> P
        if (!mbar_wait(&B.a_full, 0)) { ok = false; break; }
        tc_fence_after();
        float p[64];
        {
          uint32_t v0[32], v1[32];
          tmem_ld32(tl + Lay::kTmemA + half * 64, v0);
          tmem_ld32(tl + Lay::kTmemA + half * 64 + 32, v1);
          tmem_wait_ld();
          tc_fence_before();
          mbar_arrive(&B.a_empty);
          if (threadIdx.x == 0) AB_TRACE(5, gs);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            p[i] = __uint_as_float(v0[i]);
            p[32 + i] = __uint_as_float(v1[i]);
          }
        }
        if (COL) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float4 l4 = vl4[i];
            p[4 * i] = ab_ex2(fmaf(p[4 * i], sl, -l4.x));
            p[4 * i + 1] = ab_ex2(fmaf(p[4 * i + 1], sl, -l4.y));
            p[4 * i + 2] = ab_ex2(fmaf(p[4 * i + 2], sl, -l4.z));
            p[4 * i + 3] = ab_ex2(fmaf(p[4 * i + 3], sl, -l4.w));
          }
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) pk[i] = pack_bf16(p[2 * i], p[2 * i + 1]);
          if (gs > 0 && !mbar_wait(&B.p_free, (gs - 1) & 1)) { ok = false; break; }
          tc_fence_after();
          tmem_st32(tl + Lay::kTmemP + half * 32, pk);
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&B.p_full);
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) p[i] = ab_ex2(fmaf(p[i], sl, -l_r));
        }
        // ---- dP -> dS = P (dP - D)
        if (threadIdx.x == 0) AB_TRACE(6, gs);
        if (!mbar_wait(&B.a_full, 1)) { ok = false; break; }
        tc_fence_after();
        uint32_t pk[32];
        {
          uint32_t v0[32], v1[32];
          tmem_ld32(tl + Lay::kTmemA + half * 64, v0);
          tmem_ld32(tl + Lay::kTmemA + half * 64 + 32, v1);
          tmem_wait_ld();
          tc_fence_before();
          mbar_arrive(&B.a_empty);
          if (threadIdx.x == 0) AB_TRACE(7, gs);
          if (COL) {
            const float4* d4 = vl4 + 32;  // D follows the 128 lse values
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 a = d4[i], b = d4[8 + i];
              pk[2 * i] = pack_bf16(p[4 * i] * (__uint_as_float(v0[4 * i]) - a.x),
                                    p[4 * i + 1] * (__uint_as_float(v0[4 * i + 1]) - a.y));
              pk[2 * i + 1] = pack_bf16(p[4 * i + 2] * (__uint_as_float(v0[4 * i + 2]) - a.z),
                                        p[4 * i + 3] * (__uint_as_float(v0[4 * i + 3]) - a.w));
              pk[16 + 2 * i] = pack_bf16(p[32 + 4 * i] * (__uint_as_float(v1[4 * i]) - b.x),
                                         p[32 + 4 * i + 1] * (__uint_as_float(v1[4 * i + 1]) - b.y));
              pk[16 + 2 * i + 1] = pack_bf16(p[32 + 4 * i + 2] * (__uint_as_float(v1[4 * i + 2]) - b.z),
                                             p[32 + 4 * i + 3] * (__uint_as_float(v1[4 * i + 3]) - b.w));
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              pk[i] = pack_bf16(p[2 * i] * (__uint_as_float(v0[2 * i]) - d_r),
                                p[2 * i + 1] * (__uint_as_float(v0[2 * i + 1]) - d_r));
              pk[16 + i] = pack_bf16(p[32 + 2 * i] * (__uint_as_float(v1[2 * i]) - d_r),
                                     p[32 + 2 * i + 1] * (__uint_as_float(v1[2 * i + 1]) - d_r));
            }
          }
        }
        if (gs > 0 && !mbar_wait(&B.ds_free, (gs - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        tmem_st32(tl + Lay::kTmemDS + half * 32, pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&B.ds_full);
        if (threadIdx.x == 0) AB_TRACE(8, gs);
      }
      if (!ok) break;
      // ---- unit epilogue: accumulators (x scale for dQ / dK) -> bf16 rows, or fp32 partial sums
      if (!mbar_wait(&B.acc_full, nt & 1)) { ok = false; break; }
      if (threadIdx.x == 0) AB_TRACE(9, nt);
      tc_fence_after();
      const int slot = u.w;
      const bool live = u.x * 128 + r < seq;
#pragma unroll 1
      for (int a = 0; a < (COL ? 2 : 1); ++a) {
        const float mul = a == 0 ? scale : 1.f;
        float* const wrow = slot >= 0 ? slots + ((static_cast<int64_t>(slot) * heads + head) * 2 + a) * 128 * HD +
                                            r * HD + half * (HD / 2)
                                      : nullptr;
        __nv_bfloat16* const orow = (a == 0 ? out1 : out2) + frow * HD + half * (HD / 2);
#pragma unroll 1
        for (int c = 0; c < HD / 64; ++c) {
          uint32_t v[32];
          tmem_ld32(tl + Lay::kTmemAcc + a * HD + half * (HD / 2) + c * 32, v);
          tmem_wait_ld();
          if (!live) continue;
          if (slot >= 0) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              red_add_v4(wrow + c * 32 + 4 * q, __float_as_uint(__uint_as_float(v[4 * q]) * mul),
                         __float_as_uint(__uint_as_float(v[4 * q + 1]) * mul),
                         __float_as_uint(__uint_as_float(v[4 * q + 2]) * mul),
                         __float_as_uint(__uint_as_float(v[4 * q + 3]) * mul));
          } else {
            uint4* o4 = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              auto f = [&](int i) { return __uint_as_float(v[8 * q + i]) * mul; };
              o4[q] = make_uint4(pack_bf16(f(0), f(1)), pack_bf16(f(2), f(3)), pack_bf16(f(4), f(5)),
                                 pack_bf16(f(6), f(7)));
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&B.acc_empty);  // accumulators read: the next unit's products may start
    }
    if (!ok) atomicExch(&B.abort_flag, 1);
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, Lay::kTmemCols);
  }
}

// D[row] = dO[row] . O[row] (fp32), 16-byte pieces, HD / 8 threads per row.
template <int HD>
__global__ void attn_bwd_delta_kernel(int64_t rows, const __nv_bfloat16* __restrict__ O,
                                      const __nv_bfloat16* __restrict__ dO, float* __restrict__ delta) {
  constexpr int kPer = HD / 8;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t row = i / kPer;
  float acc = 0.f;
  if (row < rows) {
    const uint4 a = reinterpret_cast<const uint4*>(O)[i];
    const uint4 b = reinterpret_cast<const uint4*>(dO)[i];
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 x = __bfloat1622float2(pa[k]), y = __bfloat1622float2(pb[k]);
      acc = fmaf(x.x, y.x, fmaf(x.y, y.y, acc));
    }
  }
#pragma unroll
  for (int o = kPer / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (row < rows && (threadIdx.x % kPer) == 0) delta[row] = acc;
}

// aux: {mode (0 dQ, 1 dK and dV), block, slot or -1, 0}; grid (n_aux, heads).
// ZERO_SLOTS: clear the slots before the products; otherwise write the rows of
// each entry: the slot's fp32 sums as bf16, or zeros for a block with no stored partner.
template <int HD, bool ZERO_SLOTS>
__global__ void attn_bwd_aux_kernel(const int4* __restrict__ aux, int heads, int seq, float* __restrict__ slots,
                                    __nv_bfloat16* __restrict__ dQ, __nv_bfloat16* __restrict__ dK,
                                    __nv_bfloat16* __restrict__ dV) {
  const int4 x = aux[blockIdx.x];
  const int head = blockIdx.y;
  if (x.y < 0 || (x.y + 1) * 128 > seq) return;  // a block past the sequence has no rows
  const int n_out = x.x == 0 ? 1 : 2;
  if (ZERO_SLOTS) {
    if (x.z < 0) return;
    float4* s = reinterpret_cast<float4*>(slots + (static_cast<int64_t>(x.z) * heads + head) * 2 * 128 * HD);
    for (int i = threadIdx.x; i < n_out * 128 * HD / 4; i += blockDim.x) s[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  for (int a = 0; a < n_out; ++a) {
    __nv_bfloat16* out = (x.x == 0 ? dQ : (a == 0 ? dK : dV)) + (static_cast<int64_t>(head) * seq + x.y * 128) * HD;
    const float* s = x.z >= 0 ? slots + ((static_cast<int64_t>(x.z) * heads + head) * 2 + a) * 128 * HD : nullptr;
    for (int i = threadIdx.x; i < 128 * HD / 2; i += blockDim.x) {
      const float2 v = s ? reinterpret_cast<const float2*>(s)[i] : make_float2(0.f, 0.f);
      reinterpret_cast<__nv_bfloat162*>(out)[i] = __floats2bfloat162_rn(v.x, v.y);
    }
  }
}

template <int HD, bool COL>
int launch_ab_mode(const CUtensorMap* maps, const int4* units, int n_units, const int* partner, int heads, int seq,
                   const float* lse2, const float* delta, void* out1, void* out2, float* slots, float scale,
                   cudaStream_t st) {
  if (n_units <= 0) return TRNSPARSE_OK;
  using Lay = AbLayout<HD>;
  auto kern = attn_bwd_tc_kernel<HD, COL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kSmem);
  if (e != cudaSuccess) return cuda_status(e, "attention_backward_tc: set smem");
  const int64_t n_tiles = static_cast<int64_t>(n_units) * heads;
  const int grid = n_tiles < sm_count() ? (int)n_tiles : sm_count();
  // maps: 0 Q, 1 K, 2 V, 3 dO
  if (COL)
    kern<<<grid, kAbThreads, Lay::kSmem, st>>>(maps[1], maps[2], maps[0], maps[3], units, partner, (int)n_tiles,
                                               heads, seq, lse2, delta, (__nv_bfloat16*)out1, (__nv_bfloat16*)out2,
                                               slots, scale);
  else
    kern<<<grid, kAbThreads, Lay::kSmem, st>>>(maps[0], maps[3], maps[1], maps[2], units, partner, (int)n_tiles,
                                               heads, seq, lse2, delta, (__nv_bfloat16*)out1, (__nv_bfloat16*)out1,
                                               slots, scale);
  TSB_CHECK_LAUNCH(COL ? "attention_backward_tc: dK dV" : "attention_backward_tc: dQ");
  return debug_sync(st, COL ? "attention_backward_tc: dK dV (sync)" : "attention_backward_tc: dQ (sync)");
}

template <int HD>
int launch_ab(int heads, int seq, const int* rp, const int* ci, const int* ri, const int4* plan, int n_row_units,
              int n_col_units, int n_aux, const void* Q, const void* K, const void* V, const void* O, const void* dO,
              const float* lse_in, void* dQ, void* dK, void* dV, float scale, float* ws, cudaStream_t st) {
  const int64_t rows = static_cast<int64_t>(heads) * seq;
  float* lse2 = ws;
  float* delta = ws + rows;
  float* slots = ws + 2 * rows;
  {
    const int64_t n = rows * (HD / 8);
    attn_bwd_delta_kernel<HD><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(rows, (const __nv_bfloat16*)O,
                                                                          (const __nv_bfloat16*)dO, delta);
    TSB_CHECK_LAUNCH("attention_backward_tc: delta");
  }
  if (lse_in == nullptr) {
    // no saved log-sum-exp: rerun the forward for it, with dQ as the scratch output (overwritten below)
    int rc = trnsparse_bsr_attention_tc_lse(heads, seq, HD, rp, ci, Q, K, V, dQ, lse2, (double)scale, st);
    if (rc) return rc;
  } else {
    lse2 = const_cast<float*>(lse_in);
  }
  CUtensorMap maps[4];
  const void* bases[4] = {Q, K, V, dO};
  for (int i = 0; i < 4; ++i) {
    int rc = make_tmap_2d(&maps[i], bases[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, HD, rows, HD * 2, 64, 128);
    if (rc) return rc;
  }
  const int4* aux = plan + n_row_units + n_col_units;
  if (n_aux > 0) {
    attn_bwd_aux_kernel<HD, true><<<dim3(n_aux, heads), 256, 0, st>>>(aux, heads, seq, slots, (__nv_bfloat16*)dQ,
                                                                     (__nv_bfloat16*)dK, (__nv_bfloat16*)dV);
    TSB_CHECK_LAUNCH("attention_backward_tc: zero slots");
  }
  int rc = launch_ab_mode<HD, false>(maps, plan, n_row_units, ci, heads, seq, lse2, delta, dQ, dQ, slots, scale, st);
  if (rc) return rc;
  rc = launch_ab_mode<HD, true>(maps, plan + n_row_units, n_col_units, ri, heads, seq, lse2, delta, dK, dV, slots,
                                scale, st);
  if (rc) return rc;
  if (n_aux > 0) {
    attn_bwd_aux_kernel<HD, false><<<dim3(n_aux, heads), 256, 0, st>>>(aux, heads, seq, slots, (__nv_bfloat16*)dQ,
                                                                      (__nv_bfloat16*)dK, (__nv_bfloat16*)dV);
    TSB_CHECK_LAUNCH("attention_backward_tc: finish");
  }
  return debug_sync(st, "attention_backward_tc (sync)");
}

}  // namespace
}  // namespace tsb

using namespace tsb;

namespace {
// Appends one mode's units (longest first) and aux entries; returns the slot count used.
void plan_mode(int mode, int64_t n_fixed, const int* ptr, int split, std::vector<int>& units, std::vector<int>& aux,
               int& slots) {
  std::vector<std::pair<int, int>> order;  // (length, fixed block)
  for (int64_t f = 0; f < n_fixed; ++f) {
    const int len = ptr[f + 1] - ptr[f];
    if (len == 0) {
      aux.insert(aux.end(), {mode, (int)f, -1, 0});
      continue;
    }
    order.emplace_back(len, (int)f);
  }
  std::stable_sort(order.begin(), order.end(), [](const std::pair<int, int>& a, const std::pair<int, int>& b) {
    return a.first > b.first;
  });
  std::vector<int> chunks;  // (fixed, begin, end, slot) before the length sort of the pieces
  for (const auto& o : order) {
    const int f = o.second, b0 = ptr[f], len = o.first;
    int slot = -1;
    if (len > split) {
      slot = slots++;
      aux.insert(aux.end(), {mode, f, slot, 0});
    }
    for (int b = 0; b < len; b += split) chunks.insert(chunks.end(), {f, b0 + b, b0 + std::min(len, b + split), slot});
  }
  // longest pieces first
  std::vector<int> idx(chunks.size() / 4);
  for (size_t i = 0; i < idx.size(); ++i) idx[i] = (int)i;
  std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) {
    return chunks[4 * a + 2] - chunks[4 * a + 1] > chunks[4 * b + 2] - chunks[4 * b + 1];
  });
  for (int i : idx) units.insert(units.end(), chunks.begin() + 4 * i, chunks.begin() + 4 * i + 4);
}
}  // namespace

extern "C" int trnsparse_bsr_attention_backward_tc_plan(int64_t n_block_rows, int64_t n_block_cols,
                                                        const int* block_row_ptr, const int* block_col_ptr,
                                                        int split, int* plan, int64_t plan_capacity,
                                                        int64_t* counts) {
  TSB_REQUIRE(n_block_rows >= 0 && n_block_cols >= 0 && block_row_ptr && block_col_ptr && counts,
              "attention_backward_tc_plan: bad arguments");
  TSB_REQUIRE(split > 0, "attention_backward_tc_plan: split must be positive");
  std::vector<int> ru, cu, aux;
  int slots = 0;
  plan_mode(0, n_block_rows, block_row_ptr, split, ru, aux, slots);
  plan_mode(1, n_block_cols, block_col_ptr, split, cu, aux, slots);
  counts[0] = (int64_t)ru.size() / 4;
  counts[1] = (int64_t)cu.size() / 4;
  counts[2] = (int64_t)aux.size() / 4;
  counts[3] = slots;
  const int64_t need = (int64_t)(ru.size() + cu.size() + aux.size());
  if (plan == nullptr) return TRNSPARSE_OK;
  TSB_REQUIRE(plan_capacity >= need, "attention_backward_tc_plan: capacity %lld < %lld", (long long)plan_capacity,
              (long long)need);
  int* p = plan;
  for (const auto* v : {&ru, &cu, &aux}) p = std::copy(v->begin(), v->end(), p);
  return TRNSPARSE_OK;
}

extern "C" size_t trnsparse_bsr_attention_backward_tc_workspace_size(int64_t heads, int64_t seq, int64_t head_dim,
                                                                    int64_t n_slots) {
  if (heads < 0 || seq < 0 || head_dim < 0 || n_slots < 0) return 0;
  return sizeof(float) * (2 * (size_t)heads * (size_t)seq + (size_t)n_slots * heads * 2 * 128 * (size_t)head_dim);
}

extern "C" int trnsparse_bsr_attention_backward_tc(int64_t heads, int64_t seq, int64_t head_dim,
                                                   const int* block_row_ptr, const int* block_col_idx,
                                                   const int* block_row_idx, const int* plan, int n_row_units,
                                                   int n_col_units, int n_aux, int n_slots, const void* Q,
                                                   const void* K, const void* V, const void* O, const void* dO,
                                                   const float* lse, void* dQ, void* dK, void* dV, double scale,
                                                   void* ws, size_t ws_bytes, void* stream) {
  TSB_REQUIRE(heads > 0 && seq > 0 && seq % 128 == 0 && heads < 65536 && heads * seq < (1ll << 31),
              "attention_backward_tc: needs seq %% 128 == 0 (got heads=%lld seq=%lld)", (long long)heads,
              (long long)seq);
  TSB_REQUIRE(head_dim == 64 || head_dim == 128, "attention_backward_tc: head_dim must be 64 or 128 (got %lld)",
              (long long)head_dim);
  TSB_REQUIRE(Q && K && V && O && dO && dQ && dK && dV && block_row_ptr && block_col_idx && block_row_idx && plan &&
                  ws,
              "attention_backward_tc: null pointer");
  TSB_REQUIRE(n_row_units >= 0 && n_col_units >= 0 && n_aux >= 0 && n_slots >= 0,
              "attention_backward_tc: bad plan counts");
  TSB_REQUIRE(ws_bytes >= trnsparse_bsr_attention_backward_tc_workspace_size(heads, seq, head_dim, n_slots),
              "attention_backward_tc: workspace too small");
  TSB_REQUIRE((reinterpret_cast<uintptr_t>(plan) & 15u) == 0 && (reinterpret_cast<uintptr_t>(ws) & 15u) == 0 &&
                  (reinterpret_cast<uintptr_t>(lse) & 15u) == 0,
              "attention_backward_tc: plan, workspace and lse must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  const int4* pl = reinterpret_cast<const int4*>(plan);
  float* w = static_cast<float*>(ws);
  if (head_dim == 64)
    return launch_ab<64>((int)heads, (int)seq, block_row_ptr, block_col_idx, block_row_idx, pl, n_row_units,
                         n_col_units, n_aux, Q, K, V, O, dO, lse, dQ, dK, dV, (float)scale, w, st);
  return launch_ab<128>((int)heads, (int)seq, block_row_ptr, block_col_idx, block_row_idx, pl, n_row_units,
                        n_col_units, n_aux, Q, K, V, O, dO, lse, dQ, dK, dV, (float)scale, w, st);
}

#ifdef TSB_TC_TRACE
extern "C" __attribute__((visibility("default"))) int trnsparse_ab_trace_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, tsb::g_ab_trace, sizeof(tsb::g_ab_trace));
}
#endif
