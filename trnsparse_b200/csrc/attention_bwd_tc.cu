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
// Per partner block the MMA warp issues S = F1 X1^T and dP = F2 X2^T
// (128x128, K = head_dim) into TMEM columns [0,128) and [128,256); eight
// warps read them (one TMEM lane = one fixed row per thread, 64 columns per
// warp half), form P and dS in fp32 and write them back as packed bf16 into
// the columns they just read; the MMA warp then adds dS X1 (and, in column
// mode, P X2) into the TMEM accumulators at column 256 (+ head_dim) with A
// taken from TMEM and the streamed tile as an MN-major B. At the end of a
// unit the same eight warps scale the accumulators, stage them as bf16 in the
// fixed tiles' shared memory and write them with TMA stores; units of a
// block that was split over several CTAs add fp32 partial sums into a
// workspace slot instead, converted by a finishing kernel.
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

constexpr int kAbEpi = 256;               // dS / epilogue threads (warps 0-7)
constexpr int kAbThreads = kAbEpi + 64;   // + producer warp + MMA warp

template <int HD>
struct AbLayout {
  static constexpr int kChunks = HD / 64;       // 128-byte column chunks of a row
  static constexpr int kTile = 128 * HD * 2;    // one 128-row bf16 tile
  static constexpr int kF1 = 0, kF2 = kTile;    // fixed tiles (also the output staging)
  static constexpr int kX = 2 * kTile;          // streamed stages: X1, X2, lse[128], D[128]
  static constexpr int kStage = 2 * kTile + 1024;
  static constexpr int kStages = 2;
  static constexpr int kBar = kX + kStages * kStage;
  static constexpr int kSmem = kBar + 256;
  static constexpr uint32_t kTmemS = 0, kTmemDP = 128, kTmemAcc = 256;  // accumulators at 256 (+HD)
  static constexpr int kTmemCols = 512;
};

struct AbBars {
  uint64_t f_full, f_empty, acc_full, acc_empty;
  uint64_t x_full[2], x_empty[2];
  uint64_t s_full, p_full, mma_done;
  uint32_t tmem_slot;
  int abort_flag;
};

__device__ __forceinline__ float ab_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// units: {fixed block, first partner index, end partner index, workspace slot or -1}.
// Tile t covers unit t / heads of head t % heads (heads of a long unit run side by side).
template <int HD, bool COL>
__global__ void __launch_bounds__(kAbThreads, 1)
attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tf1, const __grid_constant__ CUtensorMap tf2,
                   const __grid_constant__ CUtensorMap tx1, const __grid_constant__ CUtensorMap tx2,
                   const __grid_constant__ CUtensorMap to1, const __grid_constant__ CUtensorMap to2,
                   const int4* __restrict__ units, const int* __restrict__ partner, int n_tiles, int heads,
                   int seq, const float* __restrict__ lse2, const float* __restrict__ delta,
                   float* __restrict__ slots, float scale) {
  using Lay = AbLayout<HD>;
  extern __shared__ __align__(16) uint8_t sb[];  // no static smem: the window is 1024-byte aligned
  AbBars& B = *reinterpret_cast<AbBars*>(sb + Lay::kBar);
  const int warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    mbar_init(&B.f_full, 1);
    mbar_init(&B.f_empty, kAbEpi / 32);
    mbar_init(&B.acc_full, 1);
    mbar_init(&B.acc_empty, kAbEpi);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.x_full[i], 1);
      mbar_init(&B.x_empty[i], 1);
    }
    mbar_init(&B.s_full, 1);
    mbar_init(&B.p_full, kAbEpi);
    mbar_init(&B.mma_done, 1);
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
    // ---------------- TMA producer
    if (elect_lane0() && !*abort_flag) {
      int gs = 0, nt = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x, ++nt) {
        const int4 u = units[t / heads];
        const int row0 = (t % heads) * seq;
        if (nt > 0 && !mbar_wait(&B.f_empty, (nt - 1) & 1)) { ok = false; break; }
        mbar_arrive_expect_tx(&B.f_full, 2 * Lay::kTile);
        for (int c = 0; c < Lay::kChunks; ++c) {
          tma_load_2d(sb + Lay::kF1 + c * 16384, &tf1, c * 64, row0 + u.x * 128, &B.f_full);
          tma_load_2d(sb + Lay::kF2 + c * 16384, &tf2, c * 64, row0 + u.x * 128, &B.f_full);
        }
        for (int e = u.y; e < u.z; ++e, ++gs) {
          const int st = gs & 1, use = gs >> 1;
          if (*abort_flag || (use > 0 && !mbar_wait(&B.x_empty[st], (use - 1) & 1))) { ok = false; break; }
          const int pb = partner[e];
          const int xrow = row0 + pb * 128;
          uint8_t* xs = sb + Lay::kX + st * Lay::kStage;
          mbar_arrive_expect_tx(&B.x_full[st], 2 * Lay::kTile + (COL ? 1024 : 0));
          for (int c = 0; c < Lay::kChunks; ++c) {
            tma_load_2d(xs + c * 16384, &tx1, c * 64, xrow, &B.x_full[st]);
            tma_load_2d(xs + Lay::kTile + c * 16384, &tx2, c * 64, xrow, &B.x_full[st]);
          }
          if (COL) {
            const int vrow = (pb >= 0 && pb * 128 < seq) ? xrow : row0;  // never read past the statistics
            bulk_g2s(xs + 2 * Lay::kTile, lse2 + vrow, 512, &B.x_full[st]);
            bulk_g2s(xs + 2 * Lay::kTile + 512, delta + vrow, 512, &B.x_full[st]);
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
      int gs = 0, nt = 0;
      bool ok = !*abort_flag;
      for (int t = blockIdx.x; ok && t < n_tiles; t += gridDim.x, ++nt) {
        const int4 u = units[t / heads];
        if (!mbar_wait(&B.f_full, nt & 1)) { ok = false; break; }
        for (int e = u.y; e < u.z; ++e, ++gs) {
          const int st = gs & 1, use = gs >> 1;
          if (*abort_flag || !mbar_wait(&B.x_full[st], use & 1)) { ok = false; break; }
          // the previous block's products have read P / dS out of the score columns
          if (gs > 0 && !mbar_wait(&B.mma_done, (gs - 1) & 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t x1 = smem_u32(sb + Lay::kX + st * Lay::kStage), x2 = x1 + Lay::kTile;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma<MmaKind::BF16>(tmem + Lay::kTmemS, smem_desc_sw128(f1 + off), smem_desc_sw128(x1 + off), idesc_s,
                                kk > 0);
            umma<MmaKind::BF16>(tmem + Lay::kTmemDP, smem_desc_sw128(f2 + off), smem_desc_sw128(x2 + off), idesc_s,
                                kk > 0);
          }
          umma_commit(&B.s_full);
          if (!mbar_wait(&B.p_full, gs & 1)) { ok = false; break; }
          if (e == u.y && nt > 0 && !mbar_wait(&B.acc_empty, (nt - 1) & 1)) { ok = false; break; }
          tc_fence_after();
          const bool acc = e > u.y;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {  // 128 partner rows, 16 per MMA (8 packed TMEM columns)
            const uint32_t a_col = (kk >> 2) * 64 + (kk & 3) * 8;
            umma_ts_f16(tmem + Lay::kTmemAcc, tmem + Lay::kTmemDP + a_col, smem_desc_sw128_mn(x1 + kk * 2048, 16384),
                        idesc_a, acc || kk > 0);
            if (COL)
              umma_ts_f16(tmem + Lay::kTmemAcc + HD, tmem + Lay::kTmemS + a_col,
                          smem_desc_sw128_mn(x2 + kk * 2048, 16384), idesc_a, acc || kk > 0);
          }
          umma_commit(&B.x_empty[st]);
          umma_commit(&B.mma_done);
          if (e == u.z - 1) umma_commit(&B.acc_full);
        }
      }
      if (!ok) atomicExch(&B.abort_flag, 1);
    }
  } else {
    // ---------------- dS and epilogue warps
    const int quad = warp & 3, half = warp >> 2, lr = threadIdx.x & 31;
    const int r = quad * 32 + lr;  // fixed row of this thread (TMEM lane)
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
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
        const int st = gs & 1;
        if (*abort_flag || !mbar_wait(&B.s_full, gs & 1)) { ok = false; break; }
        const float* vl = reinterpret_cast<const float*>(sb + Lay::kX + st * Lay::kStage + 2 * Lay::kTile);
        if (COL && !mbar_wait(&B.x_full[st], (gs >> 1) & 1)) { ok = false; break; }  // lse / D of the partner rows
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const uint32_t col = half * 64 + c * 32;
          uint32_t s[32], dp[32];
          tmem_ld32(tmem + lane_base + Lay::kTmemS + col, s);
          tmem_ld32(tmem + lane_base + Lay::kTmemDP + col, dp);
          tmem_wait_ld();
          uint32_t pp[16], pd[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            float l0 = l_r, l1 = l_r, d0 = d_r, d1 = d_r;
            if (COL) {
              l0 = vl[col + i];
              l1 = vl[col + i + 1];
              d0 = vl[128 + col + i];
              d1 = vl[128 + col + i + 1];
            }
            const float p0 = ab_ex2(fmaf(__uint_as_float(s[i]), sl, -l0));
            const float p1 = ab_ex2(fmaf(__uint_as_float(s[i + 1]), sl, -l1));
            pp[i / 2] = pack_bf16(p0, p1);
            pd[i / 2] = pack_bf16(p0 * (__uint_as_float(dp[i]) - d0), p1 * (__uint_as_float(dp[i + 1]) - d1));
          }
          // packed bf16 back into the columns just read: A operands of the products
          if (COL) tmem_st16(tmem + lane_base + Lay::kTmemS + half * 64 + c * 16, pp);
          tmem_st16(tmem + lane_base + Lay::kTmemDP + half * 64 + c * 16, pd);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&B.p_full);
      }
      if (!ok) break;
      // ---- unit epilogue: accumulators -> bf16 staging in the fixed tiles -> TMA stores
      if (!mbar_wait(&B.acc_full, nt & 1)) { ok = false; break; }
      tc_fence_after();
      const int slot = u.w;
#pragma unroll 1
      for (int a = 0; a < (COL ? 2 : 1); ++a) {
        const float mul = a == 0 ? scale : 1.f;
        uint8_t* const stage = sb + (a == 0 ? Lay::kF1 : Lay::kF2) + half * (Lay::kTile / 2) + quad * (Lay::kTile / 8);
        float* const wrow =
            slot >= 0 ? slots + ((static_cast<int64_t>(slot) * heads + head) * 2 + a) * 128 * HD + r * HD + half * (HD / 2)
                      : nullptr;
#pragma unroll 1
        for (int c = 0; c < HD / 64; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_base + Lay::kTmemAcc + a * HD + half * (HD / 2) + c * 32, v);
          tmem_wait_ld();
          if (slot >= 0) {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              red_add_v4(wrow + c * 32 + 4 * q, __float_as_uint(__uint_as_float(v[4 * q]) * mul),
                         __float_as_uint(__uint_as_float(v[4 * q + 1]) * mul),
                         __float_as_uint(__uint_as_float(v[4 * q + 2]) * mul),
                         __float_as_uint(__uint_as_float(v[4 * q + 3]) * mul));
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              auto f = [&](int i) { return __uint_as_float(v[8 * q + i]) * mul; };
              const int unit = c * 4 + q;  // 16-byte unit of the staged row
              const int pos =
                  HD == 128 ? (unit ^ (lr & 7)) * 16 + lr * 128 : (unit ^ ((lr >> 1) & 3)) * 16 + lr * 64;
              *reinterpret_cast<uint4*>(stage + pos) = make_uint4(pack_bf16(f(0), f(1)), pack_bf16(f(2), f(3)),
                                                                 pack_bf16(f(4), f(5)), pack_bf16(f(6), f(7)));
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&B.acc_empty);  // accumulators read: the next unit's products may start
      if (slot < 0) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lr == 0) {
          const int orow = head * seq + u.x * 128 + quad * 32;
          tma_store_2d(&to1, sb + Lay::kF1 + half * (Lay::kTile / 2) + quad * (Lay::kTile / 8), half * (HD / 2), orow);
          if (COL)
            tma_store_2d(&to2, sb + Lay::kF2 + half * (Lay::kTile / 2) + quad * (Lay::kTile / 8), half * (HD / 2),
                         orow);
          bulk_commit_group();
          bulk_wait_read_all();  // staging (the fixed tiles) may be refilled
        }
      }
      __syncwarp();
      if (lr == 0) mbar_arrive(&B.f_empty);
    }
    if (!ok) atomicExch(&B.abort_flag, 1);
    if (lr == 0) bulk_wait_all();
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
                   const float* lse2, const float* delta, float* slots, float scale, cudaStream_t st) {
  if (n_units <= 0) return TRNSPARSE_OK;
  using Lay = AbLayout<HD>;
  auto kern = attn_bwd_tc_kernel<HD, COL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kSmem);
  if (e != cudaSuccess) return cuda_status(e, "attention_backward_tc: set smem");
  const int64_t n_tiles = static_cast<int64_t>(n_units) * heads;
  const int grid = n_tiles < sm_count() ? (int)n_tiles : sm_count();
  // maps: 0 Q, 1 K, 2 V, 3 dO, 4 dQ, 5 dK, 6 dV
  if (COL)
    kern<<<grid, kAbThreads, Lay::kSmem, st>>>(maps[1], maps[2], maps[0], maps[3], maps[5], maps[6], units, partner,
                                               (int)n_tiles, heads, seq, lse2, delta, slots, scale);
  else
    kern<<<grid, kAbThreads, Lay::kSmem, st>>>(maps[0], maps[3], maps[1], maps[2], maps[4], maps[4], units, partner,
                                               (int)n_tiles, heads, seq, lse2, delta, slots, scale);
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
  CUtensorMap maps[7];
  const void* bases[7] = {Q, K, V, dO, dQ, dK, dV};
  const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  for (int i = 0; i < 7; ++i) {
    int rc = i < 4 ? make_tmap_2d(&maps[i], bases[i], dt, HD, rows, HD * 2, 64, 128)
                   : make_tmap_2d(&maps[i], bases[i], dt, HD, rows, HD * 2, HD / 2, 32,
                                  HD == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc) return rc;
  }
  const int4* aux = plan + n_row_units + n_col_units;
  if (n_aux > 0) {
    attn_bwd_aux_kernel<HD, true><<<dim3(n_aux, heads), 256, 0, st>>>(aux, heads, seq, slots, (__nv_bfloat16*)dQ,
                                                                     (__nv_bfloat16*)dK, (__nv_bfloat16*)dV);
    TSB_CHECK_LAUNCH("attention_backward_tc: zero slots");
  }
  int rc = launch_ab_mode<HD, false>(maps, plan, n_row_units, ci, heads, seq, lse2, delta, slots, scale, st);
  if (rc) return rc;
  rc = launch_ab_mode<HD, true>(maps, plan + n_row_units, n_col_units, ri, heads, seq, lse2, delta, slots, scale, st);
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
