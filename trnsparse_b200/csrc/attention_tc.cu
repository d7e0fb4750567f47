// Block-sparse attention forward on the tensor cores (bf16 in/out, fp32
// softmax), block size 128, head_dim 64 or 128.
//
// Semantics are the reference's (trnsparse/ops.py:280-357 and 549-625):
// O = exp(s - rowmax) / max(rowsum, 1e-12) @ V with s = scale * q.k over the
// stored key blocks of the query block. The kernel computes it in one pass
// with an online softmax whose running max is only moved when a block's max
// exceeds it by more than 2^8 (in base-2 exponent units), so P = 2^(s2 - m)
// stays <= 256 and the output accumulator O, which lives in TMEM, is
// rescaled only on those rare steps. Numerator and denominator use the same
// m, so the quotient equals the reference's up to rounding.
//
// Persistent CTAs (one per SM) walk the (head, 128-row query block) tiles
// round robin; 10 warps:
//   warp 8      TMA producer: per tile Q, then K and V of every stored key
//               block into a 3-stage K ring and a 2-stage V ring (128-byte
//               swizzle); K runs ahead of V because S = Q K^T is issued a
//               step before P V. Polls its barriers without blocking.
//   warp 9      TMEM owner and MMA issuer: S = Q K^T into one of two TMEM
//               score buffers (S of block j+1 is issued before O += P_j V_j,
//               so the tensor core works while the softmax warps do); P V
//               takes P straight from TMEM (A operand) and V MN-major from
//               its row-major layout. A tile's last P V is issued before
//               waiting for the next tile's Q.
//   warps 0-7   softmax: warp w reads TMEM lanes 32 (w % 4) .. +31 (one query
//               row per thread) and score columns 64 (w / 4) .. +63; the two
//               halves of a row exchange their block max (and at the end the
//               denominators) through shared memory, write P as packed bf16
//               into one of two TMEM P buffers, rescale O in TMEM when the
//               max moved, and at the end of a tile stage O / l as bf16 in
//               shared memory for one TMA store per warp.
// All waits are bounded (ptx.cuh), the exchanges between the softmax warps
// included, so a stalled partner ends in an error record, never a hang.
#include <cuda_bf16.h>

#include "tc_common.cuh"

namespace tsb {
namespace {

constexpr int kAtSoftmax = 256;                 // softmax threads (warps 0-7)
constexpr int kAtThreads = kAtSoftmax + 64;     // + producer warp + MMA warp
constexpr float kRescaleLog2 = 8.f;             // move the max only when it grows by > 2^8

#ifdef TSB_TC_TRACE
__device__ unsigned long long g_at_trace[4][128];
__device__ __forceinline__ unsigned long long at_time() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// (query block 64 of head 0 only) slot: 0 = softmax, 1 = MMA issuer, 2 = producer
#define AT_TRACE(who, i) \
  if (blockIdx.x == 64 && (i) < 128) g_at_trace[who][i] = at_time()
#else
#define AT_TRACE(who, i)
#endif

template <int HD>
struct AtLayout {
  static constexpr int kChunks = HD / 64;          // 128-byte column chunks of a Q/K/V row
  static constexpr int kTile = 128 * HD * 2;       // bytes of one 128-row Q/K/V/O tile
  static constexpr int kKStages = 3;
  static constexpr int kVStages = 2;
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kTile;
  static constexpr int kV = kK + kKStages * kTile;
  static constexpr int kOst = kV + kVStages * kTile;  // O staging for the TMA store
  static constexpr int kX = kOst + kTile;             // float [2][2][128] row exchange
  static constexpr int kBar = kX + 2 * 2 * 128 * 4;   // mbarriers, TMEM slot, abort flag
  static constexpr int kSmem = kBar + 256;
  // TMEM columns: S0 [0,128), S1 [128,256), O [256, 256+HD), P0 [384,448), P1 [448,512)
  static constexpr int kTmemCols = 512;
  static constexpr uint32_t kTmemO = 256, kTmemP = 384;
};

struct AtBars {
  uint64_t q_full, q_empty, o_done;
  uint64_t k_full[3], k_empty[3], v_full[2], v_empty[2];
  uint64_t s_full[2], s_empty[2], p_full, p_empty[2], x_bar[2];
  uint32_t tmem_slot;
  int abort_flag;
};

// 2^x on the special-function unit (PTX ex2.approx.ftz.f32).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// Tile t -> (head, query block). Head-minor order: the CTAs running at the same time work
// on all heads at once, so the K/V tiles of one head (the global key blocks above all,
// which every query block of the head reads) are not all fetched at the same moment
// (config 4: 0.212 -> 0.207 ms; query blocks in descending order measured slower).
__device__ __forceinline__ void at_tile(int t, int m_tiles, int n_tiles, int& head, int& qb) {
  const int heads = n_tiles / m_tiles;
  qb = t / heads;
  head = t - qb * heads;
}

// Walks this CTA's tiles (round robin over the grid), skipping empty block-rows,
// and the stored key blocks of each.
struct TileCursor {
  const int* row_ptr;
  int m_tiles, n_tiles, stride;
  int t, j, nb, e0, head, qb;
  bool valid;
  __device__ void seek(int from) {
    for (t = from; t < n_tiles; t += stride) {
      at_tile(t, m_tiles, n_tiles, head, qb);
      e0 = row_ptr[qb];
      nb = row_ptr[qb + 1] - e0;
      if (nb > 0) {
        j = 0;
        valid = true;
        return;
      }
    }
    valid = false;
  }
  __device__ void advance() {
    if (++j == nb) seek(t + stride);
  }
};

template <int HD>
__global__ void __launch_bounds__(kAtThreads, 1)
attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
               const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap to,
               const int* __restrict__ row_ptr, const int* __restrict__ col_idx, __nv_bfloat16* __restrict__ O,
               float* __restrict__ lse, int seq, int m_tiles, int n_tiles, float scale) {
  using Lay = AtLayout<HD>;
  // No static shared memory: the dynamic window then starts 1024-byte aligned, which the
  // 128-byte-swizzled tiles need (checked below; a misaligned base aborts with an error record).
  extern __shared__ __align__(16) uint8_t sb[];
  AtBars& B = *reinterpret_cast<AtBars*>(sb + Lay::kBar);
  float (*x_ex)[2][128] = reinterpret_cast<float (*)[2][128]>(sb + Lay::kX);
  const int warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    mbar_init(&B.q_full, 1);
    mbar_init(&B.q_empty, 1);
    mbar_init(&B.o_done, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&B.k_full[i], 1);
      mbar_init(&B.k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&B.v_full[i], 1);
      mbar_init(&B.v_empty[i], 1);
      mbar_init(&B.s_full[i], 1);
      mbar_init(&B.s_empty[i], kAtSoftmax);
      mbar_init(&B.p_empty[i], 1);
      mbar_init(&B.x_bar[i], kAtSoftmax);
    }
    mbar_init(&B.p_full, kAtSoftmax);
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
  const uint32_t t_o = tmem + Lay::kTmemO;
  volatile int* abort_flag = &B.abort_flag;

  // Persistent CTAs; every role walks the same tile list. Tiles without stored blocks are
  // written as zeros by the softmax warps and skipped by the others. Pipeline positions run
  // on across tiles: g counts key blocks, nt non-empty tiles.
  if (warp == 8) {
    // ---------------- TMA producer: K runs ahead of V (S = Q K^T comes a step before P V)
    if (elect_lane0() && !*abort_flag) {
      TileCursor kc{row_ptr, m_tiles, n_tiles, (int)gridDim.x}, vc = kc;
      kc.seek(blockIdx.x);
      vc.seek(blockIdx.x);
      int gk = 0, gv = 0, ntk = 0;
      uint64_t idle_since = 0;
      while (vc.valid && !*abort_flag) {
        bool moved = false;
        if (kc.valid) {
          const int st = gk % Lay::kKStages, u = gk / Lay::kKStages;
          bool ready = u == 0 || mbar_test_wait(&B.k_empty[st], (u - 1) & 1);
          if (ready && kc.j == 0 && ntk > 0) ready = mbar_test_wait(&B.q_empty, (ntk - 1) & 1);
          if (ready) {
            const int row0 = kc.head * seq;
            if (kc.j == 0) {
              mbar_arrive_expect_tx(&B.q_full, Lay::kTile);
              for (int c = 0; c < Lay::kChunks; ++c)
                tma_load_2d(sb + Lay::kQ + c * 16384, &tq, c * 64, row0 + kc.qb * 128, &B.q_full);
              ++ntk;
            }
            AT_TRACE(2, gk);
            const int krow = row0 + col_idx[kc.e0 + kc.j] * 128;
            mbar_arrive_expect_tx(&B.k_full[st], Lay::kTile);
            for (int c = 0; c < Lay::kChunks; ++c)
              tma_load_2d(sb + Lay::kK + st * Lay::kTile + c * 16384, &tk, c * 64, krow, &B.k_full[st]);
            ++gk;
            kc.advance();
            moved = true;
          }
        }
        if (gv < gk) {
          const int st = gv & 1, u = gv >> 1;
          if (u == 0 || mbar_test_wait(&B.v_empty[st], (u - 1) & 1)) {
            AT_TRACE(3, 64 + gv);
            const int vrow = vc.head * seq + col_idx[vc.e0 + vc.j] * 128;
            mbar_arrive_expect_tx(&B.v_full[st], Lay::kTile);
            for (int c = 0; c < Lay::kChunks; ++c)
              tma_load_2d(sb + Lay::kV + st * Lay::kTile + c * 16384, &tv, c * 64, vrow, &B.v_full[st]);
            ++gv;
            vc.advance();
            moved = true;
          }
        }
        if (moved) {
          idle_since = 0;
        } else if (idle_since == 0) {
          idle_since = global_ns();
        } else if (global_ns() - idle_since > kWaitNs) {
          record_device_error(DEVERR_MBAR_TIMEOUT);
          atomicExch(&B.abort_flag, 1);
          break;
        }
      }
    }
  } else if (warp == 9) {
    // ---------------- MMA issuer
    if (elect_lane0()) {
      constexpr uint32_t idesc_s = make_idesc(MmaKind::BF16, 128, 128);
      constexpr uint32_t idesc_o = make_idesc(MmaKind::BF16, 128, HD) | (1u << 16);  // B (V) MN-major
      const uint32_t q_addr = smem_u32(sb + Lay::kQ);
      // O += P_g V_g (P from TMEM) for block g (j = its index in the tile); `last` closes the tile
      auto issue_pv = [&](int g, int j, bool last) {
        const int b = g & 1, u = g >> 1;
        if (!mbar_wait(&B.p_full, g & 1) || !mbar_wait(&B.v_full[b], u & 1)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sb + Lay::kV + b * Lay::kTile);
        const uint32_t p_tm = tmem + Lay::kTmemP + b * 64;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // 128 keys, 16 per MMA (8 packed TMEM columns)
          umma_ts_f16(t_o, p_tm + kk * 8, smem_desc_sw128_mn(v_addr + kk * 2048, 16384), idesc_o, j > 0 || kk > 0);
        umma_commit(&B.v_empty[b]);
        umma_commit(&B.p_empty[b]);
        if (last) umma_commit(&B.o_done);
        return true;
      };
      TileCursor tc{row_ptr, m_tiles, n_tiles, (int)gridDim.x};
      int g = 0, nt = 0, pg = -1, pj = 0;
      bool plast = false, ok = !*abort_flag;
      for (tc.seek(blockIdx.x); ok && tc.valid; ++nt) {
        // close the previous tile first: its last P V must not wait behind this tile's Q load
        if (pg >= 0 && !issue_pv(pg, pj, plast)) { ok = false; break; }
        pg = -1;
        if (!mbar_wait(&B.q_full, nt & 1)) { ok = false; break; }
        const int nb = tc.nb;
        for (int j = 0; j < nb; ++j, ++g) {
          if (*abort_flag) { ok = false; break; }
          const int ks = g % Lay::kKStages, ku = g / Lay::kKStages;
          const int sb2 = g & 1, su = g >> 1;
          if (!mbar_wait(&B.k_full[ks], ku & 1)) { ok = false; break; }
          AT_TRACE(1, 3 * g);
          if (su > 0 && !mbar_wait(&B.s_empty[sb2], (su - 1) & 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sb + Lay::kK + ks * Lay::kTile);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma<MmaKind::BF16>(tmem + sb2 * 128, smem_desc_sw128(q_addr + off), smem_desc_sw128(k_addr + off),
                                idesc_s, kk > 0);
          }
          umma_commit(&B.k_empty[ks]);
          umma_commit(&B.s_full[sb2]);
          if (j == nb - 1) umma_commit(&B.q_empty);
          AT_TRACE(1, 3 * g + 1);
          // the previous block's P V runs while the softmax warps work on this block's scores
          if (pg >= 0 && !issue_pv(pg, pj, plast)) { ok = false; break; }
          AT_TRACE(1, 3 * g + 2);
          pg = g;
          pj = j;
          plast = j == nb - 1;
        }
        if (!ok) break;
        tc.seek(tc.t + tc.stride);
      }
      if (ok && pg >= 0 && !issue_pv(pg, pj, plast)) ok = false;
      if (!ok) {
        atomicExch(&B.abort_flag, 1);
        umma_commit(&B.o_done);
      }
    }
  } else {
    // ---------------- softmax warps; scores in base-2 exponent units s2 = s * log2(e)
    const int quad = warp & 3, half = warp >> 2, lr = threadIdx.x & 31;
    const int r = quad * 32 + lr;
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const float sl = scale * 1.4426950408889634f;
    uint8_t* const stage = sb + Lay::kOst + half * (Lay::kTile / 2) + quad * (Lay::kTile / 8);
    int g = 0, nt = 0, xc = 0;  // xc: row exchanges so far (block maxima and tile denominators)
    bool ok = !*abort_flag;
    // Both halves of row r publish a value; returns the partner's. Bounded.
    auto exchange = [&](float mine, float& theirs) {
      const int b = xc & 1, u = xc >> 1;
      ++xc;
      x_ex[b][half][r] = mine;
      mbar_arrive(&B.x_bar[b]);
      if (!mbar_wait(&B.x_bar[b], u & 1)) return false;
      theirs = x_ex[b][half ^ 1][r];
      return true;
    };
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
      int head, qb;
      at_tile(t, m_tiles, n_tiles, head, qb);
      const int nb = row_ptr[qb + 1] - row_ptr[qb];
      if (nb <= 0 || !ok) {  // an empty block-row is zero (as in the reference)
        uint4* orow = reinterpret_cast<uint4*>(O + static_cast<int64_t>(head * seq + qb * 128 + r) * HD +
                                               half * (HD / 2));
#pragma unroll
        for (int q = 0; q < HD / 16; ++q) orow[q] = make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      float m = -INFINITY, l_row = 0.f;
      for (int j = 0; j < nb; ++j, ++g) {
        const int sbuf = g & 1, su = g >> 1;
        if (*abort_flag || !mbar_wait(&B.s_full[sbuf], su & 1)) { ok = false; break; }
        if (threadIdx.x == 0) AT_TRACE(0, 4 * g);
        tc_fence_after();
        uint32_t v0[32], v1[32];
        tmem_ld32(tmem + lane_base + sbuf * 128 + half * 64, v0);
        tmem_ld32(tmem + lane_base + sbuf * 128 + half * 64 + 32, v1);
        tmem_wait_ld();
        auto V = [&](int i) { return __uint_as_float(i < 32 ? v0[i] : v1[i - 32]); };
        tc_fence_before();
        mbar_arrive(&B.s_empty[sbuf]);  // scores are in registers: the MMA may refill this buffer
        // block max of this half, then of the row
        float a0, a1;
        if (sl >= 0.f) {
          a0 = a1 = -INFINITY;
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            a0 = fmaxf(a0, V(i));
            a1 = fmaxf(a1, V(i + 1));
          }
          a0 = fmaxf(a0, a1);
        } else {
          a0 = a1 = INFINITY;
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            a0 = fminf(a0, V(i));
            a1 = fminf(a1, V(i + 1));
          }
          a0 = fminf(a0, a1);
        }
        const float pmax = a0 * sl;
        float other;
        if (!exchange(pmax, other)) { ok = false; break; }
        if (threadIdx.x == 0) AT_TRACE(0, 4 * g + 1);
        const float bmax = fmaxf(pmax, other);
        const float mnew = (bmax > m + kRescaleLog2) ? bmax : m;
        const float corr = ex2_approx(m - mnew);  // 0 on the first block, 1 when m is kept
        // P = 2^(s2 - m) as bf16 pairs; partial sums in four chains
        uint32_t pk[32];
        float q0 = 0.f, q1 = 0.f, q2 = 0.f, q3 = 0.f;
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float x0 = ex2_approx(fmaf(V(2 * i), sl, -mnew));
          const float x1 = ex2_approx(fmaf(V(2 * i + 1), sl, -mnew));
          const float x2 = ex2_approx(fmaf(V(2 * i + 2), sl, -mnew));
          const float x3 = ex2_approx(fmaf(V(2 * i + 3), sl, -mnew));
          q0 += x0;
          q1 += x1;
          q2 += x2;
          q3 += x3;
          pk[i] = pack_bf16(x0, x1);
          pk[i + 1] = pack_bf16(x2, x3);
        }
        l_row = l_row * corr + ((q0 + q1) + (q2 + q3));
        if (threadIdx.x == 0) AT_TRACE(0, 4 * g + 2);
        // O may be rescaled once the previous block's P V has completed
        if (j > 0 && __any_sync(0xffffffffu, mnew != m)) {
          if (!mbar_wait(&B.p_empty[(g - 1) & 1], ((g - 1) >> 1) & 1)) { ok = false; break; }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < HD / 64; ++c) {
            const uint32_t ta = t_o + lane_base + half * (HD / 2) + c * 32;
            uint32_t o[32];
            tmem_ld32(ta, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
            tmem_st32(ta, o);
          }
        }
        m = mnew;
        // P buffer g & 1 is free once the P V of block g - 2 has completed
        if (g >= 2 && !mbar_wait(&B.p_empty[g & 1], ((g >> 1) - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        tmem_st32(tmem + lane_base + Lay::kTmemP + (g & 1) * 64 + half * 32, pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&B.p_full);
        if (threadIdx.x == 0) AT_TRACE(0, 4 * g + 3);
      }
      // ---- tile epilogue: O / l (TMEM) -> bf16 staging -> one TMA store per warp
      float l_other = 0.f;
      if (ok) ok = exchange(l_row, l_other);
      if (threadIdx.x == 0) AT_TRACE(3, 4 * nt);
      ok = ok && mbar_wait(&B.o_done, nt & 1) && !*abort_flag;
      if (threadIdx.x == 0) AT_TRACE(3, 4 * nt + 1);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      const float inv = ok ? 1.f / fmaxf(l_row + l_other, 1e-12f) : 0.f;
      // base-2 log-sum-exp of the row (scores in s * scale * log2(e) units) for the backward
      if (lse != nullptr && half == 0 && ok) lse[static_cast<int64_t>(head) * seq + qb * 128 + r] = m + log2f(l_row + l_other);
      if (lr == 0) bulk_wait_read_all();  // the previous tile's store has left the staging slice
      __syncwarp();
#pragma unroll 1
      for (int c = 0; c < HD / 64; ++c) {
        uint32_t v[32];
        if (ok) {
          tmem_ld32(t_o + lane_base + half * (HD / 2) + c * 32, v);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0u;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          auto f = [&](int i) { return __uint_as_float(v[8 * q + i]) * inv; };
          const int unit = c * 4 + q;  // 16-byte unit of the staged row
          const int pos = HD == 128 ? (unit ^ (lr & 7)) * 16 + lr * 128 : (unit ^ ((lr >> 1) & 3)) * 16 + lr * 64;
          *reinterpret_cast<uint4*>(stage + pos) = make_uint4(pack_bf16(f(0), f(1)), pack_bf16(f(2), f(3)),
                                                             pack_bf16(f(4), f(5)), pack_bf16(f(6), f(7)));
        }
      }
      tc_fence_before();  // O is read before the next tile's first P V (ordered by p_full)
      fence_proxy_async_smem();
      __syncwarp();
      if (threadIdx.x == 0) AT_TRACE(3, 4 * nt + 2);
      if (lr == 0) {
        tma_store_2d(&to, stage, half * (HD / 2), head * seq + qb * 128 + quad * 32);
        bulk_commit_group();
      }
      if (!ok) atomicExch(&B.abort_flag, 1);
      ++nt;
    }
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

template <int HD>
int launch_attn_tc(const void* Q, const void* K, const void* V, void* O, float* lse, const int* rp, const int* ci,
                   int heads, int seq, float scale, cudaStream_t st) {
  using Lay = AtLayout<HD>;
  const uint64_t rows = static_cast<uint64_t>(heads) * seq;
  CUtensorMap tq, tk, tv, to;
  const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  int rc = make_tmap_2d(&tq, Q, dt, HD, rows, HD * 2, 64, 128);
  if (rc) return rc;
  rc = make_tmap_2d(&tk, K, dt, HD, rows, HD * 2, 64, 128);
  if (rc) return rc;
  rc = make_tmap_2d(&tv, V, dt, HD, rows, HD * 2, 64, 128);
  if (rc) return rc;
  // O is stored per softmax warp: 32 rows x HD/2 columns (HD bytes: 128- or 64-byte swizzle)
  rc = make_tmap_2d(&to, O, dt, HD, rows, HD * 2, HD / 2, 32,
                    HD == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  auto kern = attn_tc_kernel<HD>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kSmem);
  if (e != cudaSuccess) return cuda_status(e, "attention_tc: set smem");
  const int m_tiles = seq / 128;
  const int n_tiles = m_tiles * heads;
  const int grid = n_tiles < sm_count() ? n_tiles : sm_count();
  kern<<<grid, kAtThreads, Lay::kSmem, st>>>(tq, tk, tv, to, rp, ci, (__nv_bfloat16*)O, lse, seq, m_tiles, n_tiles,
                                                scale);
  TSB_CHECK_LAUNCH("attention_tc launch");
  return debug_sync(st, "attention_tc (sync)");
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" int trnsparse_bsr_attention_tc_lse(int64_t heads, int64_t seq, int64_t head_dim,
                                              const int* block_row_ptr, const int* block_col_idx, const void* Q,
                                              const void* K, const void* V, void* O, float* lse, double scale,
                                              void* stream) {
  TSB_REQUIRE(heads > 0 && seq > 0 && seq % 128 == 0 && heads < 65536 && heads * seq < (1ll << 31),
              "attention_tc: needs seq %% 128 == 0 (got heads=%lld seq=%lld)", (long long)heads, (long long)seq);
  TSB_REQUIRE(head_dim == 64 || head_dim == 128, "attention_tc: head_dim must be 64 or 128 (got %lld)",
              (long long)head_dim);
  TSB_REQUIRE(Q && K && V && O && block_row_ptr && block_col_idx, "attention_tc: null pointer");
  cudaStream_t st = as_stream(stream);
  if (head_dim == 64)
    return launch_attn_tc<64>(Q, K, V, O, lse, block_row_ptr, block_col_idx, (int)heads, (int)seq, (float)scale, st);
  return launch_attn_tc<128>(Q, K, V, O, lse, block_row_ptr, block_col_idx, (int)heads, (int)seq, (float)scale, st);
}

extern "C" int trnsparse_bsr_attention_tc(int64_t heads, int64_t seq, int64_t head_dim, const int* block_row_ptr,
                                          const int* block_col_idx, const void* Q, const void* K, const void* V,
                                          void* O, double scale, void* stream) {
  return trnsparse_bsr_attention_tc_lse(heads, seq, head_dim, block_row_ptr, block_col_idx, Q, K, V, O, nullptr,
                                        scale, stream);
}

#ifdef TSB_TC_TRACE
extern "C" __attribute__((visibility("default"))) int trnsparse_at_trace_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, tsb::g_at_trace, sizeof(tsb::g_at_trace));
}
#endif
