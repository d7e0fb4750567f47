// Schwarz-screened dense x dense on the tensor cores: C = (A o mask) @ B.
//
// Reference: trnsparse/ops.py:213-277 (`screened_spmm`, 1-D bound vector:
// Q = sqrt(|diag|), mask[i,j] = Q[i]*Q[j] > sqrt(threshold)) and the 2-D
// pair-bound form of trnsparse/screening.py:29-40 (`screen_quartets`:
// mask = sqrt(threshold) < Q). The NKI kernel it replaces
// (trnsparse/nki/kernels.py:86-155) uses a soft mask; this one applies the
// exact comparison, in float32 as the reference's tensor comparison does.
//
// The mask is applied inside the GEMM, between the TMA load and the MMA, so
// no masked copy of A is ever written: per 128x32 K-chunk, warp 0 loads the
// raw A tile (and, 2-D, the Q tile) with TMA; four transform warps apply the
// mask and split the result into tf32 hi/lo in place (the tiles keep their
// 128-byte-swizzled layout; the 1-D form un-swizzles offsets to find each
// element's row and column); warp 1 issues the 3xTF32 tcgen05.mma. A chunk
// with no surviving pair issues no MMA (the block skip). Work units are
// (128-row tile, N tile, contiguous range of 128-wide K blocks); units that
// split a row tile combine through float reductions into a zeroed C. When N
// spans exactly two 256-wide tiles, screened_tc2_kernel takes both N tiles in
// one unit so each masked A chunk is loaded and transformed once.
#include <cstdlib>

#include "tc_common.cuh"

namespace tsb {
namespace {

constexpr int kScThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue, warps 6-9 mask transform
constexpr int kScSmemMax = 232448;

template <int BN>
struct ScLayout {
  static constexpr int kATile = 128 * 128;  // 128 rows x 32 fp32: A (then its tf32 hi), or Q (then A's lo)
  static constexpr int kBTile = BN * 128;   // BN rows of B^T x 32 fp32, hi and lo
  static constexpr int kStage = 2 * (kATile + kBTile);
  static constexpr int kEpi = 4 * 2 * 4096;  // per epilogue warp: two 32 x 32 fp32 staging tiles
  static constexpr int kBarBytes = 1024;
  static constexpr int kAlign = 1024;        // slack to align the window to 1024 bytes
  static constexpr int kStages = (kScSmemMax - kAlign - kEpi - kBarBytes) / kStage;
  static constexpr int kEpiOff = kStages * kStage;
  static constexpr int kBarOff = kEpiOff + kEpi;
  static constexpr int kSmem = kBarOff + kBarBytes + kAlign;
  static_assert(kStages >= 2 && kStages <= 4, "operand ring");
};

struct ScBars {
  uint64_t full[4], xf[4], empty[4], acc_full[2], acc_empty[2];
  uint32_t tmem_slot;
  int abort_flag;
  int survive[4][4];
  int have[2];
};

// The CTA's share of the work: the linear range [lo, hi) of (output tile, K block) pairs,
// output tile = row_tile * nt + n_tile, K block fastest. Consecutive pairs of one output tile
// form a segment; a segment that does not cover its tile's whole K range adds into C.
struct ScSeg {
  int row_tile, n_tile, kb0, kb1;
  bool partial;
};
struct ScWalk {
  int64_t pos, hi;
  int nkb, nt;
  __device__ bool next(ScSeg& g) {
    if (pos >= hi) return false;
    const int64_t tile = pos / nkb;
    const int64_t end = min(hi, (tile + 1) * nkb);
    g.row_tile = static_cast<int>(tile / nt);
    g.n_tile = static_cast<int>(tile % nt);
    g.kb0 = static_cast<int>(pos - tile * nkb);
    g.kb1 = static_cast<int>(end - tile * nkb);
    g.partial = g.kb0 > 0 || g.kb1 < nkb;
    pos = end;
    return true;
  }
};
__device__ __forceinline__ ScWalk sc_walk(int64_t W, int nkb, int nt) {
  const int64_t G = gridDim.x;
  return ScWalk{W * blockIdx.x / G, W * (blockIdx.x + 1) / G, nkb, nt};
}

// One row of a 128 x 32 chunk, in place: A o mask split into tf32 hi (over A) and lo (over
// Q, which mode 2 reads its bounds from first). The row's 8 16-byte chunks are 128-byte
// swizzled; they are visited rotated so 8 neighbouring rows hit 8 different banks. Returns
// whether any pair of the row survives.
__device__ __forceinline__ int sc_mask_split_row(float4* arow, float4* lrow, int tr, int mode, float qi, int kx,
                                                 int64_t K, const float* __restrict__ q_vec, float t) {
  int keep = 0;
#pragma unroll
  for (int pp = 0; pp < 8; ++pp) {
    const int p = (pp + tr) & 7;
    const int L = p ^ (tr & 7);  // logical 16-byte chunk held by physical chunk p
    const float4 a = arow[p];
    float4 qv;
    if (mode == 2) {
      qv = lrow[p];
    } else {
      const int64_t c0 = kx + 4 * L;
      float qc[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) qc[u] = (c0 + u < K) ? __fsqrt_rn(fabsf(__ldg(q_vec + c0 + u))) : 0.f;
      qv = make_float4(__fmul_rn(qi, qc[0]), __fmul_rn(qi, qc[1]), __fmul_rn(qi, qc[2]), __fmul_rn(qi, qc[3]));
    }
    const float v[4] = {qv.x > t ? a.x : 0.f, qv.y > t ? a.y : 0.f, qv.z > t ? a.z : 0.f, qv.w > t ? a.w : 0.f};
    keep |= (qv.x > t) | (qv.y > t) | (qv.z > t) | (qv.w > t);
    float h[4], l[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      h[u] = tf32_rna(v[u]);
      l[u] = tf32_rna(v[u] - h[u]);
    }
    arow[p] = make_float4(h[0], h[1], h[2], h[3]);
    lrow[p] = make_float4(l[0], l[1], l[2], l[3]);
  }
  return keep;
}

// mode 1: q_vec (length K == M) holds diag integrals, mask = fl(Qi*Qj) > t
// mode 2: tq maps the 2-D bound matrix Q (M x K), mask = Q > t
// Persistent: gridDim.x CTAs split the (output tile, K block) space evenly (sc_walk).
template <int BN>
__global__ void __launch_bounds__(kScThreads, 1)
screened_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tq,
                   const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
                   const __grid_constant__ CUtensorMap tc, const float* __restrict__ q_vec, int mode, float t,
                   int64_t M, int64_t K, int64_t N, int nkb, int nt) {
  using Lay = ScLayout<BN>;
  constexpr int S = Lay::kStages;
  extern __shared__ __align__(16) uint8_t dsmem_sc[];
  const uint32_t raw = smem_u32(dsmem_sc);
  uint8_t* const sbase = dsmem_sc + (((raw + 1023u) & ~1023u) - raw);
  ScBars& Bs = *reinterpret_cast<ScBars*>(sbase + Lay::kBarOff);
  auto a_hi = [&](int s) { return sbase + s * Lay::kStage; };
  auto a_lo = [&](int s) { return sbase + s * Lay::kStage + Lay::kATile; };
  auto b_hi = [&](int s) { return sbase + s * Lay::kStage + 2 * Lay::kATile; };
  auto b_lo = [&](int s) { return sbase + s * Lay::kStage + 2 * Lay::kATile + Lay::kBTile; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t W = static_cast<int64_t>((M + 127) / 128) * nt * nkb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&Bs.full[s], 1);
      mbar_init(&Bs.xf[s], 1);
      mbar_init(&Bs.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&Bs.acc_full[i], 1);
      mbar_init(&Bs.acc_empty[i], 128);
    }
    Bs.abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&ta);
    tma_prefetch_desc(&tb_hi);
    tma_prefetch_desc(&tb_lo);
    tma_prefetch_desc(&tc);
    if (mode == 2) tma_prefetch_desc(&tq);
  }
  if (warp == 1) {
    tmem_alloc(&Bs.tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_wait();  // the set-up above overlapped the previous kernel (the operand split)
  const uint32_t tmem = Bs.tmem_slot;
  volatile int* abort_flag = &Bs.abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      ScWalk wk = sc_walk(W, nkb, nt);
      ScSeg g;
      int it = 0;
      bool ok = true;
      // A and Q stream through once per N tile; B^T (hi, lo) is re-read by every row tile
      const uint64_t stream_pol = l2_policy_evict_first(), keep_pol = l2_policy_evict_last();
      while (ok && wk.next(g)) {
        const int n0 = g.n_tile * BN;
        for (int kc = g.kb0 * 4; ok && kc < g.kb1 * 4; ++kc, ++it) {
          const int s = it % S, use = it / S;
          if (use > 0 && !mbar_wait(&Bs.empty[s], (use - 1) & 1)) { ok = false; break; }
          if (*abort_flag) { ok = false; break; }
          const int kx = kc * 32;  // K coordinate of the 32-wide chunk
          mbar_arrive_expect_tx(&Bs.full[s], mode == 2 ? Lay::kStage : Lay::kStage - Lay::kATile);
          tma_load_2d_hint(a_hi(s), &ta, kx, g.row_tile * 128, &Bs.full[s], stream_pol);
          if (mode == 2) tma_load_2d_hint(a_lo(s), &tq, kx, g.row_tile * 128, &Bs.full[s], stream_pol);
          tma_load_2d_hint(b_hi(s), &tb_hi, kx, n0, &Bs.full[s], keep_pol);
          tma_load_2d_hint(b_lo(s), &tb_lo, kx, n0, &Bs.full[s], keep_pol);
        }
      }
      if (!ok) {
        atomicExch(&Bs.abort_flag, 1);
        // never leave the CTA with copies in flight: wait for the fills nobody consumed
        for (int i = (it > S ? it - S : 0); i < it; ++i) mbar_wait(&Bs.full[i % S], (i / S) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(MmaKind::TF32, 128, BN);
      ScWalk wk = sc_walk(W, nkb, nt);
      ScSeg g;
      int it = 0, q = 0;
      bool ok = !*abort_flag;
      while (ok && wk.next(g)) {
        const int acc = q & 1;
        if (q >= 2 && !mbar_wait(&Bs.acc_empty[acc], ((q >> 1) - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        bool started = false;
        for (int kc = g.kb0 * 4; kc < g.kb1 * 4; ++kc, ++it) {
          const int s = it % S, use = it / S;
          if (*abort_flag || !mbar_wait(&Bs.xf[s], use & 1)) { ok = false; break; }
          tc_fence_after();
          if (Bs.survive[s][0] | Bs.survive[s][1] | Bs.survive[s][2] | Bs.survive[s][3]) {
            const uint32_t ah = smem_u32(a_hi(s)), al = smem_u32(a_lo(s));
            const uint32_t bh = smem_u32(b_hi(s)), bl = smem_u32(b_lo(s));
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              const uint32_t off = ks * 32;
              umma<MmaKind::TF32>(d, smem_desc_sw128(ah + off), smem_desc_sw128(bh + off), idesc, started);
              started = true;
              umma<MmaKind::TF32>(d, smem_desc_sw128(ah + off), smem_desc_sw128(bl + off), idesc, true);
              umma<MmaKind::TF32>(d, smem_desc_sw128(al + off), smem_desc_sw128(bh + off), idesc, true);
            }
          }
          umma_commit(&Bs.empty[s]);
        }
        if (!ok) break;
        Bs.have[acc] = started ? 1 : 0;
        __threadfence_block();
        umma_commit(&Bs.acc_full[acc]);
        ++q;
      }
      if (!ok) atomicExch(&Bs.abort_flag, 1);
    }
  } else if (warp >= 6) {
    // ---------------- mask + tf32 split of the A tile, in place (a thread per tile row)
    const int tr = threadIdx.x - 192;
    const int w4 = warp - 6;
    ScWalk wk = sc_walk(W, nkb, nt);
    ScSeg g;
    int it = 0;
    bool ok = !*abort_flag;
    while (ok && wk.next(g)) {
      float qi = 0.f;
      if (mode == 1) {
        const int64_t r = static_cast<int64_t>(g.row_tile) * 128 + tr;
        qi = r < M ? __fsqrt_rn(fabsf(q_vec[r])) : 0.f;
      }
      for (int kc = g.kb0 * 4; kc < g.kb1 * 4; ++kc, ++it) {
        const int s = it % S, use = it / S;
        if (*abort_flag || !mbar_wait(&Bs.full[s], use & 1)) { ok = false; break; }
        const int keep = sc_mask_split_row(reinterpret_cast<float4*>(a_hi(s) + tr * 128),
                                           reinterpret_cast<float4*>(a_lo(s) + tr * 128), tr, mode, qi, kc * 32, K,
                                           q_vec, t);
        const int wkeep = __any_sync(0xffffffffu, keep);
        if (lane == 0) Bs.survive[s][w4] = wkeep;
        fence_proxy_async_smem();  // generic-proxy writes -> tcgen05 (async proxy) reads
        asm volatile("bar.sync 1, 128;\n" ::: "memory");
        if (tr == 0) mbar_arrive(&Bs.xf[s]);
      }
    }
    if (!ok) atomicExch(&Bs.abort_flag, 1);
  } else {
    // ---------------- epilogue warps 2-5: TMEM lane quadrant = warp % 4; 32 x 32 fp32 pieces
    // staged (128-byte swizzle) and written by TMA: a store for a segment that covers its
    // tile's whole K range, a reduce-add into the cleared C otherwise.
    const int quad = warp & 3;
    uint8_t* const stage0 = sbase + Lay::kEpiOff + (warp - 2) * 8192;
    ScWalk wk = sc_walk(W, nkb, nt);
    ScSeg g;
    int q = 0, pc = 0;
    bool ok = !*abort_flag;
    while (wk.next(g)) {
      const int acc = q & 1;
      ok = ok && mbar_wait(&Bs.acc_full[acc], (q >> 1) & 1) && !*abort_flag;
      tc_fence_after();
      const bool have = __all_sync(0xffffffffu, ok) && *reinterpret_cast<volatile int*>(&Bs.have[acc]) != 0;
      const int n0 = g.n_tile * BN;
      const int64_t row0 = static_cast<int64_t>(g.row_tile) * 128 + quad * 32;
      const uint32_t t_row = tmem + acc * BN + (static_cast<uint32_t>(quad * 32) << 16);
      if (ok && (have || !g.partial)) {  // a screened-out partial segment adds nothing
#pragma unroll 1
        for (int p = 0; p < BN / 32 && n0 + p * 32 < N; ++p, ++pc) {
          uint8_t* stage = stage0 + (pc & 1) * 4096;
          if (pc >= 2) {
            if (lane == 0) bulk_wait_read_1();  // the store issued two pieces ago has read its tile
            __syncwarp();
          }
          uint32_t w[32];
          if (have) {
            tmem_ld32(t_row + p * 32, w);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i] = 0u;
          }
#pragma unroll
          for (int x = 0; x < 8; ++x)
            *reinterpret_cast<uint4*>(stage + lane * 128 + ((x ^ (lane & 7)) * 16)) =
                make_uint4(w[4 * x], w[4 * x + 1], w[4 * x + 2], w[4 * x + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && row0 < M) {
            if (g.partial)
              tma_reduce_add_2d(&tc, stage, n0 + p * 32, static_cast<int>(row0));
            else
              tma_store_2d(&tc, stage, n0 + p * 32, static_cast<int>(row0));
            bulk_commit_group();
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&Bs.acc_empty[acc]);
      ++q;
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

// Two 256-wide N tiles at once (N in (256, 512]): a work unit is (row tile, K block range)
// and both N tiles accumulate in the two TMEM accumulators, so every masked / split A chunk
// feeds both tiles' MMAs: A and Q are read and transformed once instead of once per N tile.
// Shared memory holds an A ring (A hi + lo) and a B^T ring (hi + lo, one N tile per slot)
// consumed twice as fast; the epilogue drains both accumulators at the end of a unit (not
// overlapped with the next unit's MMAs: each CTA has one or two units).
struct Sc2Layout {
  static constexpr int kATile = 128 * 128;                    // 128 rows x 32 fp32
  static constexpr int kASlot = 2 * kATile;                   // A (then hi) + Q (then lo)
  static constexpr int kBTile = 256 * 128;                    // 256 rows of B^T x 32 fp32
  static constexpr int kBSlot = 2 * kBTile;                   // hi + lo
  static constexpr int kASlots = 2, kBSlots = 2;
  static constexpr int kA = 0, kB = kASlots * kASlot;
  static constexpr int kEpiOff = kB + kBSlots * kBSlot;
  static constexpr int kEpi = 4 * 2 * 4096;
  static constexpr int kBarOff = kEpiOff + kEpi;
  static constexpr int kBarBytes = 1024;
  static constexpr int kSmem = kBarOff + kBarBytes + 1024;  // + alignment slack
  static_assert(kSmem <= kScSmemMax, "shared memory");
};

struct Sc2Bars {
  uint64_t a_full[2], a_xf[2], a_empty[2], b_full[2], b_empty[2], acc_full, acc_empty;
  uint32_t tmem_slot;
  int abort_flag;
  int survive[2][4];
  int have;
};

__global__ void __launch_bounds__(kScThreads, 1)
screened_tc2_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tq,
                    const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
                    const __grid_constant__ CUtensorMap tc, const float* __restrict__ q_vec, int mode, float t,
                    int64_t M, int64_t K, int64_t N, int nkb) {
  using Lay = Sc2Layout;
  extern __shared__ __align__(16) uint8_t dsmem_sc2[];
  const uint32_t raw = smem_u32(dsmem_sc2);
  uint8_t* const sbase = dsmem_sc2 + (((raw + 1023u) & ~1023u) - raw);
  Sc2Bars& Bs = *reinterpret_cast<Sc2Bars*>(sbase + Lay::kBarOff);
  auto a_hi = [&](int s) { return sbase + Lay::kA + s * Lay::kASlot; };
  auto a_lo = [&](int s) { return sbase + Lay::kA + s * Lay::kASlot + Lay::kATile; };
  auto b_hi = [&](int s) { return sbase + Lay::kB + s * Lay::kBSlot; };
  auto b_lo = [&](int s) { return sbase + Lay::kB + s * Lay::kBSlot + Lay::kBTile; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t W = static_cast<int64_t>((M + 127) / 128) * nkb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&Bs.a_full[s], 1);
      mbar_init(&Bs.a_xf[s], 1);
      mbar_init(&Bs.a_empty[s], 1);
      mbar_init(&Bs.b_full[s], 1);
      mbar_init(&Bs.b_empty[s], 1);
    }
    mbar_init(&Bs.acc_full, 1);
    mbar_init(&Bs.acc_empty, 128);
    Bs.abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&ta);
    tma_prefetch_desc(&tb_hi);
    tma_prefetch_desc(&tb_lo);
    tma_prefetch_desc(&tc);
    if (mode == 2) tma_prefetch_desc(&tq);
  }
  if (warp == 1) {
    tmem_alloc(&Bs.tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dep_wait();  // the set-up above overlapped the previous kernel (the operand split)
  const uint32_t tmem = Bs.tmem_slot;
  volatile int* abort_flag = &Bs.abort_flag;

  if (warp == 0) {
    // ---------------- TMA producer: per K chunk A (+ Q) into the A ring, then B^T of N tile 0
    // and of N tile 1 into the B ring
    if (lane == 0) {
      ScWalk wk = sc_walk(W, nkb, 1);
      ScSeg g;
      int ia = 0, ib = 0;
      bool ok = true;
      const uint64_t stream_pol = l2_policy_evict_first(), keep_pol = l2_policy_evict_last();
      while (ok && wk.next(g)) {
        for (int kc = g.kb0 * 4; ok && kc < g.kb1 * 4; ++kc) {
          const int sa = ia & 1, ua = ia >> 1;
          const int kx = kc * 32;
          if (*abort_flag || (ua > 0 && !mbar_wait(&Bs.a_empty[sa], (ua - 1) & 1))) { ok = false; break; }
          mbar_arrive_expect_tx(&Bs.a_full[sa], mode == 2 ? Lay::kASlot : Lay::kATile);
          tma_load_2d_hint(a_hi(sa), &ta, kx, g.row_tile * 128, &Bs.a_full[sa], stream_pol);
          if (mode == 2) tma_load_2d_hint(a_lo(sa), &tq, kx, g.row_tile * 128, &Bs.a_full[sa], stream_pol);
          ++ia;  // counted once issued (the clean-up below waits for every issued fill)
          for (int h = 0; h < 2; ++h, ++ib) {
            const int sb = ib & 1, ub = ib >> 1;
            if (*abort_flag || (ub > 0 && !mbar_wait(&Bs.b_empty[sb], (ub - 1) & 1))) { ok = false; break; }
            mbar_arrive_expect_tx(&Bs.b_full[sb], Lay::kBSlot);
            tma_load_2d_hint(b_hi(sb), &tb_hi, kx, h * 256, &Bs.b_full[sb], keep_pol);
            tma_load_2d_hint(b_lo(sb), &tb_lo, kx, h * 256, &Bs.b_full[sb], keep_pol);
          }
        }
      }
      if (!ok) {
        atomicExch(&Bs.abort_flag, 1);
        // never leave the CTA with copies in flight: wait for the fills nobody consumed
        for (int i = (ia > 2 ? ia - 2 : 0); i < ia; ++i) mbar_wait(&Bs.a_full[i & 1], (i >> 1) & 1);
        for (int i = (ib > 2 ? ib - 2 : 0); i < ib; ++i) mbar_wait(&Bs.b_full[i & 1], (i >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: accumulator h at TMEM columns 256 h
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(MmaKind::TF32, 128, 256);
      ScWalk wk = sc_walk(W, nkb, 1);
      ScSeg g;
      int ia = 0, ib = 0, q = 0;
      bool ok = !*abort_flag;
      while (ok && wk.next(g)) {
        if (q >= 1 && !mbar_wait(&Bs.acc_empty, (q - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        bool started = false;
        for (int kc = g.kb0 * 4; ok && kc < g.kb1 * 4; ++kc, ++ia) {
          const int sa = ia & 1, ua = ia >> 1;
          if (*abort_flag || !mbar_wait(&Bs.a_xf[sa], ua & 1)) { ok = false; break; }
          tc_fence_after();
          const bool live = (Bs.survive[sa][0] | Bs.survive[sa][1] | Bs.survive[sa][2] | Bs.survive[sa][3]) != 0;
          const uint32_t ah = smem_u32(a_hi(sa)), al = smem_u32(a_lo(sa));
          for (int h = 0; h < 2; ++h, ++ib) {
            const int sb = ib & 1, ub = ib >> 1;
            if (*abort_flag || !mbar_wait(&Bs.b_full[sb], ub & 1)) { ok = false; break; }
            tc_fence_after();
            if (live) {
              const uint32_t bh = smem_u32(b_hi(sb)), bl = smem_u32(b_lo(sb));
              const uint32_t d = tmem + h * 256;
#pragma unroll
              for (int ks = 0; ks < 4; ++ks) {
                const uint32_t off = ks * 32;
                umma<MmaKind::TF32>(d, smem_desc_sw128(ah + off), smem_desc_sw128(bh + off), idesc,
                                    started || ks > 0);
                umma<MmaKind::TF32>(d, smem_desc_sw128(ah + off), smem_desc_sw128(bl + off), idesc, true);
                umma<MmaKind::TF32>(d, smem_desc_sw128(al + off), smem_desc_sw128(bh + off), idesc, true);
              }
            }
            umma_commit(&Bs.b_empty[sb]);
          }
          if (!ok) break;
          if (live) started = true;
          umma_commit(&Bs.a_empty[sa]);
        }
        if (!ok) break;
        Bs.have = started ? 1 : 0;
        __threadfence_block();
        umma_commit(&Bs.acc_full);
        ++q;
      }
      if (!ok) atomicExch(&Bs.abort_flag, 1);
    }
  } else if (warp >= 6) {
    // ---------------- mask + tf32 split of the A tile, in place (a thread per tile row),
    // once per K chunk for both N tiles
    const int tr = threadIdx.x - 192;
    const int w4 = warp - 6;
    ScWalk wk = sc_walk(W, nkb, 1);
    ScSeg g;
    int ia = 0;
    bool ok = !*abort_flag;
    while (ok && wk.next(g)) {
      float qi = 0.f;
      if (mode == 1) {
        const int64_t r = static_cast<int64_t>(g.row_tile) * 128 + tr;
        qi = r < M ? __fsqrt_rn(fabsf(q_vec[r])) : 0.f;
      }
      for (int kc = g.kb0 * 4; kc < g.kb1 * 4; ++kc, ++ia) {
        const int sa = ia & 1, ua = ia >> 1;
        if (*abort_flag || !mbar_wait(&Bs.a_full[sa], ua & 1)) { ok = false; break; }
        const int keep = sc_mask_split_row(reinterpret_cast<float4*>(a_hi(sa) + tr * 128),
                                           reinterpret_cast<float4*>(a_lo(sa) + tr * 128), tr, mode, qi, kc * 32, K,
                                           q_vec, t);
        const int wkeep = __any_sync(0xffffffffu, keep);
        if (lane == 0) Bs.survive[sa][w4] = wkeep;
        fence_proxy_async_smem();  // generic-proxy writes -> tcgen05 (async proxy) reads
        asm volatile("bar.sync 1, 128;\n" ::: "memory");
        if (tr == 0) mbar_arrive(&Bs.a_xf[sa]);
      }
    }
    if (!ok) atomicExch(&Bs.abort_flag, 1);
  } else {
    // ---------------- epilogue warps 2-5: both accumulators of a unit, 32 x 32 fp32 pieces
    // staged (128-byte swizzle) and written by TMA (reduce-add into the cleared C for a unit
    // that covers only part of its row tile's K range)
    const int quad = warp & 3;
    uint8_t* const stage0 = sbase + Lay::kEpiOff + (warp - 2) * 8192;
    ScWalk wk = sc_walk(W, nkb, 1);
    ScSeg g;
    int q = 0, pc = 0;
    bool ok = !*abort_flag;
    while (wk.next(g)) {
      ok = ok && mbar_wait(&Bs.acc_full, q & 1) && !*abort_flag;
      tc_fence_after();
      const bool have = __all_sync(0xffffffffu, ok) && *reinterpret_cast<volatile int*>(&Bs.have) != 0;
      const int64_t row0 = static_cast<int64_t>(g.row_tile) * 128 + quad * 32;
      if (ok && (have || !g.partial)) {  // a screened-out partial unit adds nothing
#pragma unroll 1
        for (int p = 0; p < 16 && p * 32 < N; ++p, ++pc) {
          const uint32_t t_row = tmem + (p >> 3) * 256 + (p & 7) * 32 + (static_cast<uint32_t>(quad * 32) << 16);
          uint8_t* stage = stage0 + (pc & 1) * 4096;
          if (pc >= 2) {
            if (lane == 0) bulk_wait_read_1();  // the store issued two pieces ago has read its tile
            __syncwarp();
          }
          uint32_t w[32];
          if (have) {
            tmem_ld32(t_row, w);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i] = 0u;
          }
#pragma unroll
          for (int x = 0; x < 8; ++x)
            *reinterpret_cast<uint4*>(stage + lane * 128 + ((x ^ (lane & 7)) * 16)) =
                make_uint4(w[4 * x], w[4 * x + 1], w[4 * x + 2], w[4 * x + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && row0 < M) {
            if (g.partial)
              tma_reduce_add_2d(&tc, stage, p * 32, static_cast<int>(row0));
            else
              tma_store_2d(&tc, stage, p * 32, static_cast<int>(row0));
            bulk_commit_group();
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&Bs.acc_empty);
      ++q;
    }
    if (lane == 0) bulk_wait_all();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int BN>
int launch_sc(const CUtensorMap& ta, const CUtensorMap& tq, const CUtensorMap& bhi, const CUtensorMap& blo,
              const CUtensorMap& cm, const float* q_vec, int mode, float t, int64_t M, int64_t K, int64_t N,
              int nkb, int nt, int grid, cudaStream_t st) {
  using Lay = ScLayout<BN>;
  auto kern = screened_tc_kernel<BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kSmem);
  if (e != cudaSuccess) return cuda_status(e, "screened_tc: set smem");
  e = launch_pdl(kern, dim3(grid), dim3(kScThreads), Lay::kSmem, st, ta, tq, bhi, blo, cm, q_vec, mode, t, M, K, N, nkb,
                 nt);
  if (e != cudaSuccess) return cuda_status(e, "screened_tc launch");
  return debug_sync(st, "screened_tc: main kernel (sync)");
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" size_t trnsparse_screened_spmm_workspace_size(int64_t K, int64_t N) {
  const int64_t k_pad = (K + 127) / 128 * 128;
  return 2 * align256(sizeof(float) * (size_t)k_pad * (size_t)(N < 0 ? 0 : N));
}

extern "C" int trnsparse_screened_spmm(int64_t M, int64_t K, int64_t N, const float* A, int64_t lda,
                                       const float* bounds, int bounds_kind, int64_t ldq, double threshold,
                                       const float* B, int64_t ldb, float* C, int64_t ldc, void* ws,
                                       size_t ws_bytes, void* stream) {
  TSB_REQUIRE(M >= 0 && K >= 0 && N >= 0, "screened_spmm: negative size");
  TSB_REQUIRE(bounds_kind == 1 || bounds_kind == 2, "screened_spmm: bounds_kind must be 1 (vector) or 2 (matrix)");
  TSB_REQUIRE(bounds_kind != 1 || M == K, "screened_spmm: the 1-D bound vector needs square A (M=%lld K=%lld)",
              (long long)M, (long long)K);
  TSB_REQUIRE(lda >= K && ldb >= N && ldc >= N && (bounds_kind == 1 || ldq >= K), "screened_spmm: bad leading dim");
  if (M == 0 || N == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(C && (K == 0 || (A && bounds && B)), "screened_spmm: null pointer");
  const size_t need = trnsparse_screened_spmm_workspace_size(K, N);
  TSB_REQUIRE(ws && ws_bytes >= need, "screened_spmm: workspace too small (%zu < %zu)", ws_bytes, need);
  if (lda % 4 || (bounds_kind == 2 && ldq % 4))
    return fail(TRNSPARSE_ERR_ALIGN, "screened_spmm: row strides of A and Q must be multiples of 4 floats");
  TSB_REQUIRE(ldc % 4 == 0 && (reinterpret_cast<uintptr_t>(C) & 15u) == 0,
              "screened_spmm: C must be 16-byte aligned with ldc a multiple of 4");
  cudaStream_t st = as_stream(stream);
  const int64_t nkb = (K + 127) / 128;
  const int64_t mt = (M + 127) / 128;
  const int bn = N > 128 ? 256 : 128;
  const int64_t nt = (N + bn - 1) / bn;
  TSB_REQUIRE(mt * nt * nkb < (1ll << 40) && nkb < (1 << 24), "screened_spmm: sizes out of range");
  // both 256-wide N tiles in one unit when N is in (256, 512] (TRNSPARSE_SCREENED_DUAL=0: off)
  static const bool dual_ok = [] {
    const char* v = getenv("TRNSPARSE_SCREENED_DUAL");
    return v == nullptr || v[0] != '0';
  }();
  const bool dual = dual_ok && bn == 256 && nt == 2;
  // persistent grid: the (output tile, K block) pairs split evenly over at most one CTA per SM
  const int64_t W = mt * (dual ? 1 : nt) * nkb;
  const int grid = static_cast<int>(W < sm_count() ? W : sm_count());
  bool partial = false;  // does any CTA's range start or end inside an output tile?
  for (int64_t c = 0; c <= grid && !partial && K > 0; ++c) partial = (W * c / grid) % nkb != 0;
  if (partial || K == 0) {
    cudaError_t e = cudaMemset2DAsync(C, sizeof(float) * (size_t)ldc, 0, sizeof(float) * (size_t)N, (size_t)M, st);
    if (e != cudaSuccess) return cuda_status(e, "screened_spmm: zero C");
  }
  if (K == 0) return TRNSPARSE_OK;
  // B (K x N) -> B^T (N x k_pad) split into tf32 hi / lo
  const int64_t k_pad = nkb * 128;
  float* bt_hi = static_cast<float*>(ws);
  float* bt_lo = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + align256(sizeof(float) * (size_t)k_pad * (size_t)N));
  dim3 tg((unsigned)(k_pad / 32), (unsigned)((N + 31) / 32));
  TSB_REQUIRE(tg.y < 65536, "screened_spmm: N too large");
  transpose_b_kernel<true, float><<<tg, dim3(32, 8), 0, st>>>(K, N, B, ldb, k_pad, bt_hi, bt_lo);
  TSB_CHECK_LAUNCH("screened_spmm: transpose B");
  CUtensorMap ta, tq, bh, bl;
  const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  int rc = make_tmap_2d(&ta, A, dt, (uint64_t)K, (uint64_t)M, (uint64_t)lda * 4, 32, 128);
  if (rc) return rc;
  if (bounds_kind == 2) {
    rc = make_tmap_2d(&tq, bounds, dt, (uint64_t)K, (uint64_t)M, (uint64_t)ldq * 4, 32, 128);
    if (rc) return rc;
  } else {
    tq = ta;
  }
  rc = make_tmap_2d(&bh, bt_hi, dt, (uint64_t)k_pad, (uint64_t)N, (uint64_t)k_pad * 4, 32, (uint32_t)bn);
  if (rc) return rc;
  rc = make_tmap_2d(&bl, bt_lo, dt, (uint64_t)k_pad, (uint64_t)N, (uint64_t)k_pad * 4, 32, (uint32_t)bn);
  if (rc) return rc;
  CUtensorMap cm;
  rc = make_tmap_2d(&cm, C, dt, (uint64_t)N, (uint64_t)M, (uint64_t)ldc * 4, 32, 32);
  if (rc) return rc;
  const float t = static_cast<float>(sqrt(threshold));
  const float* qv = bounds_kind == 1 ? bounds : nullptr;
  if (dual) {
    auto kern = screened_tc2_kernel;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Sc2Layout::kSmem);
    if (e != cudaSuccess) return cuda_status(e, "screened_tc2: set smem");
    e = launch_pdl(kern, dim3(grid), dim3(kScThreads), Sc2Layout::kSmem, st, ta, tq, bh, bl, cm, qv, bounds_kind, t, M,
                   K, N, (int)nkb);
    if (e != cudaSuccess) return cuda_status(e, "screened_tc2 launch");
    return debug_sync(st, "screened_tc2: main kernel (sync)");
  }
  return bn == 128 ? launch_sc<128>(ta, tq, bh, bl, cm, qv, bounds_kind, t, M, K, N, (int)nkb, (int)nt, grid, st)
                   : launch_sc<256>(ta, tq, bh, bl, cm, qv, bounds_kind, t, M, K, N, (int)nkb, (int)nt, grid, st);
}
