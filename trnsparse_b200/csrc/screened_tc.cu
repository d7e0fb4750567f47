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
// (128-row tile, contiguous range of 128-wide K blocks); units that split a
// row tile combine through float reductions into a zeroed C.
#include "tc_common.cuh"

namespace tsb {
namespace {

constexpr int kScThreads = 256;  // warps 0-3: TMA / MMA / TMEM drain; warps 4-7: mask transform

template <int BN>
struct ScLayout {
  static constexpr int kATile = 128 * 128;
  static constexpr int kBTile = BN * 128;
  static constexpr int kStage = 2 * (kATile + kBTile);
  static constexpr int kStages = 200 * 1024 / kStage;
  static constexpr int kSmem = kStages * kStage + 1024;
  static_assert(kStages * kStage >= 128 * (BN + 4) * 4, "epilogue tile must fit in the operand ring");
};

// mode 1: q_vec (length K == M) holds diag integrals, mask = fl(Qi*Qj) > t
// mode 2: tq maps the 2-D bound matrix Q (M x K), mask = Q > t
template <int BN>
__global__ void __launch_bounds__(kScThreads, 1)
screened_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tq,
                   const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
                   const float* __restrict__ q_vec, int mode, float t, int64_t M, int64_t K, int64_t N, int nkb,
                   int nsplit, float* __restrict__ C, int64_t ldc) {
  using Lay = ScLayout<BN>;
  constexpr int S = Lay::kStages;
  extern __shared__ __align__(16) uint8_t dsmem_sc[];
  __shared__ __align__(8) uint64_t full_bar[S];
  __shared__ __align__(8) uint64_t xf_bar[S];
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ __align__(8) uint64_t done_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ int survive[S][4];
  __shared__ int any_mma;
  __shared__ float qrow[128];

  const uint32_t raw = smem_u32(dsmem_sc);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const sbase = dsmem_sc + (base - raw);
  auto a_hi = [&](int s) { return sbase + s * Lay::kStage; };
  auto a_lo = [&](int s) { return sbase + s * Lay::kStage + Lay::kATile; };
  auto b_hi = [&](int s) { return sbase + s * Lay::kStage + 2 * Lay::kATile; };
  auto b_lo = [&](int s) { return sbase + s * Lay::kStage + 2 * Lay::kATile + Lay::kBTile; };

  const int warp = threadIdx.x >> 5;
  const int row_tile = blockIdx.x / nsplit;
  const int part = blockIdx.x - row_tile * nsplit;
  const int kb0 = static_cast<int>((static_cast<int64_t>(nkb) * part) / nsplit);
  const int kb1 = static_cast<int>((static_cast<int64_t>(nkb) * (part + 1)) / nsplit);
  const int total = (kb1 - kb0) * 4;  // 32-wide fp32 chunks
  const int n0 = blockIdx.y * BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&xf_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&done_bar, 1);
    abort_flag = (base & 1023u) ? 1 : 0;
    if (abort_flag) record_device_error(DEVERR_SELFCHECK_SMEM);
    any_mma = 0;
    fence_mbar_init();
    tma_prefetch_desc(&ta);
    tma_prefetch_desc(&tb_hi);
    tma_prefetch_desc(&tb_lo);
    if (mode == 2) tma_prefetch_desc(&tq);
  }
  if (mode == 1 && threadIdx.x >= 128) {
    const int64_t r = static_cast<int64_t>(row_tile) * 128 + (threadIdx.x - 128);
    qrow[threadIdx.x - 128] = r < M ? __fsqrt_rn(fabsf(q_vec[r])) : 0.f;
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

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
      const int kx = (kb0 + it / 4) * 128 + (it % 4) * 32;  // K coordinate of the chunk
      mbar_arrive_expect_tx(&full_bar[s], mode == 2 ? Lay::kStage : Lay::kStage - Lay::kATile);
      tma_load_2d(a_hi(s), &ta, kx, row_tile * 128, &full_bar[s]);
      if (mode == 2) tma_load_2d(a_lo(s), &tq, kx, row_tile * 128, &full_bar[s]);
      tma_load_2d(b_hi(s), &tb_hi, kx, n0, &full_bar[s]);
      tma_load_2d(b_lo(s), &tb_lo, kx, n0, &full_bar[s]);
      issued = it + 1;
    }
    if (*(volatile int*)&abort_flag) {
      for (int it = (issued > S ? issued - S : 0); it < issued; ++it) mbar_wait(&full_bar[it % S], (it / S) & 1);
    }
  } else if (warp == 1 && elect_lane0()) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc = make_idesc(MmaKind::TF32, 128, BN);
    bool acc = false;
    for (int it = 0; it < total; ++it) {
      if (*(volatile int*)&abort_flag) break;
      const int s = it % S, use = it / S;
      if (!mbar_wait(&xf_bar[s], use & 1)) {
        atomicExch(&abort_flag, 1);
        break;
      }
      tc_fence_after();
      if (survive[s][0] | survive[s][1] | survive[s][2] | survive[s][3]) {
        const uint32_t ah = smem_u32(a_hi(s)), al = smem_u32(a_lo(s));
        const uint32_t bh = smem_u32(b_hi(s)), bl = smem_u32(b_lo(s));
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t off = ks * 32;
          umma<MmaKind::TF32>(tmem, smem_desc_sw128(ah + off), smem_desc_sw128(bh + off), idesc, acc);
          acc = true;
          umma<MmaKind::TF32>(tmem, smem_desc_sw128(ah + off), smem_desc_sw128(bl + off), idesc, true);
          umma<MmaKind::TF32>(tmem, smem_desc_sw128(al + off), smem_desc_sw128(bh + off), idesc, true);
        }
      }
      umma_commit(&empty_bar[s]);
    }
    any_mma = acc ? 1 : 0;
    umma_commit(&done_bar);
  } else if (warp >= 4) {
    // ---------------- mask + tf32 split, in place
    const int tr = threadIdx.x - 128;  // tile row owned by this thread
    const int w4 = warp - 4;
    const float qi = mode == 1 ? qrow[tr] : 0.f;
    for (int it = 0; it < total; ++it) {
      if (*(volatile int*)&abort_flag) break;
      const int s = it % S, use = it / S;
      if (!mbar_wait(&full_bar[s], use & 1)) {
        atomicExch(&abort_flag, 1);
        break;
      }
      const int kx = (kb0 + it / 4) * 128 + (it % 4) * 32;
      float4* arow = reinterpret_cast<float4*>(a_hi(s) + tr * 128);
      float4* lrow = reinterpret_cast<float4*>(a_lo(s) + tr * 128);
      int keep = 0;
#pragma unroll
      for (int pp = 0; pp < 8; ++pp) {
        const int p = (pp + tr) & 7;   // rotate so 8 neighbouring rows hit 8 different banks
        const int L = p ^ (tr & 7);    // logical 16-byte chunk held by physical chunk p
        float4 a = arow[p];
        float4 q;
        if (mode == 2) {
          q = lrow[p];
        } else {
          const int64_t c0 = kx + 4 * L;
          float qc[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) qc[u] = (c0 + u < K) ? __fsqrt_rn(fabsf(__ldg(q_vec + c0 + u))) : 0.f;
          q = make_float4(__fmul_rn(qi, qc[0]), __fmul_rn(qi, qc[1]), __fmul_rn(qi, qc[2]), __fmul_rn(qi, qc[3]));
        }
        float v[4] = {q.x > t ? a.x : 0.f, q.y > t ? a.y : 0.f, q.z > t ? a.z : 0.f, q.w > t ? a.w : 0.f};
        keep |= (q.x > t) | (q.y > t) | (q.z > t) | (q.w > t);
        float h[4], l[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          h[u] = tf32_rna(v[u]);
          l[u] = tf32_rna(v[u] - h[u]);
        }
        arow[p] = make_float4(h[0], h[1], h[2], h[3]);
        lrow[p] = make_float4(l[0], l[1], l[2], l[3]);
      }
      const int wkeep = __any_sync(0xffffffffu, keep);
      if ((threadIdx.x & 31) == 0) survive[s][w4] = wkeep;
      fence_proxy_async_smem();  // generic-proxy writes -> tcgen05 (async proxy) reads
      asm volatile("bar.sync 1, 128;\n" ::: "memory");
      if (threadIdx.x == 128) mbar_arrive(&xf_bar[s]);
    }
  }
  __syncwarp();

  // ---------------- epilogue
  const bool ok = mbar_wait(&done_bar, 0);
  tc_fence_after();
  __syncthreads();
  const bool single = nsplit == 1;  // this CTA owns the whole row tile: plain stores
  const bool have = any_mma != 0;   // false: every chunk was screened out, the tile is zero
  const bool run = ok && !*(volatile int*)&abort_flag && (have || single);
  constexpr int LDS = BN + 4;
  float* stile = reinterpret_cast<float*>(sbase);
  if (run && have && warp < 4) {
    const int r_local = warp * 32 + (threadIdx.x & 31);
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
    const int64_t row0 = static_cast<int64_t>(row_tile) * 128;
    const bool vec = (ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(C) & 15u) == 0) && (n0 + BN <= N);
    if (vec) {
      constexpr int F4 = BN / 4;
      for (int f = threadIdx.x; f < 128 * F4; f += kScThreads) {
        const int rl = f / F4, c4 = f - rl * F4;
        const int64_t row = row0 + rl;
        if (row < M) {
          const float4 v = have ? *reinterpret_cast<const float4*>(stile + rl * LDS + 4 * c4) : make_float4(0.f, 0.f, 0.f, 0.f);
          float* dst = C + row * ldc + n0 + 4 * c4;
          if (single) *reinterpret_cast<float4*>(dst) = v;
          else red_add_v4(dst, __float_as_uint(v.x), __float_as_uint(v.y), __float_as_uint(v.z), __float_as_uint(v.w));
        }
      }
    } else {
      for (int f = threadIdx.x; f < 128 * BN; f += kScThreads) {
        const int rl = f / BN, c = f - rl * BN;
        const int64_t row = row0 + rl, col = n0 + c;
        if (row < M && col < N) {
          if (single) C[row * ldc + col] = have ? stile[rl * LDS + c] : 0.f;
          else red_add(C + row * ldc + col, __float_as_uint(stile[rl * LDS + c]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

template <int BN>
int launch_sc(const CUtensorMap& ta, const CUtensorMap& tq, const CUtensorMap& bhi, const CUtensorMap& blo,
              const float* q_vec, int mode, float t, int64_t M, int64_t K, int64_t N, int nkb, int nsplit, float* C,
              int64_t ldc, cudaStream_t st) {
  using Lay = ScLayout<BN>;
  auto kern = screened_tc_kernel<BN>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kSmem);
  if (e != cudaSuccess) return cuda_status(e, "screened_tc: set smem");
  const int64_t mt = (M + 127) / 128;
  dim3 grid((unsigned)(mt * nsplit), (unsigned)((N + BN - 1) / BN));
  kern<<<grid, kScThreads, Lay::kSmem, st>>>(ta, tq, bhi, blo, q_vec, mode, t, M, K, N, nkb, nsplit, C, ldc);
  TSB_CHECK_LAUNCH("screened_tc launch");
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
  cudaStream_t st = as_stream(stream);
  const int64_t nkb = (K + 127) / 128;
  const int64_t mt = (M + 127) / 128;
  const int bn = N > 128 ? 256 : 128;
  const int64_t nt = (N + bn - 1) / bn;
  int nsplit = 1;
  while (mt * nt * nsplit < sm_count() && nsplit * 2 <= nkb) nsplit *= 2;
  if (nsplit > 1 || K == 0) {
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
  const float t = static_cast<float>(sqrt(threshold));
  const float* qv = bounds_kind == 1 ? bounds : nullptr;
  return bn == 128 ? launch_sc<128>(ta, tq, bh, bl, qv, bounds_kind, t, M, K, N, (int)nkb, nsplit, C, ldc, st)
                   : launch_sc<256>(ta, tq, bh, bl, qv, bounds_kind, t, M, K, N, (int)nkb, nsplit, C, ldc, st);
}
