// Output tiles of X Y^T on the tensor cores (tcgen05 + TMA + TMEM): the
// adjoint products of the block-sparse ops.
//
//   BSR block gradient   dblocks[k] = dC[rows of block-row i] . B[rows of
//                        block-column j]^T for every stored block k = (i, j)
//                        (the reference's _BSRSpMMFunction.backward,
//                        trnsparse/nki/dispatch.py:331-369): X = dC (m x k),
//                        Y = B (n x k), one 128 x 128 tile per stored block,
//                        written packed in block order.
//   screened dA          dA = (dC B^T) o mask (_ScreenedSpMMFunction.backward,
//                        nki/dispatch.py:447-484): X = dC (M x N), Y = B
//                        (K x N), every 128 x 128 tile of the dense M x K
//                        result, the exact fp32 Schwarz mask applied in the
//                        epilogue (1-D: fl(sqrt|d_r| sqrt|d_c|) > t, 2-D:
//                        Q[r, c] > t).
//
// X and Y are row-major with the contraction index contiguous, so both are
// K-major MMA operands loaded as they lie (TMA, 128-byte swizzle). fp32 runs
// 3xTF32 on tf32 hi / lo copies made by one split pass into the workspace
// (zero-padded to a whole 32-wide K chunk); bf16 runs kind::f16 on the
// operands in place (a padded copy only when a row is not 16-byte aligned or
// K < 64). Persistent CTAs (one per SM, 6 warps) take tiles round-robin:
//   warp 0      TMA producer (X and Y chunks into a ring of stages)
//   warp 1      TMEM owner and MMA issuer, two 128 x 128 fp32 accumulators
//               used alternately so a tile's MMAs overlap the previous
//               tile's epilogue
//   warps 2-5   epilogue: TMEM lane quadrant = warp % 4, 32-row x 128-byte
//               pieces through a swizzled staging tile and a TMA store
#include <algorithm>

#include "tc_common.cuh"

namespace tsb {
namespace {

constexpr int kNtThreads = 192;
constexpr int kNtSmemMax = 232448;

template <MmaKind KIND>
struct NtCfg {
  static constexpr int kElem = KIND == MmaKind::TF32 ? 4 : 2;
  static constexpr int kChunk = 128 / kElem;                    // K elements per 128-byte chunk
  static constexpr int kParts = KIND == MmaKind::TF32 ? 2 : 1;  // hi (+ lo)
  static constexpr int kTile = 128 * 128;                       // 128 rows x 128 bytes
  static constexpr int kStage = 2 * kParts * kTile;             // X parts, then Y parts
  static constexpr int kEpi = 4 * 2 * 4096;
  static constexpr int kBarBytes = 512;
  static constexpr int kAlign = 1024;
  static constexpr int kStagesFit = (kNtSmemMax - kAlign - kEpi - kBarBytes) / kStage;
  static constexpr int kStages = kStagesFit > 6 ? 6 : kStagesFit;
  static constexpr int kEpiOff = kStages * kStage;
  static constexpr int kBarOff = kEpiOff + kEpi;
  static constexpr int kSmem = kBarOff + kBarBytes + kAlign;
  static_assert(kStages >= 2, "operand ring");
};

struct NtBars {
  uint64_t full[6], empty[6], acc_full[2], acc_empty[2];
  uint32_t tmem_slot;
  int abort_flag;
};

// Tile u: packed (tiles != nullptr): (i, j) = tiles[2u], tiles[2u+1], written at rows
// [128u, 128u + 128) of a 128-column output; dense (tiles == nullptr): (i, j) = (u / nj, u % nj),
// written at [128 i, 128 j] of the out_rows x out_cols output.
struct NtTile {
  int i, j, ox, oy;
};
__device__ __forceinline__ NtTile nt_tile(const int* tiles, int nj, int u) {
  NtTile t;
  if (tiles) {
    t.i = tiles[2 * u];
    t.j = tiles[2 * u + 1];
    t.ox = 0;
    t.oy = 128 * u;
  } else {
    t.i = u / nj;
    t.j = u - t.i * nj;
    t.ox = 128 * t.j;
    t.oy = 128 * t.i;
  }
  return t;
}

// MASK 0: none; 1: q_vec holds the diagonal integrals (keep fl(sqrt|d_r| sqrt|d_c|) > t);
// 2: qmat (ldq) holds the pair bounds (keep Q[r, c] > t). Masks apply to dense outputs.
template <MmaKind KIND, bool OUT_BF16, int MASK>
__global__ void __launch_bounds__(kNtThreads, 1)
nt_tc_kernel(const __grid_constant__ CUtensorMap tx_hi, const __grid_constant__ CUtensorMap tx_lo,
             const __grid_constant__ CUtensorMap ty_hi, const __grid_constant__ CUtensorMap ty_lo,
             const __grid_constant__ CUtensorMap tout, const int* __restrict__ tiles, int n_tiles, int nj,
             int n_chunks, int64_t out_rows, int64_t out_cols, const float* __restrict__ q_vec,
             const float* __restrict__ qmat, int64_t ldq, float t) {
  using Cfg = NtCfg<KIND>;
  constexpr int S = Cfg::kStages;
  extern __shared__ __align__(16) uint8_t nt_smem[];
  const uint32_t raw = smem_u32(nt_smem);
  uint8_t* const sbase = nt_smem + (((raw + 1023u) & ~1023u) - raw);
  NtBars& Bs = *reinterpret_cast<NtBars*>(sbase + Cfg::kBarOff);
  auto x_tile = [&](int s, int part) { return sbase + s * Cfg::kStage + part * Cfg::kTile; };
  auto y_tile = [&](int s, int part) { return sbase + s * Cfg::kStage + (Cfg::kParts + part) * Cfg::kTile; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&Bs.full[s], 1);
      mbar_init(&Bs.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&Bs.acc_full[i], 1);
      mbar_init(&Bs.acc_empty[i], 128);
    }
    Bs.abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tx_hi);
    tma_prefetch_desc(&ty_hi);
    tma_prefetch_desc(&tout);
  }
  if (warp == 1) {
    tmem_alloc(&Bs.tmem_slot, 256);
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
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < n_tiles; u += gridDim.x) {
        const NtTile tl = nt_tile(tiles, nj, u);
        for (int c = 0; c < n_chunks; ++c, ++it) {
          const int s = it % S, use = it / S;
          if (use > 0 && !mbar_wait(&Bs.empty[s], (use - 1) & 1)) { ok = false; break; }
          if (*abort_flag) { ok = false; break; }
          mbar_arrive_expect_tx(&Bs.full[s], Cfg::kStage);
          tma_load_2d(x_tile(s, 0), &tx_hi, c * Cfg::kChunk, tl.i * 128, &Bs.full[s]);
          tma_load_2d(y_tile(s, 0), &ty_hi, c * Cfg::kChunk, tl.j * 128, &Bs.full[s]);
          if constexpr (KIND == MmaKind::TF32) {
            tma_load_2d(x_tile(s, 1), &tx_lo, c * Cfg::kChunk, tl.i * 128, &Bs.full[s]);
            tma_load_2d(y_tile(s, 1), &ty_lo, c * Cfg::kChunk, tl.j * 128, &Bs.full[s]);
          }
        }
      }
      if (!ok) {
        atomicExch(&Bs.abort_flag, 1);
        for (int i = (it > S ? it - S : 0); i < it; ++i) mbar_wait(&Bs.full[i % S], (i / S) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(KIND, 128, 128);  // both operands K-major
      int it = 0, q = 0;
      bool ok = !*abort_flag;
      for (int u = blockIdx.x; ok && u < n_tiles; u += gridDim.x, ++q) {
        const int acc = q & 1;
        if (q >= 2 && !mbar_wait(&Bs.acc_empty[acc], ((q >> 1) - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + acc * 128;
        for (int c = 0; c < n_chunks; ++c, ++it) {
          const int s = it % S, use = it / S;
          if (*abort_flag || !mbar_wait(&Bs.full[s], use & 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t xh = smem_u32(x_tile(s, 0)), yh = smem_u32(y_tile(s, 0));
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {  // 4 MMAs of 32 bytes of K per 128-byte chunk
            const uint32_t off = ks * 32;
            const bool accum = c > 0 || ks > 0;
            umma<KIND>(d, smem_desc_sw128(xh + off), smem_desc_sw128(yh + off), idesc, accum);
            if constexpr (KIND == MmaKind::TF32) {
              const uint32_t xl = smem_u32(x_tile(s, 1)), yl = smem_u32(y_tile(s, 1));
              umma<KIND>(d, smem_desc_sw128(xh + off), smem_desc_sw128(yl + off), idesc, true);
              umma<KIND>(d, smem_desc_sw128(xl + off), smem_desc_sw128(yh + off), idesc, true);
            }
          }
          umma_commit(&Bs.empty[s]);
        }
        if (!ok) break;
        umma_commit(&Bs.acc_full[acc]);
      }
      if (!ok) atomicExch(&Bs.abort_flag, 1);
    }
  } else {
    // ---------------- epilogue warps 2-5
    const int quad = warp & 3;
    uint8_t* const stage0 = sbase + Cfg::kEpiOff + (warp - 2) * 8192;
    constexpr int PW = OUT_BF16 ? 64 : 32;  // output columns per 128-byte staged row
    int q = 0, pc = 0;
    bool ok = !*abort_flag;
    for (int u = blockIdx.x; u < n_tiles; u += gridDim.x, ++q) {
      const NtTile tl = nt_tile(tiles, nj, u);
      const int acc = q & 1;
      ok = ok && mbar_wait(&Bs.acc_full[acc], (q >> 1) & 1) && !*abort_flag;
      tc_fence_after();
      const bool run = __all_sync(0xffffffffu, ok);
      const uint32_t t_row = tmem + acc * 128 + (static_cast<uint32_t>(quad * 32) << 16);
      const int64_t row = static_cast<int64_t>(tl.oy) + quad * 32 + lane;  // this lane's output row
      float qr = 0.f;
      if (MASK == 1 && row < out_rows) qr = __fsqrt_rn(fabsf(q_vec[row]));
#pragma unroll 1
      for (int p = 0; run && p < 128 / PW && tl.ox + p * PW < out_cols; ++p, ++pc) {
        uint8_t* stage = stage0 + (pc & 1) * 4096;
        if (pc >= 2) {
          if (lane == 0) bulk_wait_read_1();
          __syncwarp();
        }
        uint32_t v0[32], v1[32];
        tmem_ld32(t_row + p * PW, v0);
        if constexpr (OUT_BF16) tmem_ld32(t_row + p * PW + 32, v1);
        tmem_wait_ld();
        if constexpr (MASK != 0) {
          const int64_t c0 = static_cast<int64_t>(tl.ox) + p * PW;
#pragma unroll
          for (int e = 0; e < PW; ++e) {
            const int64_t col = c0 + e;
            bool keep = false;
            if (row < out_rows && col < out_cols) {
              if (MASK == 1) keep = __fmul_rn(qr, __fsqrt_rn(fabsf(__ldg(q_vec + col)))) > t;
              else keep = __ldg(qmat + row * ldq + col) > t;
            }
            uint32_t& w = e < 32 ? v0[e] : v1[e - 32];
            if (!keep) w = 0u;
          }
        }
        uint32_t w[32];
        if constexpr (OUT_BF16) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            w[i] = pack_bf16(__uint_as_float(v0[2 * i]), __uint_as_float(v0[2 * i + 1]));
            w[16 + i] = pack_bf16(__uint_as_float(v1[2 * i]), __uint_as_float(v1[2 * i + 1]));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = v0[i];
        }
#pragma unroll
        for (int x = 0; x < 8; ++x)
          *reinterpret_cast<uint4*>(stage + lane * 128 + ((x ^ (lane & 7)) * 16)) =
              make_uint4(w[4 * x], w[4 * x + 1], w[4 * x + 2], w[4 * x + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && tl.oy + quad * 32 < out_rows) {
          tma_store_2d(&tout, stage, tl.ox + p * PW, tl.oy + quad * 32);
          bulk_commit_group();
        }
      }
      tc_fence_before();
      mbar_arrive(&Bs.acc_empty[acc]);
    }
    if (lane == 0) bulk_wait_all();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// hi / lo tf32 split of a rows x K row-major fp32 matrix (leading dimension ld) into
// rows x Kp matrices, zero past column K.
__global__ void split_pad_kernel(int64_t rows, int64_t K, const float* __restrict__ src, int64_t ld, int64_t Kp,
                                 float* __restrict__ hi, float* __restrict__ lo) {
  grid_dep_launch();
  const int64_t total = rows * Kp;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = e / Kp, c = e - r * Kp;
    const float x = c < K ? src[r * ld + c] : 0.f;
    const float h = tf32_rna(x);
    hi[e] = h;
    lo[e] = tf32_rna(x - h);
  }
}

// rows x K bf16 -> rows x Kp (zero-padded), for operands TMA cannot read in place.
__global__ void pad_bf16_kernel(int64_t rows, int64_t K, const uint16_t* __restrict__ src, int64_t ld, int64_t Kp,
                                uint16_t* __restrict__ dst) {
  const int64_t total = rows * Kp;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = e / Kp, c = e - r * Kp;
    dst[e] = c < K ? src[r * ld + c] : uint16_t(0);
  }
}

template <MmaKind KIND, bool OUT_BF16, int MASK>
int launch_nt(const CUtensorMap& xh, const CUtensorMap& xl, const CUtensorMap& yh, const CUtensorMap& yl,
              const CUtensorMap& om, const int* tiles, int n_tiles, int nj, int n_chunks, int64_t out_rows,
              int64_t out_cols, const float* q_vec, const float* qmat, int64_t ldq, float t, cudaStream_t st) {
  using Cfg = NtCfg<KIND>;
  auto kern = nt_tc_kernel<KIND, OUT_BF16, MASK>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem);
  if (e != cudaSuccess) return cuda_status(e, "nt_tc: set smem");
  const int grid = n_tiles < sm_count() ? n_tiles : sm_count();
  e = launch_pdl(kern, dim3(grid), dim3(kNtThreads), Cfg::kSmem, st, xh, xl, yh, yl, om, tiles, n_tiles, nj, n_chunks,
                 out_rows, out_cols, q_vec, qmat, ldq, t);
  if (e != cudaSuccess) return cuda_status(e, "nt_tc launch");
  return debug_sync(st, "nt_tc: main kernel (sync)");
}

inline int64_t nt_pad_k(int64_t K, int dtype) {
  const int64_t chunk = dtype == TRNSPARSE_F32 ? 32 : 64;
  return (K + chunk - 1) / chunk * chunk;
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" size_t trnsparse_nt_tc_workspace_size(int64_t mx, int64_t my, int64_t K, int dtype) {
  if (mx < 0 || my < 0 || K < 0) return 0;
  const int64_t Kp = nt_pad_k(K, dtype);
  if (dtype == TRNSPARSE_F32) return 2 * align256(4 * (size_t)mx * Kp) + 2 * align256(4 * (size_t)my * Kp);
  return align256(2 * (size_t)mx * Kp) + align256(2 * (size_t)my * Kp);
}

extern "C" int trnsparse_nt_tc(int64_t mx, int64_t my, int64_t K, int dtype, const void* X, int64_t ldx,
                               const void* Y, int64_t ldy, const int* tiles, int64_t n_tiles, void* out,
                               int64_t ldo, int out_dtype, int64_t out_rows, int64_t out_cols, int mask_kind,
                               const float* bounds, int64_t ldq, double threshold, void* ws, size_t ws_bytes,
                               void* stream) {
  TSB_REQUIRE(mx >= 0 && my >= 0 && K >= 0 && n_tiles >= 0, "nt_tc: negative size");
  TSB_REQUIRE(dtype == TRNSPARSE_F32 || dtype == TRNSPARSE_BF16, "nt_tc: dtype must be F32 or BF16");
  TSB_REQUIRE(out_dtype == TRNSPARSE_F32 || out_dtype == TRNSPARSE_BF16, "nt_tc: out_dtype must be F32 or BF16");
  TSB_REQUIRE(mask_kind >= 0 && mask_kind <= 2, "nt_tc: mask_kind must be 0, 1 or 2");
  TSB_REQUIRE(mask_kind == 0 || (tiles == nullptr && bounds), "nt_tc: a mask needs the dense layout and bounds");
  TSB_REQUIRE(ldx >= K && ldy >= K, "nt_tc: leading dimension smaller than K");
  const bool packed = tiles != nullptr;
  const int64_t mt = (mx + 127) / 128, nt = (my + 127) / 128;
  if (!packed) {
    TSB_REQUIRE(out_rows <= mx && out_cols <= my, "nt_tc: dense output larger than X Y^T");
    n_tiles = mt * nt;
  }
  if (n_tiles == 0 || (!packed && (out_rows == 0 || out_cols == 0))) return TRNSPARSE_OK;
  TSB_REQUIRE(out && X && Y, "nt_tc: null pointer");
  TSB_REQUIRE(n_tiles < (1ll << 31) / 128 && mx < (1ll << 31) && my < (1ll << 31), "nt_tc: sizes out of range");
  const int osz = out_dtype == TRNSPARSE_BF16 ? 2 : 4;
  const int64_t ocols = packed ? 128 : out_cols;
  const int64_t orows = packed ? 128 * n_tiles : out_rows;
  TSB_REQUIRE(ldo >= ocols && (ldo * osz) % 16 == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0,
              "nt_tc: out must be 16-byte aligned with 16-byte rows");
  const size_t need = trnsparse_nt_tc_workspace_size(mx, my, K, dtype);
  TSB_REQUIRE(ws_bytes >= need && (need == 0 || ws), "nt_tc: workspace too small (%zu < %zu)", ws_bytes, need);
  cudaStream_t st = as_stream(stream);
  const int64_t Kp = nt_pad_k(K, dtype);
  const int n_chunks = static_cast<int>(Kp / (dtype == TRNSPARSE_F32 ? 32 : 64));
  CUtensorMap xh, xl, yh, yl, om;
  int rc;
  if (dtype == TRNSPARSE_F32) {
    float* xhi = static_cast<float*>(ws);
    float* xlo = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xhi) + align256(4 * (size_t)mx * Kp));
    float* yhi = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xlo) + align256(4 * (size_t)mx * Kp));
    float* ylo = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(yhi) + align256(4 * (size_t)my * Kp));
    auto grid_of = [](int64_t n) { return static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 16 * sm_count())); };
    if (mx * Kp > 0)
      split_pad_kernel<<<grid_of(mx * Kp), 256, 0, st>>>(mx, K, static_cast<const float*>(X), ldx, Kp, xhi, xlo);
    if (my * Kp > 0)
      split_pad_kernel<<<grid_of(my * Kp), 256, 0, st>>>(my, K, static_cast<const float*>(Y), ldy, Kp, yhi, ylo);
    TSB_CHECK_LAUNCH("nt_tc: split operands");
    const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    rc = make_tmap_2d(&xh, xhi, dt, (uint64_t)Kp, (uint64_t)mx, 4 * Kp, 32, 128);
    if (!rc) rc = make_tmap_2d(&xl, xlo, dt, (uint64_t)Kp, (uint64_t)mx, 4 * Kp, 32, 128);
    if (!rc) rc = make_tmap_2d(&yh, yhi, dt, (uint64_t)Kp, (uint64_t)my, 4 * Kp, 32, 128);
    if (!rc) rc = make_tmap_2d(&yl, ylo, dt, (uint64_t)Kp, (uint64_t)my, 4 * Kp, 32, 128);
    if (rc) return rc;
  } else {
    const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    auto place = [&](const void* src, int64_t rows, int64_t ld, void* spare, const void** use, int64_t* use_ld) {
      if (K >= 64 && ld % 8 == 0 && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        *use = src;
        *use_ld = ld;
        return;
      }
      if (rows * Kp > 0)
        pad_bf16_kernel<<<(unsigned)std::min<int64_t>((rows * Kp + 255) / 256, 16 * sm_count()), 256, 0, st>>>(
            rows, K, static_cast<const uint16_t*>(src), ld, Kp, static_cast<uint16_t*>(spare));
      *use = spare;
      *use_ld = Kp;
    };
    const void *xs, *ys;
    int64_t xld, yld;
    void* xspare = ws;
    void* yspare = ws ? static_cast<uint8_t*>(ws) + align256(2 * (size_t)mx * Kp) : nullptr;
    place(X, mx, ldx, xspare, &xs, &xld);
    place(Y, my, ldy, yspare, &ys, &yld);
    TSB_CHECK_LAUNCH("nt_tc: pad operands");
    const uint64_t kcols = (uint64_t)(xs == X ? K : Kp);
    rc = make_tmap_2d(&xh, xs, dt, xs == X ? (uint64_t)K : (uint64_t)Kp, (uint64_t)mx, 2 * xld, 64, 128);
    if (!rc) rc = make_tmap_2d(&yh, ys, dt, ys == Y ? (uint64_t)K : (uint64_t)Kp, (uint64_t)my, 2 * yld, 64, 128);
    (void)kcols;
    if (rc) return rc;
    xl = xh;
    yl = yh;
  }
  rc = out_dtype == TRNSPARSE_BF16
           ? make_tmap_2d(&om, out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)ocols, (uint64_t)orows, 2 * ldo, 64, 32)
           : make_tmap_2d(&om, out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (uint64_t)ocols, (uint64_t)orows, 4 * ldo, 32, 32);
  if (rc) return rc;
  const float t = static_cast<float>(sqrt(threshold));
  const int nj = static_cast<int>(nt);
  const int nt_i = static_cast<int>(n_tiles);
  const float* qv = mask_kind == 1 ? bounds : nullptr;
  const float* qm = mask_kind == 2 ? bounds : nullptr;
#define TSB_NT_LAUNCH(K_, OB_, M_) \
  launch_nt<K_, OB_, M_>(xh, xl, yh, yl, om, tiles, nt_i, nj, n_chunks, orows, ocols, qv, qm, ldq, t, st)
  const bool ob = out_dtype == TRNSPARSE_BF16;
  if (dtype == TRNSPARSE_F32) {
    if (mask_kind == 1) return ob ? TSB_NT_LAUNCH(MmaKind::TF32, true, 1) : TSB_NT_LAUNCH(MmaKind::TF32, false, 1);
    if (mask_kind == 2) return ob ? TSB_NT_LAUNCH(MmaKind::TF32, true, 2) : TSB_NT_LAUNCH(MmaKind::TF32, false, 2);
    return ob ? TSB_NT_LAUNCH(MmaKind::TF32, true, 0) : TSB_NT_LAUNCH(MmaKind::TF32, false, 0);
  }
  if (mask_kind == 1) return ob ? TSB_NT_LAUNCH(MmaKind::BF16, true, 1) : TSB_NT_LAUNCH(MmaKind::BF16, false, 1);
  if (mask_kind == 2) return ob ? TSB_NT_LAUNCH(MmaKind::BF16, true, 2) : TSB_NT_LAUNCH(MmaKind::BF16, false, 2);
  return ob ? TSB_NT_LAUNCH(MmaKind::BF16, true, 0) : TSB_NT_LAUNCH(MmaKind::BF16, false, 0);
#undef TSB_NT_LAUNCH
}
