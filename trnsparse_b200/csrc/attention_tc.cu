// Block-sparse attention forward on the tensor cores (bf16 in/out, fp32
// softmax), block size 128, head_dim 64 or 128.
//
// Semantics are the reference's two-pass form (trnsparse/ops.py:280-357):
// pass 1 computes, per query row, the max and the stable exp-sum of
// scale * q.k over all stored key blocks; pass 2 recomputes the scores and
// accumulates exp(s - max) / max(sum, 1e-12) @ V. Keeping the two passes
// (3 GEMMs per block instead of an online softmax's 2) means the output
// accumulator never has to be rescaled, so it stays in TMEM and is written by
// the tensor cores only.
//
// One CTA = one (head, 128-row query block); 6 warps:
//   warp 4      TMA producer: Q once, then K (both passes) and V (pass 2)
//               into 2-stage rings (128-byte swizzle).
//   warp 5      TMEM owner and MMA issuer: S = Q K^T into one of two TMEM
//               score buffers; O += P V into the TMEM output (V is used
//               MN-major straight from its row-major layout).
//   warps 0-3   softmax: thread r owns query row r = its TMEM lane; reads S
//               with tcgen05.ld, keeps (max, sum) in registers (pass 1),
//               writes P = exp(s - max) / sum as bf16 into a 128-byte-swizzled
//               shared tile (pass 2), and finally drains O to global memory.
// All waits are bounded (ptx.cuh).
#include <cuda_bf16.h>

#include "tc_common.cuh"

namespace tsb {
namespace {

constexpr int kAtThreads = 192;

template <int HD>
struct AtLayout {
  static constexpr int kChunks = HD / 64;          // 128-byte column chunks of a Q/K/V row
  static constexpr int kTile = 128 * HD * 2;       // bytes of one 128-row Q/K/V tile
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kTile;            // 2 stages
  static constexpr int kV = kK + 2 * kTile;        // 2 stages
  static constexpr int kP = kV + 2 * kTile;        // 128 x 128 bf16 = 32 KB
  static constexpr int kSmem = kP + 128 * 128 * 2 + 1024;
  static constexpr int kTmemCols = 512;            // S0 [0,128), S1 [128,256), O [256, 256+HD)
};

// MN-major, 128-byte-swizzled operand (V as B of O += P V): 8-row atoms along
// K at 1024 bytes (SBO), 64-wide N chunks at `lbo` bytes (LBO).
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int HD>
__global__ void __launch_bounds__(kAtThreads, 1)
attn_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
               const __grid_constant__ CUtensorMap tv, const int* __restrict__ row_ptr,
               const int* __restrict__ col_idx, __nv_bfloat16* __restrict__ O, int seq, int m_tiles, float scale) {
  using Lay = AtLayout<HD>;
  extern __shared__ __align__(16) uint8_t dsmem_at[];
  __shared__ __align__(8) uint64_t q_full, o_done;
  __shared__ __align__(8) uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  __shared__ __align__(8) uint64_t s_full[2], s_empty[2], p_full, p_empty;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const uint32_t raw = smem_u32(dsmem_at);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const sb = dsmem_at + (base - raw);
  const int warp = threadIdx.x >> 5;
  const int qb = blockIdx.x, head = blockIdx.y;
  const int e0 = row_ptr[qb], e1 = row_ptr[qb + 1];
  const int nb = e1 - e0;
  const int steps = 2 * nb;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&o_done, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
    }
    mbar_init(&p_full, 128);
    mbar_init(&p_empty, 1);
    abort_flag = (base & 1023u) ? 1 : 0;
    if (abort_flag) record_device_error(DEVERR_SELFCHECK_SMEM);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(&tmem_slot, Lay::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const uint32_t t_o = tmem + 256;
  const int qrow0 = head * seq + qb * 128;
  const bool active = nb > 0 && !abort_flag;

  if (active) {
    if (warp == 4 && elect_lane0()) {
      // ---------------- TMA producer
      mbar_arrive_expect_tx(&q_full, Lay::kTile);
      for (int c = 0; c < Lay::kChunks; ++c) tma_load_2d(sb + Lay::kQ + c * 16384, &tq, c * 64, qrow0, &q_full);
      int vi = 0;
      for (int step = 0; step < steps; ++step) {
        const int blk = col_idx[e0 + (step % nb)];
        const int krow = head * seq + blk * 128;
        const int ks = step & 1, ku = step >> 1;
        if (ku > 0 && !mbar_wait(&k_empty[ks], (ku - 1) & 1)) { atomicExch(&abort_flag, 1); break; }
        if (*(volatile int*)&abort_flag) break;
        mbar_arrive_expect_tx(&k_full[ks], Lay::kTile);
        for (int c = 0; c < Lay::kChunks; ++c)
          tma_load_2d(sb + Lay::kK + ks * Lay::kTile + c * 16384, &tk, c * 64, krow, &k_full[ks]);
        if (step >= nb) {
          const int vs = vi & 1, vu = vi >> 1;
          if (vu > 0 && !mbar_wait(&v_empty[vs], (vu - 1) & 1)) { atomicExch(&abort_flag, 1); break; }
          mbar_arrive_expect_tx(&v_full[vs], Lay::kTile);
          for (int c = 0; c < Lay::kChunks; ++c)
            tma_load_2d(sb + Lay::kV + vs * Lay::kTile + c * 16384, &tv, c * 64, krow, &v_full[vs]);
          ++vi;
        }
      }
    } else if (warp == 5 && elect_lane0()) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc_s = make_idesc(MmaKind::BF16, 128, 128);
      constexpr uint32_t idesc_o = make_idesc(MmaKind::BF16, 128, HD) | (1u << 16);  // B (V) MN-major
      const uint32_t q_addr = smem_u32(sb + Lay::kQ);
      bool o_acc = false;
      bool ok = mbar_wait(&q_full, 0);
      auto issue_pv = [&](int j) {  // O += P_j V_j (pass-2 block j)
        const int vs = j & 1, vu = j >> 1;
        if (!mbar_wait(&p_full, j & 1) || !mbar_wait(&v_full[vs], vu & 1)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sb + Lay::kP);
        const uint32_t v_addr = smem_u32(sb + Lay::kV + vs * Lay::kTile);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // 128 keys, 16 per MMA
          const uint64_t ad = smem_desc_sw128(p_addr + (kk >> 2) * 16384 + (kk & 3) * 32);
          const uint64_t bd = smem_desc_sw128_mn(v_addr + kk * 2048, 16384);
          umma<MmaKind::BF16>(t_o, ad, bd, idesc_o, o_acc);
          o_acc = true;
        }
        umma_commit(&v_empty[vs]);
        umma_commit(&p_empty);
        return true;
      };
      for (int step = 0; ok && step < steps; ++step) {
        if (*(volatile int*)&abort_flag) { ok = false; break; }
        const int ks = step & 1, ku = step >> 1;
        const int sbuf = step & 1, su = step >> 1;
        if (!mbar_wait(&k_full[ks], ku & 1)) { ok = false; break; }
        if (su > 0 && !mbar_wait(&s_empty[sbuf], (su - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sb + Lay::kK + ks * Lay::kTile);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma<MmaKind::BF16>(tmem + sbuf * 128, smem_desc_sw128(q_addr + off), smem_desc_sw128(k_addr + off),
                              idesc_s, kk > 0);
        }
        umma_commit(&k_empty[ks]);
        umma_commit(&s_full[sbuf]);
        if (step - 1 >= nb && !issue_pv(step - 1 - nb)) { ok = false; break; }
      }
      if (ok && !issue_pv(nb - 1)) ok = false;
      if (!ok) atomicExch(&abort_flag, 1);
      umma_commit(&o_done);
    } else if (warp < 4) {
      // ---------------- softmax warps
      const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
      const int r = warp * 32 + (threadIdx.x & 31);
      float m = -INFINITY, l = 0.f, inv = 0.f;
      for (int step = 0; step < steps; ++step) {
        if (*(volatile int*)&abort_flag) break;
        const int sbuf = step & 1, su = step >> 1;
        if (!mbar_wait(&s_full[sbuf], su & 1)) { atomicExch(&abort_flag, 1); break; }
        tc_fence_after();
        if (step < nb) {
          // pass 1: running max / stable sum over the block's 128 scores
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t v[32];
            tmem_ld32(tmem + lane_base + sbuf * 128 + c * 32, v);
            tmem_wait_ld();
            float cm = -INFINITY;
#pragma unroll
            for (int i = 0; i < 32; ++i) cm = fmaxf(cm, __uint_as_float(v[i]) * scale);
            const float mn = fmaxf(m, cm);
            float sum = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) sum += __expf(__uint_as_float(v[i]) * scale - mn);
            l = l * __expf(m - mn) + sum;
            m = mn;
          }
          tc_fence_before();
          mbar_arrive(&s_empty[sbuf]);
          if (step == nb - 1) inv = 1.f / fmaxf(l, 1e-12f);
        } else {
          // pass 2: P = exp(s - m) / l as bf16 into the swizzled P tile
          const int j = step - nb;
          if (j > 0 && !mbar_wait(&p_empty, (j - 1) & 1)) { atomicExch(&abort_flag, 1); break; }
          uint8_t* prow = sb + Lay::kP + r * 128;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t v[32];
            tmem_ld32(tmem + lane_base + sbuf * 128 + c * 32, v);
            tmem_wait_ld();
            // keys 32c .. 32c+31 -> chunk (c >> 1), 16-byte units u = (c & 1) * 4 + 0..3
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint32_t w[4];
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                const float a = __expf(__uint_as_float(v[8 * q + 2 * h]) * scale - m) * inv;
                const float b = __expf(__uint_as_float(v[8 * q + 2 * h + 1]) * scale - m) * inv;
                w[h] = pack_bf16(a, b);
              }
              const int u = (c & 1) * 4 + q;
              uint4* dst = reinterpret_cast<uint4*>(prow + (c >> 1) * 16384 + ((u ^ (r & 7)) * 16));
              *dst = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
          tc_fence_before();
          mbar_arrive(&s_empty[sbuf]);
          fence_proxy_async_smem();
          mbar_arrive(&p_full);
        }
      }
    }
  }
  __syncwarp();
  // ---------------- epilogue: O (TMEM) -> bf16 rows in global memory
  bool ok = true;
  if (active) ok = mbar_wait(&o_done, 0);
  tc_fence_after();
  if (warp < 4 && qb < m_tiles) {
    const int r = warp * 32 + (threadIdx.x & 31);
    __nv_bfloat16* orow = O + static_cast<int64_t>(qrow0 + r) * HD;
    const bool have = active && ok && !*(volatile int*)&abort_flag;
#pragma unroll 1
    for (int c = 0; c < HD / 32; ++c) {
      uint32_t v[32];
      if (have) {
        tmem_ld32(t_o + (static_cast<uint32_t>(warp * 32) << 16) + c * 32, v);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0u;
      }
      uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        dst[q] = make_uint4(pack_bf16(__uint_as_float(v[8 * q]), __uint_as_float(v[8 * q + 1])),
                            pack_bf16(__uint_as_float(v[8 * q + 2]), __uint_as_float(v[8 * q + 3])),
                            pack_bf16(__uint_as_float(v[8 * q + 4]), __uint_as_float(v[8 * q + 5])),
                            pack_bf16(__uint_as_float(v[8 * q + 6]), __uint_as_float(v[8 * q + 7])));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, Lay::kTmemCols);
  }
}

template <int HD>
int launch_attn_tc(const void* Q, const void* K, const void* V, void* O, const int* rp, const int* ci, int heads,
                   int seq, float scale, cudaStream_t st) {
  using Lay = AtLayout<HD>;
  const uint64_t rows = static_cast<uint64_t>(heads) * seq;
  CUtensorMap tq, tk, tv;
  const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  int rc = make_tmap_2d(&tq, Q, dt, HD, rows, HD * 2, 64, 128);
  if (rc) return rc;
  rc = make_tmap_2d(&tk, K, dt, HD, rows, HD * 2, 64, 128);
  if (rc) return rc;
  rc = make_tmap_2d(&tv, V, dt, HD, rows, HD * 2, 64, 128);
  if (rc) return rc;
  auto kern = attn_tc_kernel<HD>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kSmem);
  if (e != cudaSuccess) return cuda_status(e, "attention_tc: set smem");
  const int m_tiles = seq / 128;
  dim3 grid((unsigned)m_tiles, (unsigned)heads);
  kern<<<grid, kAtThreads, Lay::kSmem, st>>>(tq, tk, tv, rp, ci, (__nv_bfloat16*)O, seq, m_tiles, scale);
  TSB_CHECK_LAUNCH("attention_tc launch");
  return debug_sync(st, "attention_tc (sync)");
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" int trnsparse_bsr_attention_tc(int64_t heads, int64_t seq, int64_t head_dim, const int* block_row_ptr,
                                          const int* block_col_idx, const void* Q, const void* K, const void* V,
                                          void* O, double scale, void* stream) {
  TSB_REQUIRE(heads > 0 && seq > 0 && seq % 128 == 0 && heads < 65536 && heads * seq < (1ll << 31),
              "attention_tc: needs seq %% 128 == 0 (got heads=%lld seq=%lld)", (long long)heads, (long long)seq);
  TSB_REQUIRE(head_dim == 64 || head_dim == 128, "attention_tc: head_dim must be 64 or 128 (got %lld)",
              (long long)head_dim);
  TSB_REQUIRE(Q && K && V && O && block_row_ptr && block_col_idx, "attention_tc: null pointer");
  cudaStream_t st = as_stream(stream);
  if (head_dim == 64)
    return launch_attn_tc<64>(Q, K, V, O, block_row_ptr, block_col_idx, (int)heads, (int)seq, (float)scale, st);
  return launch_attn_tc<128>(Q, K, V, O, block_row_ptr, block_col_idx, (int)heads, (int)seq, (float)scale, st);
}
