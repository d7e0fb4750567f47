// Peer-memory communication for the block-row-sharded solvers (one process
// per GPU, all GPUs of one NVLink/NVSwitch box).
//
// Each rank allocates one buffer with trnsparse_peer_alloc and shares its
// CUDA IPC handle; every rank opens every other rank's buffer, so a kernel can
// store straight into a peer's memory over NVLink. The buffer holds the
// rank's solver workspace (so halo rows are written directly into the
// receiver's vectors) followed by a small exchange area:
//   flags[3][world]      int64, written by rank q into slot [area][q]
//   vals[3][world][4]    float64 partial sums, same indexing (up to four per exchange)
//   epoch                int64, bumped once per solve on every rank
//   tickets[4]           uint32 CTA arrival counters of the solver kernels
// trnsparse_peer_reduce_push replaces "all-reduce two doubles + halo
// exchange" with one single-CTA kernel: push halo rows and the local partials
// to every peer, fence, raise this rank's flag on every peer, wait (bounded)
// for every peer's flag, then sum the partials in rank order, so every rank
// gets bit-identical totals. Flags hold increasing sequence numbers
// (epoch * stride + step + 1), so nothing is ever reset. Three areas: the
// solve's setup exchange uses area 2 and iterations alternate 0 / 1, so two
// consecutive exchanges never share an area (a rank may run one exchange
// ahead of a peer, never two) — including across back-to-back solves.
//
// Plain stores and loads only: no TMA, no multicast.
#include <string.h>

#include "common.cuh"
#include "ptx.cuh"

namespace tsb {
namespace {

__device__ __forceinline__ void st_release_sys(long long* p, long long v) {
  asm volatile("st.release.sys.global.s64 [%0], %1;\n" ::"l"(p), "l"(v) : "memory");
}

struct CommArea {
  long long* flags;  // [3][world]
  double* vals;      // [3][world][4]
  long long* epoch;
};

__device__ __forceinline__ CommArea area_of(char* base, size_t comm_off, int world) {
  CommArea a;
  a.flags = reinterpret_cast<long long*>(base + comm_off);
  a.vals = reinterpret_cast<double*>(base + comm_off + 24 * world);
  a.epoch = reinterpret_cast<long long*>(base + comm_off + 120 * world);
  return a;
}

constexpr int kMaxWorld = 16;

__global__ void __launch_bounds__(256)
reduce_push_kernel(char* const* __restrict__ peers, int world, int rank, size_t comm_off, double* my_a, double* my_b,
                   int area, long long stride, long long step, const float* __restrict__ src,
                   const long long* __restrict__ sends, int n_sends, int chunk) {
  __shared__ long long seq_s;
  char* mine = peers[rank];
  const CommArea me = area_of(mine, comm_off, world);
  if (threadIdx.x == 0) seq_s = (*me.epoch) * stride + step + 1;
  // 1. halo rows: each send = (source element offset, destination rank, destination byte offset)
  for (int s = 0; s < n_sends; ++s) {
    const long long so = sends[3 * s], dr = sends[3 * s + 1], dofs = sends[3 * s + 2];
    float* dst = reinterpret_cast<float*>(peers[dr] + dofs);
    for (int i = threadIdx.x; i < chunk / 4; i += blockDim.x)
      reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src + so)[i];
  }
  __syncthreads();
  const long long seq = seq_s;
  // 2. local partials into every rank's vals[area][rank]
  if (threadIdx.x < world) {
    const CommArea pq = area_of(peers[threadIdx.x], comm_off, world);
    double* v = pq.vals + (static_cast<size_t>(area) * world + rank) * 4;
    v[0] = my_a ? *my_a : 0.0;
    v[1] = my_b ? *my_b : 0.0;
  }
  // the stores above happen-before (barrier) each flag's release at system scope
  __syncthreads();
  // 3. raise this rank's flag on every peer
  if (threadIdx.x < world) {
    const CommArea pq = area_of(peers[threadIdx.x], comm_off, world);
    st_release_sys(pq.flags + static_cast<size_t>(area) * world + rank, seq);
  }
  // 4. wait for every peer's flag in this rank's area (bounded)
  // bounded; once any exchange has timed out, later ones do not wait again
  if (threadIdx.x < world && *(volatile int*)&g_device_error != DEVERR_PEER_TIMEOUT)
    wait_flag_geq(me.flags + static_cast<size_t>(area) * world + threadIdx.x, seq, 64);
  __syncthreads();
  // 5. totals in rank order (identical on every rank)
  if (threadIdx.x == 0) {
    __threadfence_system();
    double ta = 0.0, tb = 0.0;
    for (int q = 0; q < world; ++q) {
      const volatile double* v = me.vals + (static_cast<size_t>(area) * world + q) * 4;
      ta += v[0];
      tb += v[1];
    }
    if (my_a) *my_a = ta;
    if (my_b) *my_b = tb;
  }
}

__global__ void bump_epoch_kernel(char* mine, size_t comm_off, int world) {
  const CommArea me = area_of(mine, comm_off, world);
  *me.epoch += 1;
}

}  // namespace
}  // namespace tsb

using namespace tsb;

extern "C" size_t trnsparse_peer_comm_bytes(int world) { return static_cast<size_t>(120 * world + 64); }

extern "C" int trnsparse_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  TSB_REQUIRE(bytes > 0 && ptr && ipc_handle, "peer_alloc: bad argument");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_status(e, "peer_alloc: cudaMalloc");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_status(e, "peer_alloc: IPC handle");
  }
  *ptr = p;
  return TRNSPARSE_OK;
}

extern "C" int trnsparse_peer_open(const void* ipc_handle, void** ptr) {
  TSB_REQUIRE(ipc_handle && ptr, "peer_open: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return cuda_status(e, "peer_open: cudaIpcOpenMemHandle");
}

extern "C" int trnsparse_peer_close(void* ptr) { return cuda_status(cudaIpcCloseMemHandle(ptr), "peer_close"); }

extern "C" int trnsparse_peer_free(void* ptr) { return cuda_status(cudaFree(ptr), "peer_free"); }

extern "C" int trnsparse_peer_bump_epoch(void* mine, size_t comm_off, int world, void* stream) {
  TSB_REQUIRE(mine && world > 0, "peer_bump_epoch: bad argument");
  bump_epoch_kernel<<<1, 1, 0, as_stream(stream)>>>(static_cast<char*>(mine), comm_off, world);
  TSB_CHECK_LAUNCH("peer_bump_epoch");
  return TRNSPARSE_OK;
}

extern "C" int trnsparse_peer_reduce_push(void* const* peers, int world, int rank, size_t comm_off, double* my_a,
                                          double* my_b, int area, long long stride, long long step,
                                          const float* src, const long long* sends, int n_sends, int chunk,
                                          void* stream) {
  TSB_REQUIRE(peers && world > 0 && world <= kMaxWorld && rank >= 0 && rank < world && area >= 0 && area <= 2,
              "peer_reduce_push: bad argument");
  TSB_REQUIRE(n_sends == 0 || (src && sends && chunk > 0 && chunk % 4 == 0), "peer_reduce_push: bad halo list");
  reduce_push_kernel<<<1, 256, 0, as_stream(stream)>>>(reinterpret_cast<char* const*>(peers), world, rank, comm_off,
                                                      my_a, my_b, area, stride, step, src, sends, n_sends, chunk);
  TSB_CHECK_LAUNCH("peer_reduce_push");
  return TRNSPARSE_OK;
}
