// BSR SpMV and the fused BSR iterative solvers (CG, Chebyshev, Richardson,
// power iteration) of trnsparse/iterative.py, with every scalar kept on the
// device: no host round trip per iteration. Each solver iteration is one
// fused SpMV launch (plus one vector launch for CG); convergence tests run at
// the start of the next launch, which returns early once a status word says
// the solve is finished, so the host only polls the status between chunks of
// iterations.
//
// Arithmetic follows the reference's tensor expressions operation by
// operation (separate roundings, scalars rounded to float32 where torch
// would), except that inner products are accumulated in float64.
#include "bsr_mv.cuh"
#include "ptx.cuh"

#include <math.h>

namespace tsb {
namespace {

enum { REASON_NONE = 0, REASON_CONVERGED = 1, REASON_MAXITER = 2, REASON_BREAKDOWN = 3, REASON_ZERO_RHS = 4 };

// First 64 bytes of every solver workspace (layout mirrored in Python).
struct SolverStatus {
  int done;
  int iters;
  int reason;
  int pad;
  double rel;   // final relative residual (CG) / eigenvalue (power)
  double bb;    // ||b||^2
  double pad2[4];
};
static_assert(sizeof(SolverStatus) == 64, "status layout");

// CG uses slot k as {a: p_k.Ap_k, b: r_0.z_0 (slot 0 only), c: r_{k+1}.r_{k+1},
// d: r_{k+1}.z_{k+1}}; c and d are adjacent so a distributed solve can reduce
// both with one collective. Power iteration uses {a: lambda, b: ||A v||^2}.
struct Slot { double a, b, c, d; };

__device__ __forceinline__ double cg_rz(const Slot* s, int k) { return k == 0 ? s[0].b : s[k - 1].d; }

inline size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

struct CgWs {
  SolverStatus* st;
  Slot* slots;   // max_iter + 2
  float *r, *p0, *p1, *ap;
};

inline size_t cg_ws_size(int64_t n, int max_iter) {
  return align256(64) + align256(sizeof(Slot) * (size_t)(max_iter + 2)) + 4 * align256(sizeof(float) * (size_t)n);
}

inline CgWs cg_ws(void* base, int64_t n, int max_iter) {
  char* p = static_cast<char*>(base);
  CgWs w;
  w.st = reinterpret_cast<SolverStatus*>(p);
  p += align256(64);
  w.slots = reinterpret_cast<Slot*>(p);
  p += align256(sizeof(Slot) * (size_t)(max_iter + 2));
  const size_t vb = align256(sizeof(float) * (size_t)n);
  w.r = reinterpret_cast<float*>(p);
  w.p0 = reinterpret_cast<float*>(p + vb);
  w.p1 = reinterpret_cast<float*>(p + 2 * vb);
  w.ap = reinterpret_cast<float*>(p + 3 * vb);
  return w;
}

__device__ __forceinline__ void set_done(SolverStatus* st, int iters, int reason, double rel) {
  st->iters = iters;
  st->reason = reason;
  st->rel = rel;
  __threadfence();
  st->done = 1;
}

// ---------------------------------------------------------------- plain SpMV
struct PlainOp {
  static constexpr int kDots = 0;
  const float* xv;
  const float* yin;
  float* out;
  float alpha, beta;
  __device__ bool begin(int) const { return true; }
  __device__ float x(int64_t c) const { return xv[c]; }
  __device__ float4 x4(int64_t c) const { return ld4(xv + c); }
  __device__ void row(int64_t r, float y, double*, double*) const {
    float v = __fmul_rn(alpha, y);
    if (yin) v = __fadd_rn(v, __fmul_rn(beta, yin[r]));
    out[r] = v;
  }
  __device__ void finish(double, double) const {}
};

// ---------------------------------------------------------------- vector kernel
// Element-wise op over n entries with up to two float64 partial sums.
template <class Op>
__global__ void __launch_bounds__(256) vec_kernel(int64_t n, Op op) {
  __shared__ double red[8];
  if (!op.begin(blockIdx.x)) return;
  double d0 = 0.0, d1 = 0.0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * 256)
    op.elem(i, &d0, &d1);
  const double t0 = block_sum256(d0, red);
  const double t1 = block_sum256(d1, red);
  if (threadIdx.x == 0) op.finish(t0, t1);
  run_tail(op);
}

inline unsigned vec_grid(int64_t n) {
  int64_t g = (n + 255) / 256;
  const int64_t cap = 4 * static_cast<int64_t>(sm_count());
  if (g > cap) g = cap;
  return static_cast<unsigned>(g < 1 ? 1 : g);
}

// ---------------------------------------------------------------- CG
// r0 = b (x0 == 0) ; z0 = M r0 ; p_{-1} = 0 ; bb = b.b ; rz_0 = r0.z0
struct CgStartVec {
  const float *b, *inv_d;
  CgWs w;
  __device__ bool begin(int) const { return true; }
  __device__ void elem(int64_t i, double* d0, double* d1) const {
    const float r = b[i];
    w.r[i] = r;
    w.p1[i] = 0.f;
    const float z = inv_d ? __fmul_rn(r, inv_d[i]) : r;
    *d0 += (double)b[i] * (double)b[i];
    *d1 += (double)r * (double)z;
  }
  __device__ void finish(double t0, double t1) const {
    atomicAdd(&w.st->bb, t0);
    atomicAdd(&w.slots[0].b, t1);
  }
};

// r0 = b - A x0 (fused into the SpMV epilogue)
struct CgStartMv {
  static constexpr int kDots = 2;
  const float *b, *x0, *inv_d;
  CgWs w;
  __device__ bool begin(int) const { return true; }
  __device__ float x(int64_t c) const { return x0[c]; }
  __device__ float4 x4(int64_t c) const { return ld4(x0 + c); }
  __device__ void row(int64_t i, float y, double* d0, double* d1) const {
    const float r = __fsub_rn(b[i], y);
    w.r[i] = r;
    w.p1[i] = 0.f;
    const float z = inv_d ? __fmul_rn(r, inv_d[i]) : r;
    *d0 += (double)b[i] * (double)b[i];
    *d1 += (double)r * (double)z;
  }
  __device__ void finish(double t0, double t1) const {
    atomicAdd(&w.st->bb, t0);
    atomicAdd(&w.slots[0].b, t1);
  }
};

// Iteration k, part 1: tail of iteration k-1 (convergence test, beta), then
// p_k = z_k + beta_k p_{k-1} gathered on the fly, Ap = A p_k, pAp partials.
struct CgMv {
  static constexpr int kDots = 1;
  const float* inv_d;
  CgWs w;
  const float* pprev;
  float* pcur;
  int k, max_iter;
  double tol;
  int64_t halo_begin;  // columns >= halo_begin are halo copies of other ranks' rows (sharded solve)
  mutable float beta;
  __device__ bool begin(int cta) const {
    SolverStatus* st = w.st;
    if (*(volatile int*)&st->done) return false;
    const double bnorm = sqrt(st->bb);
    if (k == 0) {
      if (bnorm < 1e-15) {
        if (cta == 0 && threadIdx.x == 0) set_done(st, 0, REASON_ZERO_RHS, 0.0);
        return false;
      }
      beta = 0.f;
      return true;
    }
    const double rel = (double)(float)sqrt(w.slots[k - 1].c) / bnorm;
    if (rel < tol) {
      if (cta == 0 && threadIdx.x == 0) set_done(st, k, REASON_CONVERGED, rel);
      return false;
    }
    if (k >= max_iter) {
      if (cta == 0 && threadIdx.x == 0) set_done(st, max_iter, REASON_MAXITER, rel);
      return false;
    }
    beta = (float)(cg_rz(w.slots, k) / cg_rz(w.slots, k - 1));
    return true;
  }
  __device__ __forceinline__ float pk(int64_t c) const {
    const float r = w.r[c];
    const float z = inv_d ? __fmul_rn(r, inv_d[c]) : r;
    return __fadd_rn(z, __fmul_rn(beta, pprev[c]));
  }
  // Halo entries of p_k are stored by whichever thread computes them (every
  // writer stores the same value), so the next iteration finds p_k there.
  __device__ float x(int64_t c) const {
    const float p = pk(c);
    if (c >= halo_begin) pcur[c] = p;
    return p;
  }
  __device__ float4 x4(int64_t c) const {
    const float4 p = make_float4(pk(c), pk(c + 1), pk(c + 2), pk(c + 3));
    if (c >= halo_begin) *reinterpret_cast<float4*>(pcur + c) = p;
    return p;
  }
  __device__ void row(int64_t i, float y, double* d0, double*) const {
    const float p = pk(i);
    pcur[i] = p;
    w.ap[i] = y;
    *d0 += (double)p * (double)y;
  }
  __device__ void finish(double t0, double) const { atomicAdd(&w.slots[k].a, t0); }
};

// Iteration k, part 2: breakdown test, alpha, x += alpha p, r -= alpha Ap,
// partial r.r (slot k) and r.z (slot k+1).
struct CgUpdate {
  const float* inv_d;
  float* x;
  CgWs w;
  const float* pcur;
  int k, max_iter;
  mutable float alpha;
  __device__ bool begin(int cta) const {
    SolverStatus* st = w.st;
    if (*(volatile int*)&st->done) return false;
    const double pap = w.slots[k].a;
    if (fabs(pap) < 1e-30) {
      if (cta == 0 && threadIdx.x == 0) {
        const double rel = k > 0 ? (double)(float)sqrt(w.slots[k - 1].c) / sqrt(st->bb) : nan("");
        set_done(st, max_iter, REASON_BREAKDOWN, rel);
      }
      return false;
    }
    alpha = (float)(cg_rz(w.slots, k) / pap);
    return true;
  }
  __device__ void elem(int64_t i, double* d0, double* d1) const {
    x[i] = __fadd_rn(x[i], __fmul_rn(alpha, pcur[i]));
    const float r = __fsub_rn(w.r[i], __fmul_rn(alpha, w.ap[i]));
    w.r[i] = r;
    const float z = inv_d ? __fmul_rn(r, inv_d[i]) : r;
    *d0 += (double)r * (double)r;
    *d1 += (double)r * (double)z;
  }
  __device__ void finish(double t0, double t1) const {
    atomicAdd(&w.slots[k].c, t0);
    atomicAdd(&w.slots[k].d, t1);
  }
};

// ---------------------------------------------------------------- Chebyshev / Richardson
// x_{k+1} = x_k + a_k (b - A x_k) [+ b_k (x_k - x_{k-1})]
struct ChebMv {
  static constexpr int kDots = 0;
  const float *b, *xk, *xprev;
  float* xnext;
  float a, bcoef;
  bool momentum;
  __device__ bool begin(int) const { return true; }
  __device__ float x(int64_t c) const { return xk[c]; }
  __device__ float4 x4(int64_t c) const { return ld4(xk + c); }
  __device__ void row(int64_t i, float y, double*, double*) const {
    const float r = __fsub_rn(b[i], y);
    float xn = __fadd_rn(xk[i], __fmul_rn(a, r));
    if (momentum) xn = __fadd_rn(xn, __fmul_rn(bcoef, __fsub_rn(xk[i], xprev[i])));
    xnext[i] = xn;
  }
  __device__ void finish(double, double) const {}
};

// ||b - A x||^2 into *acc
struct ResidualMv {
  static constexpr int kDots = 1;
  const float *b, *xv;
  double* acc;
  __device__ bool begin(int) const { return true; }
  __device__ float x(int64_t c) const { return xv[c]; }
  __device__ float4 x4(int64_t c) const { return ld4(xv + c); }
  __device__ void row(int64_t i, float y, double* d0, double*) const {
    const float r = __fsub_rn(b[i], y);
    *d0 += (double)r * (double)r;
  }
  __device__ void finish(double t0, double) const { atomicAdd(acc, t0); }
};

struct DotVec {
  const float *u, *v;
  double* acc;
  __device__ bool begin(int) const { return true; }
  __device__ void elem(int64_t i, double* d0, double*) const { *d0 += (double)u[i] * (double)v[i]; }
  __device__ void finish(double t0, double) const { atomicAdd(acc, t0); }
};

// ---------------------------------------------------------------- power iteration
struct PowWs {
  SolverStatus* st;
  Slot* slots;  // slot k+1 holds (v_k . A v_k, ||A v_k||^2); slot 0 holds ||v0||^2 in .b
  float *av0, *av1;
};

inline size_t pow_ws_size(int64_t n, int max_iter) {
  return align256(64) + align256(sizeof(Slot) * (size_t)(max_iter + 2)) + 2 * align256(sizeof(float) * (size_t)n);
}

inline PowWs pow_ws(void* base, int64_t n, int max_iter) {
  char* p = static_cast<char*>(base);
  PowWs w;
  w.st = reinterpret_cast<SolverStatus*>(p);
  p += align256(64);
  w.slots = reinterpret_cast<Slot*>(p);
  p += align256(sizeof(Slot) * (size_t)(max_iter + 2));
  const size_t vb = align256(sizeof(float) * (size_t)n);
  w.av0 = reinterpret_cast<float*>(p);
  w.av1 = reinterpret_cast<float*>(p + vb);
  return w;
}

// v_k = src / ||src|| (src = v0 for k = 0, else A v_{k-1}); A v_k; partials.
struct PowMv {
  static constexpr int kDots = 2;
  PowWs w;
  const float* src;
  float* vout;
  float* avout;
  int k, max_iter;
  double tol;
  mutable float nrm;
  __device__ bool begin(int cta) const {
    SolverStatus* st = w.st;
    if (*(volatile int*)&st->done) return false;
    nrm = (float)sqrt(w.slots[k].b);
    if (k > 0) {
      if ((double)nrm < 1e-30) {
        if (cta == 0 && threadIdx.x == 0) set_done(st, k, REASON_BREAKDOWN, 0.0);
        return false;
      }
      const double lam = w.slots[k].a;
      const double lam_prev = k > 1 ? w.slots[k - 1].a : 0.0;
      if (fabs(lam - lam_prev) < tol) {
        if (cta == 0 && threadIdx.x == 0) set_done(st, k, REASON_CONVERGED, lam);
        return false;
      }
      if (k >= max_iter) {
        if (cta == 0 && threadIdx.x == 0) set_done(st, max_iter, REASON_MAXITER, lam);
        return false;
      }
    }
    return true;
  }
  __device__ __forceinline__ float vk(int64_t c) const { return __fdiv_rn(src[c], nrm); }
  __device__ float x(int64_t c) const { return vk(c); }
  __device__ float4 x4(int64_t c) const { return make_float4(vk(c), vk(c + 1), vk(c + 2), vk(c + 3)); }
  __device__ void row(int64_t i, float y, double* d0, double* d1) const {
    const float v = vk(i);
    vout[i] = v;
    avout[i] = y;
    *d0 += (double)v * (double)y;
    *d1 += (double)y * (double)y;
  }
  __device__ void finish(double t0, double t1) const {
    atomicAdd(&w.slots[k + 1].a, t0);
    atomicAdd(&w.slots[k + 1].b, t1);
  }
};

// After the loop: if the solve stopped on convergence or the iteration cap,
// the returned vector is A v_{k-1} / ||A v_{k-1}||.
struct PowFinal {
  PowWs w;
  float* vout;
  mutable float nrm;
  mutable const float* src;
  __device__ bool begin(int) const {
    const SolverStatus* st = w.st;
    if (!st->done || st->reason == REASON_BREAKDOWN || st->iters < 1) return false;
    const int k = st->iters;
    nrm = (float)sqrt(w.slots[k].b);
    src = ((k - 1) & 1) ? w.av1 : w.av0;
    return true;
  }
  __device__ void elem(int64_t i, double*, double*) const { vout[i] = __fdiv_rn(src[i], nrm); }
  __device__ void finish(double, double) const {}
};

struct PowStart {
  const float* v0;
  PowWs w;
  __device__ bool begin(int) const { return true; }
  __device__ void elem(int64_t i, double* d0, double*) const { *d0 += (double)v0[i] * (double)v0[i]; }
  __device__ void finish(double t0, double) const { atomicAdd(&w.slots[0].b, t0); }
};

// ---------------------------------------------------------------- helpers
int check_desc(const BsrDesc& d, const char* what) {
  if (d.m < 0 || d.n < 0 || d.b <= 0 || d.n_blocks < 0)
    return fail(TRNSPARSE_ERR_ARG, "%s: bad BSR geometry (m=%lld n=%lld b=%d n_blocks=%lld)", what, (long long)d.m,
                (long long)d.n, d.b, (long long)d.n_blocks);
  if (!d.row_ptr || (d.n_blocks > 0 && (!d.col_idx || !d.blocks)))
    return fail(TRNSPARSE_ERR_ARG, "%s: null BSR array", what);
  return TRNSPARSE_OK;
}

bool all_aligned(std::initializer_list<const void*> ps) {
  for (const void* p : ps)
    if (p && !aligned16(p)) return false;
  return true;
}

template <class Op>
int launch_vec(int64_t n, const Op& op, cudaStream_t st, const char* what, unsigned max_ctas = 0) {
  unsigned g = vec_grid(n);
  if (max_ctas > 0 && g > max_ctas) g = max_ctas;
  vec_kernel<Op><<<g, 256, 0, st>>>(n, op);
  TSB_CHECK_LAUNCH(what);
  return TRNSPARSE_OK;
}

}  // namespace
}  // namespace tsb

using namespace tsb;

#define BSR_DESC_ARGS int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr, const int* col_idx, const float* blocks
#define BSR_DESC BsrDesc{m, n, b, n_blocks, row_ptr, col_idx, blocks}

extern "C" int trnsparse_bsr_spmv(BSR_DESC_ARGS, const float* x, double alpha, const float* y, double beta, float* out,
                                  void* stream) {
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_spmv");
  if (rc) return rc;
  if (m == 0) return TRNSPARSE_OK;
  TSB_REQUIRE(x && out, "bsr_spmv: null x/out");
  if (y && beta == 0.0) y = nullptr;
  PlainOp op{x, y, out, (float)alpha, (float)beta};
  return launch_bsr_mv(d, op, all_aligned({x}), as_stream(stream), "bsr_spmv launch");
}

extern "C" size_t trnsparse_bsr_cg_workspace_size(int64_t n, int max_iter) {
  return cg_ws_size(n < 0 ? 0 : n, max_iter < 0 ? 0 : max_iter);
}

extern "C" int trnsparse_bsr_cg_start(BSR_DESC_ARGS, const float* b_vec, const float* x, int x_is_zero,
                                      const float* inv_d, int max_iter, void* ws, size_t ws_bytes, void* stream) {
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_cg_start");
  if (rc) return rc;
  TSB_REQUIRE(m == n, "bsr_cg: A must be square (got %lld x %lld)", (long long)m, (long long)n);
  TSB_REQUIRE(max_iter >= 0, "bsr_cg: max_iter < 0");
  TSB_REQUIRE(ws && ws_bytes >= cg_ws_size(n, max_iter), "bsr_cg: workspace too small (%zu < %zu)", ws_bytes,
              cg_ws_size(n, max_iter));
  TSB_REQUIRE(b_vec && x, "bsr_cg: null b/x");
  cudaStream_t st = as_stream(stream);
  const CgWs w = cg_ws(ws, n, max_iter);
  cudaError_t e = cudaMemsetAsync(ws, 0, align256(64) + align256(sizeof(Slot) * (size_t)(max_iter + 2)), st);
  if (e != cudaSuccess) return cuda_status(e, "bsr_cg_start: memset");
  if (n == 0) return TRNSPARSE_OK;
  if (x_is_zero) return launch_vec(n, CgStartVec{b_vec, inv_d, w}, st, "bsr_cg_start vec");
  CgStartMv op{b_vec, x, inv_d, w};
  return launch_bsr_mv(d, op, all_aligned({x}), st, "bsr_cg_start mv");
}

extern "C" int trnsparse_bsr_cg_iterate(BSR_DESC_ARGS, float* x, const float* inv_d, double tol, int max_iter,
                                        int k_begin, int k_end, void* ws, void* stream) {
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_cg_iterate");
  if (rc) return rc;
  TSB_REQUIRE(ws && x, "bsr_cg_iterate: null workspace/x");
  TSB_REQUIRE(0 <= k_begin && k_begin <= k_end && k_end <= max_iter + 1, "bsr_cg_iterate: bad range [%d, %d)", k_begin,
              k_end);
  if (n == 0) return TRNSPARSE_OK;
  cudaStream_t st = as_stream(stream);
  const CgWs w = cg_ws(ws, n, max_iter);
  const bool vec_ok = all_aligned({inv_d, w.r, w.p0, w.p1});
  for (int k = k_begin; k < k_end; ++k) {
    float* pcur = (k & 1) ? w.p1 : w.p0;
    const float* pprev = (k & 1) ? w.p0 : w.p1;
    CgMv mv{inv_d, w, pprev, pcur, k, max_iter, tol, n, 0.f};
    rc = launch_bsr_mv(d, mv, vec_ok, st, "bsr_cg mv");
    if (rc) return rc;
    if (k >= max_iter) break;  // the launch above only records the final status
    rc = launch_vec(n, CgUpdate{inv_d, x, w, pcur, k, max_iter, 0.f}, st, "bsr_cg update");
    if (rc) return rc;
  }
  return TRNSPARSE_OK;
}

extern "C" int trnsparse_bsr_chebyshev(BSR_DESC_ARGS, const float* b_vec, const float* alpha, const float* beta, int K,
                                       float* x, float* work, double* rr_out, void* stream) {
  // alpha/beta: host arrays of K float32 coefficients; x: x0 in, x_K out;
  // work: 2n floats of scratch; rr_out: device double, receives ||b - A x_K||^2.
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_chebyshev");
  if (rc) return rc;
  TSB_REQUIRE(m == n, "bsr_chebyshev: A must be square");
  TSB_REQUIRE(K >= 0 && (K == 0 || (alpha && beta)), "bsr_chebyshev: bad coefficients");
  TSB_REQUIRE(b_vec && x && work && rr_out, "bsr_chebyshev: null pointer");
  if (n == 0) return TRNSPARSE_OK;
  cudaStream_t st = as_stream(stream);
  float* buf[3] = {x, work, work + n};
  const bool vec_ok = all_aligned({x, work, work + n});
  // x_{-1} = x_0 (reference: x_prev = x.clone()); only read when k > 0
  for (int k = 0; k < K; ++k) {
    const float* xk = buf[k % 3];
    const float* xp = buf[(k + 2) % 3];
    float* xn = buf[(k + 1) % 3];
    ChebMv op{b_vec, xk, xp, xn, alpha[k], beta[k], k > 0};
    rc = launch_bsr_mv(d, op, vec_ok, st, "bsr_chebyshev mv");
    if (rc) return rc;
  }
  if (K % 3 != 0) {
    cudaError_t e = cudaMemcpyAsync(x, buf[K % 3], sizeof(float) * (size_t)n, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_status(e, "bsr_chebyshev: copy result");
  }
  cudaError_t e = cudaMemsetAsync(rr_out, 0, sizeof(double), st);
  if (e != cudaSuccess) return cuda_status(e, "bsr_chebyshev: memset");
  return launch_bsr_mv(d, ResidualMv{b_vec, x, rr_out}, all_aligned({x}), st, "bsr_chebyshev residual");
}

extern "C" int trnsparse_bsr_richardson(BSR_DESC_ARGS, const float* b_vec, double omega, int K, float* x, float* work,
                                        double* rr_out, void* stream) {
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_richardson");
  if (rc) return rc;
  TSB_REQUIRE(m == n, "bsr_richardson: A must be square");
  TSB_REQUIRE(K >= 0 && b_vec && x && work && rr_out, "bsr_richardson: bad argument");
  if (n == 0) return TRNSPARSE_OK;
  cudaStream_t st = as_stream(stream);
  float* buf[2] = {x, work};
  const bool vec_ok = all_aligned({x, work});
  for (int k = 0; k < K; ++k) {
    ChebMv op{b_vec, buf[k & 1], nullptr, buf[(k + 1) & 1], (float)omega, 0.f, false};
    rc = launch_bsr_mv(d, op, vec_ok, st, "bsr_richardson mv");
    if (rc) return rc;
  }
  if (K & 1) {
    cudaError_t e = cudaMemcpyAsync(x, work, sizeof(float) * (size_t)n, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_status(e, "bsr_richardson: copy result");
  }
  cudaError_t e = cudaMemsetAsync(rr_out, 0, sizeof(double), st);
  if (e != cudaSuccess) return cuda_status(e, "bsr_richardson: memset");
  return launch_bsr_mv(d, ResidualMv{b_vec, x, rr_out}, all_aligned({x}), st, "bsr_richardson residual");
}

extern "C" int trnsparse_dot(int64_t n, const float* u, const float* v, double* acc, void* stream) {
  TSB_REQUIRE(n >= 0 && u && v && acc, "dot: bad argument");
  cudaStream_t st = as_stream(stream);
  cudaError_t e = cudaMemsetAsync(acc, 0, sizeof(double), st);
  if (e != cudaSuccess) return cuda_status(e, "dot: memset");
  if (n == 0) return TRNSPARSE_OK;
  return launch_vec(n, DotVec{u, v, acc}, st, "dot");
}

extern "C" size_t trnsparse_bsr_power_workspace_size(int64_t n, int max_iter) {
  return pow_ws_size(n < 0 ? 0 : n, max_iter < 0 ? 0 : max_iter);
}

extern "C" int trnsparse_bsr_power_iterate(BSR_DESC_ARGS, const float* v0, float* v, double tol, int max_iter,
                                           int k_begin, int k_end, void* ws, size_t ws_bytes, void* stream) {
  // k_begin == 0 starts the solve (clears the workspace, ||v0||); k_end ==
  // max_iter + 1 also writes the final vector into v.
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_power");
  if (rc) return rc;
  TSB_REQUIRE(m == n, "bsr_power: A must be square");
  TSB_REQUIRE(max_iter >= 0 && v0 && v && ws && ws_bytes >= pow_ws_size(n, max_iter), "bsr_power: bad argument");
  TSB_REQUIRE(0 <= k_begin && k_begin <= k_end && k_end <= max_iter + 1, "bsr_power: bad range");
  if (n == 0) return TRNSPARSE_OK;
  cudaStream_t st = as_stream(stream);
  const PowWs w = pow_ws(ws, n, max_iter);
  if (k_begin == 0) {
    cudaError_t e = cudaMemsetAsync(ws, 0, align256(64) + align256(sizeof(Slot) * (size_t)(max_iter + 2)), st);
    if (e != cudaSuccess) return cuda_status(e, "bsr_power: memset");
    rc = launch_vec(n, PowStart{v0, w}, st, "bsr_power start");
    if (rc) return rc;
  }
  const bool vec_ok = all_aligned({v0, w.av0, w.av1});
  for (int k = k_begin; k < k_end; ++k) {
    const float* src = k == 0 ? v0 : (((k - 1) & 1) ? w.av1 : w.av0);
    float* av = (k & 1) ? w.av1 : w.av0;
    PowMv op{w, src, v, av, k, max_iter, tol, 0.f};
    rc = launch_bsr_mv(d, op, vec_ok, st, "bsr_power mv");
    if (rc) return rc;
  }
  if (k_end == max_iter + 1) return launch_vec(n, PowFinal{w, v, 0.f, nullptr}, st, "bsr_power final");
  return TRNSPARSE_OK;
}

extern "C" int trnsparse_bsr_power_finish(int64_t n, float* v, int max_iter, void* ws, void* stream) {
  TSB_REQUIRE(n >= 0 && v && ws, "bsr_power_finish: bad argument");
  if (n == 0) return TRNSPARSE_OK;
  const PowWs w = pow_ws(ws, n, max_iter);
  return launch_vec(n, PowFinal{w, v, 0.f, nullptr}, as_stream(stream), "bsr_power final");
}

// Clears the status record, the scalar slots and the p / Ap vectors of a CG
// workspace, but not r: in a sharded solve a faster peer may already have
// stored this solve's halo rows of r before this rank starts (the own part of
// r is written by the start kernel).
inline cudaError_t clear_cg_ws(void* ws, int64_t n_ext, int max_iter, cudaStream_t st) {
  const size_t head = align256(64) + align256(sizeof(Slot) * (size_t)(max_iter + 2));
  const size_t vb = align256(sizeof(float) * (size_t)n_ext);
  cudaError_t e = cudaMemsetAsync(ws, 0, head, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(static_cast<char*>(ws) + head + vb, 0, 3 * vb, st);
  return e;
}

// ---------------------------------------------------------------- sharded CG
// A rank owns rows [0, n_own) of its block-rows; its BSR geometry has
// m = n_own rows and n = n_ext columns, columns >= n_own being halo copies of
// other ranks' rows. Vectors in the workspace are n_ext long. The caller
// reduces the scalar slots across ranks between phases and refreshes the
// halo part of r (and, once, inv_d) from the owning ranks.

extern "C" int trnsparse_bsr_cg_layout(int64_t n, int max_iter, size_t* offsets) {
  TSB_REQUIRE(offsets && n >= 0 && max_iter >= 0, "bsr_cg_layout: bad argument");
  const size_t slots = align256(64);
  const size_t vec0 = slots + align256(sizeof(Slot) * (size_t)(max_iter + 2));
  const size_t vb = align256(sizeof(float) * (size_t)n);
  offsets[0] = 0;           // status record
  offsets[1] = slots;       // Slot[max_iter + 2], 32 bytes each
  offsets[2] = vec0;        // r
  offsets[3] = vec0 + vb;   // p (even k)
  offsets[4] = vec0 + 2 * vb;  // p (odd k)
  offsets[5] = vec0 + 3 * vb;  // Ap
  return TRNSPARSE_OK;
}

extern "C" int trnsparse_bsr_cg_dist_start(int64_t n_own, int64_t n_ext, const float* b_vec, const float* inv_d,
                                           int max_iter, void* ws, size_t ws_bytes, void* stream) {
  TSB_REQUIRE(n_own >= 0 && n_ext >= n_own && max_iter >= 0 && b_vec && ws, "bsr_cg_dist_start: bad argument");
  TSB_REQUIRE(ws_bytes >= cg_ws_size(n_ext, max_iter), "bsr_cg_dist_start: workspace too small");
  cudaStream_t st = as_stream(stream);
  cudaError_t e = clear_cg_ws(ws, n_ext, max_iter, st);
  if (e != cudaSuccess) return cuda_status(e, "bsr_cg_dist_start: memset");
  if (n_own == 0) return TRNSPARSE_OK;
  return launch_vec(n_own, CgStartVec{b_vec, inv_d, cg_ws(ws, n_ext, max_iter)}, st, "bsr_cg_dist_start");
}

extern "C" int trnsparse_bsr_cg_dist_phase(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                                           const int* col_idx, const float* blocks, float* x, const float* inv_d,
                                           double tol, int max_iter, int k, int phase, void* ws, void* stream) {
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_cg_dist_phase");
  if (rc) return rc;
  TSB_REQUIRE(ws && x && k >= 0 && k <= max_iter && (phase == 0 || phase == 1), "bsr_cg_dist_phase: bad argument");
  if (m == 0) return TRNSPARSE_OK;
  cudaStream_t st = as_stream(stream);
  const CgWs w = cg_ws(ws, n, max_iter);
  float* pcur = (k & 1) ? w.p1 : w.p0;
  const float* pprev = (k & 1) ? w.p0 : w.p1;
  if (phase == 0) {
    CgMv mv{inv_d, w, pprev, pcur, k, max_iter, tol, m, 0.f};
    return launch_bsr_mv(d, mv, all_aligned({inv_d, w.r, w.p0, w.p1}), st, "bsr_cg_dist mv");
  }
  if (k >= max_iter) return TRNSPARSE_OK;
  return launch_vec(m, CgUpdate{inv_d, x, w, pcur, k, max_iter, 0.f}, st, "bsr_cg_dist update");
}

// ---------------------------------------------------------------- sharded CG, communication fused
// Same iteration as the sharded phases above, but the exchanges happen inside
// the solver kernels: the last CTA of a kernel (ticket counter) pushes this
// rank's partial sums — and, after the x/r update, its boundary rows of r —
// straight into every peer's buffer over NVLink and raises its flag; the next
// kernel's CTAs wait (bounded) in their prologue for every peer's flag and
// sum the partials in rank order. Two launches per iteration, no host
// involvement. The buffers are the CUDA-IPC mapped ones of trnsparse_peer_*;
// the exchange area layout is the one documented in peer.cu, with three
// ticket counters after the epoch.
namespace tsb {
namespace {

struct PeerCtx {
  char* const* peers;   // device array, world entries
  int world, rank;
  size_t comm_off;
  long long stride;
  const long long* sends;  // halo r rows: (src elem offset, dst rank, dst byte offset)
  int n_sends, chunk;
};

__device__ __forceinline__ long long* pc_flags(const PeerCtx& p, char* base) {
  return reinterpret_cast<long long*>(base + p.comm_off);
}
__device__ __forceinline__ double* pc_vals(const PeerCtx& p, char* base) {
  return reinterpret_cast<double*>(base + p.comm_off + 24 * p.world);
}
__device__ __forceinline__ long long* pc_epoch(const PeerCtx& p, char* base) {
  return reinterpret_cast<long long*>(base + p.comm_off + 72 * p.world);
}
__device__ __forceinline__ unsigned int* pc_ticket(const PeerCtx& p, int which) {
  return reinterpret_cast<unsigned int*>(p.peers[p.rank] + p.comm_off + 72 * p.world + 8) + which;
}
__device__ __forceinline__ long long pc_seq(const PeerCtx& p, long long step) {
  return (*reinterpret_cast<volatile long long*>(pc_epoch(p, p.peers[p.rank]))) * p.stride + step + 1;
}

__device__ __forceinline__ long long ld_acq_sys(const long long* q) {
  long long v;
  asm volatile("ld.acquire.sys.global.s64 %0, [%1];\n" : "=l"(v) : "l"(q) : "memory");
  return v;
}
__device__ __forceinline__ void st_rel_sys(long long* q, long long v) {
  asm volatile("st.release.sys.global.s64 [%0], %1;\n" ::"l"(q), "l"(v) : "memory");
}

// All threads of the CTA: wait for every rank's flag of `area` to reach the
// step's sequence number, then return the rank-ordered sums of its partials.
__device__ double2 pc_wait_sum(const PeerCtx& p, int area, long long step) {
  __shared__ double2 tot;
  char* mine = p.peers[p.rank];
  const long long seq = pc_seq(p, step);
  if (threadIdx.x < p.world) {
    const long long* f = pc_flags(p, mine) + area * p.world + threadIdx.x;
    uint32_t i = 0;
    while (ld_acq_sys(f) < seq) {
      if (++i > kSpinLimit) {
        record_device_error(DEVERR_PEER_TIMEOUT);
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const volatile double* v = pc_vals(p, mine) + area * p.world * 2;
    double a = 0.0, b = 0.0;
    for (int q = 0; q < p.world; ++q) {
      a += v[2 * q];
      b += v[2 * q + 1];
    }
    tot = make_double2(a, b);
  }
  __syncthreads();
  return tot;
}

// All threads: if this is the kernel's last CTA, publish the complete local
// partials (*a, *b) and optionally the halo rows of `src`, then raise flags.
__device__ void pc_publish(const PeerCtx& p, int which, int area, long long step, const double* a, const double* b,
                           const float* src, bool halo) {
  __shared__ int last;
  __shared__ double2 part;
  __syncthreads();  // every thread's stores of this CTA precede the ticket
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned t = atomicAdd(pc_ticket(p, which), 1u);
    last = ((t + 1) % gridDim.x) == 0;
    if (last) {
      __threadfence();
      part = make_double2(a ? *(volatile const double*)a : 0.0, b ? *(volatile const double*)b : 0.0);
    }
  }
  __syncthreads();
  if (!last) return;
  const long long seq = pc_seq(p, step);
  if (halo) {
    for (int s = 0; s < p.n_sends; ++s) {
      const long long so = p.sends[3 * s], dr = p.sends[3 * s + 1], dofs = p.sends[3 * s + 2];
      float4* dst = reinterpret_cast<float4*>(p.peers[dr] + dofs);
      const volatile float4* sp = reinterpret_cast<const volatile float4*>(src + so);
      for (int i = threadIdx.x; i < p.chunk / 4; i += blockDim.x) {
        const float4 v = make_float4(sp[i].x, sp[i].y, sp[i].z, sp[i].w);
        dst[i] = v;
      }
    }
  }
  if (threadIdx.x < p.world) {
    double* v = pc_vals(p, p.peers[threadIdx.x]) + (area * p.world + p.rank) * 2;
    v[0] = part.x;
    v[1] = part.y;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < p.world) st_rel_sys(pc_flags(p, p.peers[threadIdx.x]) + area * p.world + p.rank, seq);
}

// step numbering: 0 = setup, 1 + 2k = p.Ap of iteration k, 2 + 2k = r.r / r.z of iteration k

struct CgStartFused {
  const float *b, *inv_d;
  CgWs w;
  PeerCtx p;
  __device__ bool begin(int) const { return true; }
  __device__ void elem(int64_t i, double* d0, double* d1) const {
    const float r = b[i];
    w.r[i] = r;
    const float z = inv_d ? __fmul_rn(r, inv_d[i]) : r;
    *d0 += (double)b[i] * (double)b[i];
    *d1 += (double)r * (double)z;
  }
  __device__ void finish(double t0, double t1) const {
    atomicAdd(&w.st->bb, t0);
    atomicAdd(&w.slots[0].b, t1);
  }
  __device__ void tail() const { pc_publish(p, 0, 2, 0, &w.st->bb, &w.slots[0].b, w.r, true); }
};

struct CgMvFused {
  static constexpr int kDots = 1;
  const float* inv_d;
  CgWs w;
  const float* pprev;
  float* pcur;
  int k, max_iter;
  double tol;
  int64_t halo_begin;
  PeerCtx p;
  mutable float beta;
  __device__ bool begin(int cta) const {
    SolverStatus* st = w.st;
    if (*(volatile int*)&st->done) return false;
    const double2 t = k == 0 ? pc_wait_sum(p, 2, 0) : pc_wait_sum(p, 1, 2 + 2 * (k - 1));
    if (k == 0) {
      const double bnorm = sqrt(t.x);
      if (cta == 0 && threadIdx.x == 0) {
        st->bb = t.x;
        w.slots[0].b = t.y;
      }
      if (bnorm < 1e-15) {
        if (cta == 0 && threadIdx.x == 0) set_done(st, 0, REASON_ZERO_RHS, 0.0);
        return false;
      }
      beta = 0.f;
      return true;
    }
    if (cta == 0 && threadIdx.x == 0) {
      w.slots[k - 1].c = t.x;
      w.slots[k - 1].d = t.y;
    }
    const double bnorm = sqrt(*(volatile double*)&st->bb);
    const double rel = (double)(float)sqrt(t.x) / bnorm;
    if (rel < tol) {
      if (cta == 0 && threadIdx.x == 0) set_done(st, k, REASON_CONVERGED, rel);
      return false;
    }
    if (k >= max_iter) {
      if (cta == 0 && threadIdx.x == 0) set_done(st, max_iter, REASON_MAXITER, rel);
      return false;
    }
    const double rz_prev = k == 1 ? *(volatile double*)&w.slots[0].b : *(volatile double*)&w.slots[k - 2].d;
    beta = (float)(t.y / rz_prev);
    return true;
  }
  __device__ __forceinline__ float pk(int64_t c) const {
    const float r = w.r[c];
    const float z = inv_d ? __fmul_rn(r, inv_d[c]) : r;
    return __fadd_rn(z, __fmul_rn(beta, pprev[c]));
  }
  __device__ float x(int64_t c) const {
    const float v = pk(c);
    if (c >= halo_begin) pcur[c] = v;
    return v;
  }
  __device__ float4 x4(int64_t c) const {
    const float4 v = make_float4(pk(c), pk(c + 1), pk(c + 2), pk(c + 3));
    if (c >= halo_begin) *reinterpret_cast<float4*>(pcur + c) = v;
    return v;
  }
  __device__ void row(int64_t i, float y, double* d0, double*) const {
    const float v = pk(i);
    pcur[i] = v;
    w.ap[i] = y;
    *d0 += (double)v * (double)y;
  }
  __device__ void finish(double t0, double) const { atomicAdd(&w.slots[k].a, t0); }
  __device__ void tail() const { pc_publish(p, 1, 0, 1 + 2 * k, &w.slots[k].a, nullptr, nullptr, false); }
};

struct CgUpdateFused {
  const float* inv_d;
  float* x;
  CgWs w;
  const float* pcur;
  int k, max_iter;
  PeerCtx p;
  mutable float alpha;
  __device__ bool begin(int cta) const {
    SolverStatus* st = w.st;
    if (*(volatile int*)&st->done) return false;
    const double2 t = pc_wait_sum(p, 0, 1 + 2 * k);
    const double pap = t.x;
    if (cta == 0 && threadIdx.x == 0) w.slots[k].a = pap;
    if (fabs(pap) < 1e-30) {
      if (cta == 0 && threadIdx.x == 0) {
        const double rel = k > 0 ? (double)(float)sqrt(*(volatile double*)&w.slots[k - 1].c) /
                                       sqrt(*(volatile double*)&st->bb)
                                 : nan("");
        set_done(st, max_iter, REASON_BREAKDOWN, rel);
      }
      return false;
    }
    const double rz = k == 0 ? *(volatile double*)&w.slots[0].b : *(volatile double*)&w.slots[k - 1].d;
    alpha = (float)(rz / pap);
    return true;
  }
  __device__ void elem(int64_t i, double* d0, double* d1) const {
    x[i] = __fadd_rn(x[i], __fmul_rn(alpha, pcur[i]));
    const float r = __fsub_rn(w.r[i], __fmul_rn(alpha, w.ap[i]));
    w.r[i] = r;
    const float z = inv_d ? __fmul_rn(r, inv_d[i]) : r;
    *d0 += (double)r * (double)r;
    *d1 += (double)r * (double)z;
  }
  __device__ void finish(double t0, double t1) const {
    atomicAdd(&w.slots[k].c, t0);
    atomicAdd(&w.slots[k].d, t1);
  }
  __device__ void tail() const { pc_publish(p, 2, 1, 2 + 2 * k, &w.slots[k].c, &w.slots[k].d, w.r, true); }
};

__global__ void fused_bump_epoch(char* const* peers, int rank, size_t comm_off, int world) {
  *reinterpret_cast<long long*>(peers[rank] + comm_off + 72 * world) += 1;
}

}  // namespace
}  // namespace tsb

#define PEER_ARGS void* const* peers, int world, int rank, size_t comm_off, const long long* sends, int n_sends
#define PEER_CTX PeerCtx{reinterpret_cast<char* const*>(peers), world, rank, comm_off, 2ll * max_iter + 4, sends, n_sends, b}

extern "C" int trnsparse_bsr_cg_fused_start(int64_t n_own, int64_t n_ext, int b, const float* b_vec,
                                            const float* inv_d, int max_iter, void* ws, size_t ws_bytes, PEER_ARGS,
                                            void* stream) {
  TSB_REQUIRE(n_own >= 0 && n_ext >= n_own && max_iter >= 0 && b_vec && ws && peers && world > 0 && rank >= 0 &&
                  rank < world && (n_sends == 0 || sends),
              "bsr_cg_fused_start: bad argument");
  TSB_REQUIRE(ws_bytes >= cg_ws_size(n_ext, max_iter), "bsr_cg_fused_start: workspace too small");
  cudaStream_t st = as_stream(stream);
  cudaError_t e = clear_cg_ws(ws, n_ext, max_iter, st);
  if (e != cudaSuccess) return cuda_status(e, "bsr_cg_fused_start: memset");
  fused_bump_epoch<<<1, 1, 0, st>>>(reinterpret_cast<char* const*>(peers), rank, comm_off, world);
  TSB_CHECK_LAUNCH("bsr_cg_fused_start: epoch");
  return launch_vec(n_own, CgStartFused{b_vec, inv_d, cg_ws(ws, n_ext, max_iter), PEER_CTX}, st,
                    "bsr_cg_fused_start");
}

extern "C" int trnsparse_bsr_cg_fused_phase(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                                            const int* col_idx, const float* blocks, float* x, const float* inv_d,
                                            double tol, int max_iter, int k, int phase, void* ws, PEER_ARGS,
                                            void* stream) {
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_cg_fused_phase");
  if (rc) return rc;
  TSB_REQUIRE(ws && x && k >= 0 && k <= max_iter && (phase == 0 || phase == 1) && peers && world > 0,
              "bsr_cg_fused_phase: bad argument");
  TSB_REQUIRE(d.fast(), "bsr_cg_fused_phase: needs block size 128 and block-aligned shapes");
  cudaStream_t st = as_stream(stream);
  const CgWs w = cg_ws(ws, n, max_iter);
  float* pcur = (k & 1) ? w.p1 : w.p0;
  const float* pprev = (k & 1) ? w.p0 : w.p1;
  if (phase == 0) {
    CgMvFused mv{inv_d, w, pprev, pcur, k, max_iter, tol, m, PEER_CTX, 0.f};
    // persistent CTAs: every CTA pays the peer-flag wait of its prologue once
    return launch_bsr_mv(d, mv, all_aligned({inv_d, w.r, w.p0, w.p1}), st, "bsr_cg_fused mv", 3 * sm_count());
  }
  if (k >= max_iter) return TRNSPARSE_OK;
  return launch_vec(m, CgUpdateFused{inv_d, x, w, pcur, k, max_iter, PEER_CTX, 0.f}, st, "bsr_cg_fused update",
                    sm_count());
}

// ---------------------------------------------------------------- sharded CG, one kernel per iteration
// The two fused kernels of an iteration merged into one cooperative launch
// (all CTAs co-resident): prologue waits for the previous iteration's
// r.r / r.z and halo, SpMV with p on the fly, last CTA publishes p.Ap, every
// CTA waits for the global p.Ap, updates x and r on the rows it computed and
// the last CTA publishes r.r / r.z and the halo rows of r.
namespace tsb {
namespace {

__global__ void __launch_bounds__(256)
cg_iter_coop_kernel(const int* __restrict__ row_ptr, const int* __restrict__ col_idx,
                    const float4* __restrict__ blocks, int n_block_rows, CgMvFused mv, CgUpdateFused up) {
  __shared__ float ys[128];
  __shared__ double red[8];
  if (!mv.begin(blockIdx.x)) return;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  double d0 = 0.0, d1 = 0.0;
  for (int i = blockIdx.x; i < n_block_rows; i += gridDim.x) {
    float acc[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) acc[r] = 0.f;
    const int e = row_ptr[i + 1];
    for (int idx = row_ptr[i]; idx < e; ++idx) {
      const int64_t j = col_idx[idx];
      const float4 xv = mv.x4(j * 128 + 4 * lane);
      const float4* bp = blocks + static_cast<int64_t>(idx) * 4096 + (w * 16) * 32 + lane;
      float4 a[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) a[r] = __ldcs(bp + r * 32);
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        acc[r] = fmaf(a[r].x, xv.x, acc[r]);
        acc[r] = fmaf(a[r].y, xv.y, acc[r]);
        acc[r] = fmaf(a[r].z, xv.z, acc[r]);
        acc[r] = fmaf(a[r].w, xv.w, acc[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const float v = warp_sum(acc[r]);
      if (lane == r) ys[w * 16 + r] = v;
    }
    __syncthreads();
    if (threadIdx.x < 128) mv.row(static_cast<int64_t>(i) * 128 + threadIdx.x, ys[threadIdx.x], &d0, &d1);
    __syncthreads();
  }
  {
    const double t0 = block_sum256(d0, red);
    if (threadIdx.x == 0) mv.finish(t0, 0.0);
  }
  mv.tail();
  if (mv.k >= mv.max_iter) return;
  if (!up.begin(blockIdx.x)) return;
  double e0 = 0.0, e1 = 0.0;
  for (int i = blockIdx.x; i < n_block_rows; i += gridDim.x)
    if (threadIdx.x < 128) up.elem(static_cast<int64_t>(i) * 128 + threadIdx.x, &e0, &e1);
  const double t0 = block_sum256(e0, red);
  const double t1 = block_sum256(e1, red);
  if (threadIdx.x == 0) up.finish(t0, t1);
  up.tail();
}

}  // namespace
}  // namespace tsb

extern "C" int trnsparse_bsr_cg_coop_iter(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                                          const int* col_idx, const float* blocks, float* x, const float* inv_d,
                                          double tol, int max_iter, int k, void* ws, PEER_ARGS, void* stream) {
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_cg_coop_iter");
  if (rc) return rc;
  TSB_REQUIRE(ws && x && k >= 0 && k <= max_iter && peers && world > 0, "bsr_cg_coop_iter: bad argument");
  TSB_REQUIRE(d.fast(), "bsr_cg_coop_iter: needs block size 128 and block-aligned shapes");
  cudaStream_t st = as_stream(stream);
  const CgWs w = cg_ws(ws, n, max_iter);
  TSB_REQUIRE(all_aligned({inv_d, w.r, w.p0, w.p1, x}), "bsr_cg_coop_iter: vectors must be 16-byte aligned");
  float* pcur = (k & 1) ? w.p1 : w.p0;
  const float* pprev = (k & 1) ? w.p0 : w.p1;
  CgMvFused mv{inv_d, w, pprev, pcur, k, max_iter, tol, m, PEER_CTX, 0.f};
  CgUpdateFused up{inv_d, x, w, pcur, k, max_iter, PEER_CTX, 0.f};
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, cg_iter_coop_kernel, 256, 0);
  if (e != cudaSuccess) return cuda_status(e, "bsr_cg_coop_iter: occupancy");
  int64_t nbr = d.block_rows();
  int64_t grid = static_cast<int64_t>(sm_count()) * (per_sm < 1 ? 1 : per_sm);
  if (grid > nbr) grid = nbr;
  if (grid < 1) grid = 1;
  const float4* bl = reinterpret_cast<const float4*>(blocks);
  int nbr_i = (int)nbr;
  void* args[] = {(void*)&row_ptr, (void*)&col_idx, (void*)&bl, (void*)&nbr_i, (void*)&mv, (void*)&up};
  e = cudaLaunchCooperativeKernel((const void*)cg_iter_coop_kernel, dim3((unsigned)grid), dim3(256), args, 0, st);
  if (e != cudaSuccess) return cuda_status(e, "bsr_cg_coop_iter: cooperative launch");
  return TRNSPARSE_OK;
}
