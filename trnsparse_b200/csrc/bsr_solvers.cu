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

enum {
  REASON_NONE = 0,
  REASON_CONVERGED = 1,
  REASON_MAXITER = 2,
  REASON_BREAKDOWN = 3,
  REASON_ZERO_RHS = 4,
  REASON_PEER_TIMEOUT = 5,  // a sharded solve's exchange with a peer timed out
};

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
  CGT_ENTER
  if (!op.begin(blockIdx.x)) return;
  CGT(1);
  double d0 = 0.0, d1 = 0.0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < n; i += static_cast<int64_t>(gridDim.x) * 256)
    op.elem(i, &d0, &d1);
  const double t0 = block_sum256(d0, red);
  const double t1 = block_sum256(d1, red);
  if (threadIdx.x == 0) op.finish(t0, t1);
  CGT(2);
  run_tail(op);
  CGT(3);
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

// ---------------------------------------------------------------- row-shard steps
// One step of the fixed-step solvers / power iteration on a block-row shard
// (m own rows, n = own + halo columns); the caller refreshes the halo and
// reduces the partial sums across ranks between steps.
struct PowStepMv {
  static constexpr int kDots = 2;
  const float* vin;
  float* wout;
  double* dots;  // [0] += v.w, [1] += w.w over the own rows
  __device__ bool begin(int) const { return true; }
  __device__ float x(int64_t c) const { return vin[c]; }
  __device__ float4 x4(int64_t c) const { return ld4(vin + c); }
  __device__ void row(int64_t i, float y, double* d0, double* d1) const {
    wout[i] = y;
    *d0 += (double)vin[i] * (double)y;
    *d1 += (double)y * (double)y;
  }
  __device__ void finish(double t0, double t1) const {
    atomicAdd(&dots[0], t0);
    atomicAdd(&dots[1], t1);
  }
};

struct DivNorm {
  const float* x;
  const double* ss;
  float* y;
  mutable float nrm;
  __device__ bool begin(int) const {
    nrm = (float)sqrt(*ss);
    return true;
  }
  __device__ void elem(int64_t i, double*, double*) const { y[i] = __fdiv_rn(x[i], nrm); }
  __device__ void finish(double, double) const {}
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

extern "C" int trnsparse_bsr_chebyshev_step(BSR_DESC_ARGS, const float* b_vec, const float* xk, const float* xprev,
                                            float* xnext, double a, double bcoef, int momentum, void* stream) {
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_chebyshev_step");
  if (rc) return rc;
  TSB_REQUIRE(b_vec && xk && xnext && (!momentum || xprev), "bsr_chebyshev_step: null pointer");
  if (m == 0) return TRNSPARSE_OK;
  ChebMv op{b_vec, xk, xprev, xnext, (float)a, (float)bcoef, momentum != 0};
  return launch_bsr_mv(d, op, all_aligned({xk}), as_stream(stream), "bsr_chebyshev_step");
}

extern "C" int trnsparse_bsr_residual_sq(BSR_DESC_ARGS, const float* b_vec, const float* x, double* acc,
                                         void* stream) {
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_residual_sq");
  if (rc) return rc;
  TSB_REQUIRE(b_vec && x && acc, "bsr_residual_sq: null pointer");
  if (m == 0) return TRNSPARSE_OK;
  return launch_bsr_mv(d, ResidualMv{b_vec, x, acc}, all_aligned({x}), as_stream(stream), "bsr_residual_sq");
}

extern "C" int trnsparse_bsr_power_step(BSR_DESC_ARGS, const float* v, float* w, double* dots, void* stream) {
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_power_step");
  if (rc) return rc;
  TSB_REQUIRE(v && w && dots, "bsr_power_step: null pointer");
  if (m == 0) return TRNSPARSE_OK;
  return launch_bsr_mv(d, PowStepMv{v, w, dots}, all_aligned({v}), as_stream(stream), "bsr_power_step");
}

extern "C" int trnsparse_vec_div_norm(int64_t n, const float* x, const double* ss, float* y, void* stream) {
  TSB_REQUIRE(n >= 0 && (n == 0 || (x && ss && y)), "vec_div_norm: bad argument");
  if (n == 0) return TRNSPARSE_OK;
  return launch_vec(n, DivNorm{x, ss, y, 0.f}, as_stream(stream), "vec_div_norm");
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
  long long seq0;  // epoch * stride once known (a one-launch solve reads the epoch once), else -1
};

__device__ __forceinline__ long long* pc_flags(const PeerCtx& p, char* base) {
  return reinterpret_cast<long long*>(base + p.comm_off);
}
__device__ __forceinline__ double* pc_vals(const PeerCtx& p, char* base) {
  return reinterpret_cast<double*>(base + p.comm_off + 24 * p.world);
}
__device__ __forceinline__ long long* pc_epoch(const PeerCtx& p, char* base) {
  return reinterpret_cast<long long*>(base + p.comm_off + 120 * p.world);
}
__device__ __forceinline__ unsigned int* pc_ticket(const PeerCtx& p, int which) {
  return reinterpret_cast<unsigned int*>(p.peers[p.rank] + p.comm_off + 120 * p.world + 8) + which;
}
__device__ __forceinline__ long long pc_seq_base(const PeerCtx& p) {
  return (*reinterpret_cast<volatile long long*>(pc_epoch(p, p.peers[p.rank]))) * p.stride;
}
__device__ __forceinline__ long long pc_seq(const PeerCtx& p, long long step) {
  return (p.seq0 >= 0 ? p.seq0 : pc_seq_base(p)) + step + 1;
}

__device__ __forceinline__ void st_rel_sys(long long* q, long long v) {
  asm volatile("st.release.sys.global.s64 [%0], %1;\n" ::"l"(q), "l"(v) : "memory");
}

// All threads of the CTA: wait for every rank's flag of `area` to reach the
// step's sequence number, then return the rank-ordered sums of its partials.
__device__ __forceinline__ bool peer_failed() { return *(volatile int*)&g_device_error == DEVERR_PEER_TIMEOUT; }

// A wait that timed out (or follows one: the error word is sticky) yields NaN
// totals; the callers see peer_failed() and end the solve as failed.
__device__ double2 pc_wait_sum(const PeerCtx& p, int area, long long step) {
  __shared__ double2 tot;
  __shared__ int fail;
  char* mine = p.peers[p.rank];
  const long long seq = pc_seq(p, step);
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (threadIdx.x < p.world) {
    const bool ok = *(volatile int*)&g_device_error != DEVERR_PEER_TIMEOUT &&
                    wait_flag_geq(pc_flags(p, mine) + area * p.world + threadIdx.x, seq, 32);
    if (!ok) fail = 1;
  }
  __syncthreads();
  if (fail) return make_double2(nan(""), nan(""));
  if (threadIdx.x == 0) {
    const volatile double* v = pc_vals(p, mine) + area * p.world * 4;
    double a = 0.0, b = 0.0;
    for (int q = 0; q < p.world; ++q) {
      a += v[4 * q];
      b += v[4 * q + 1];
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
    // acq_rel: releases this CTA's stores (ordered before by the barrier); the last CTA
    // acquires every other CTA's
    unsigned t;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;\n" : "=r"(t) : "l"(pc_ticket(p, which)) : "memory");
    last = ((t + 1) % gridDim.x) == 0;
    if (last) part = make_double2(a ? *(volatile const double*)a : 0.0, b ? *(volatile const double*)b : 0.0);
  }
  __syncthreads();
  if (!last) return;
#ifdef TSB_CG_TRACE
  if (threadIdx.x == 0) g_cg_trace[(g_cg_trace_n - 1) & 511u][4] = cgt_now();
#endif
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
    double* v = pc_vals(p, p.peers[threadIdx.x]) + (area * p.world + p.rank) * 4;
    v[0] = part.x;
    v[1] = part.y;
  }
  // the halo and partial stores above happen-before (barrier) the flag's release at system scope
  __syncthreads();
  if (threadIdx.x < p.world) st_rel_sys(pc_flags(p, p.peers[threadIdx.x]) + area * p.world + p.rank, seq);
#ifdef TSB_CG_TRACE
  if (threadIdx.x == 0) g_cg_trace[(g_cg_trace_n - 1) & 511u][5] = cgt_now();
#endif
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
    if (peer_failed()) {
      if (cta == 0 && threadIdx.x == 0) set_done(st, k, REASON_PEER_TIMEOUT, nan(""));
      return false;
    }
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
    if (peer_failed()) {
      if (cta == 0 && threadIdx.x == 0) set_done(st, k, REASON_PEER_TIMEOUT, nan(""));
      return false;
    }
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
  *reinterpret_cast<long long*>(peers[rank] + comm_off + 120 * world) += 1;
}

}  // namespace
}  // namespace tsb

#define PEER_ARGS void* const* peers, int world, int rank, size_t comm_off, const long long* sends, int n_sends
#define PEER_CTX PeerCtx{reinterpret_cast<char* const*>(peers), world, rank, comm_off, 2ll * max_iter + 4, sends, n_sends, b, -1}

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
    return launch_bsr_mv(d, mv, all_aligned({inv_d, w.r, w.p0, w.p1}), st, "bsr_cg_fused mv", 3 * sm_count(),
                         fits_l2(static_cast<size_t>(n_blocks) * 128 * 128 * 4));
  }
  if (k >= max_iter) return TRNSPARSE_OK;
  return launch_vec(m, CgUpdateFused{inv_d, x, w, pcur, k, max_iter, PEER_CTX, 0.f}, st, "bsr_cg_fused update",
                    sm_count());
}

// ---------------------------------------------------------------- sharded CG, one kernel per solve
// The two fused kernels of every iteration merged into one cooperative
// launch (all CTAs co-resident) that loops over the iterations: each
// iteration's prologue waits for the previous r.r / r.z and halo, the SpMV
// computes p on the fly, the last CTA publishes p.Ap, every CTA waits for the
// global p.Ap, updates x and r on its block-rows, and the last CTA publishes
// r.r / r.z and the halo rows of r. The peer flags double as the grid-wide
// barrier between the phases (each rank's own flag is raised by its last CTA
// only after every CTA has taken its ticket), so no launch boundary remains.
namespace tsb {
namespace {

template <bool KEEP>
__global__ void __launch_bounds__(256, 2)  // two CTAs per SM: every block-row in flight at once
cg_solve_coop_kernel(const int* __restrict__ row_ptr, const int* __restrict__ col_idx,
                     const float4* __restrict__ blocks, int n_block_rows, CgMvFused mv, CgUpdateFused up,
                     float* p0, float* p1, int k_begin, int k_end) {
  __shared__ float ys[128];
  __shared__ double red[8];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  mv.p.seq0 = up.p.seq0 = pc_seq_base(mv.p);  // the epoch is fixed for the whole solve
#ifdef TSB_CG_TRACE
  __shared__ unsigned cgt_slot;
#endif
  for (int k = k_begin; k <= k_end; ++k) {
#ifdef TSB_CG_TRACE
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      cgt_slot = atomicAdd(&g_cg_trace_n, 1u) & 511u;
      g_cg_trace[cgt_slot][0] = cgt_now();
    }
#endif
    mv.k = up.k = k;
    mv.pcur = (k & 1) ? p1 : p0;
    up.pcur = mv.pcur;
    mv.pprev = (k & 1) ? p0 : p1;
    mv.beta = up.alpha = 0.f;
    if (!mv.begin(blockIdx.x)) return;
    CGT(1);
    double d0 = 0.0;
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
        for (int r = 0; r < 16; ++r) a[r] = KEEP ? __ldg(bp + r * 32) : __ldcs(bp + r * 32);
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
      double dd = 0.0;
      if (threadIdx.x < 128) mv.row(static_cast<int64_t>(i) * 128 + threadIdx.x, ys[threadIdx.x], &d0, &dd);
      __syncthreads();
    }
    CGT(2);
    {
      const double t0 = block_sum256(d0, red);
      if (threadIdx.x == 0) mv.finish(t0, 0.0);
    }
    mv.tail();
    CGT(3);
    if (k >= mv.max_iter) return;
    if (!up.begin(blockIdx.x)) return;
    CGT(6);
    double e0 = 0.0, e1 = 0.0;
    for (int i = blockIdx.x; i < n_block_rows; i += gridDim.x)
      if (threadIdx.x < 128) up.elem(static_cast<int64_t>(i) * 128 + threadIdx.x, &e0, &e1);
    const double t0 = block_sum256(e0, red);
    const double t1 = block_sum256(e1, red);
    if (threadIdx.x == 0) up.finish(t0, t1);
    up.tail();
    CGT(7);
  }
}

}  // namespace
}  // namespace tsb

extern "C" int trnsparse_bsr_cg_coop_run(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                                         const int* col_idx, const float* blocks, float* x, const float* inv_d,
                                         double tol, int max_iter, int k_begin, int k_end, void* ws, PEER_ARGS,
                                         void* stream) {
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_cg_coop_run");
  if (rc) return rc;
  TSB_REQUIRE(ws && x && 0 <= k_begin && k_begin <= k_end && k_end <= max_iter && peers && world > 0,
              "bsr_cg_coop_run: bad argument");
  TSB_REQUIRE(d.fast(), "bsr_cg_coop_run: needs block size 128 and block-aligned shapes");
  cudaStream_t st = as_stream(stream);
  const CgWs w = cg_ws(ws, n, max_iter);
  TSB_REQUIRE(all_aligned({inv_d, w.r, w.p0, w.p1, x}), "bsr_cg_coop_run: vectors must be 16-byte aligned");
  CgMvFused mv{inv_d, w, w.p1, w.p0, k_begin, max_iter, tol, m, PEER_CTX, 0.f};
  CgUpdateFused up{inv_d, x, w, w.p0, k_begin, max_iter, PEER_CTX, 0.f};
  const bool keep = fits_l2(static_cast<size_t>(n_blocks) * 128 * 128 * 4);
  const void* kern = keep ? (const void*)cg_solve_coop_kernel<true> : (const void*)cg_solve_coop_kernel<false>;
  int per_sm = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0);
  if (e != cudaSuccess) return cuda_status(e, "bsr_cg_coop_run: occupancy");
  int64_t nbr = d.block_rows();
  int64_t grid = static_cast<int64_t>(sm_count()) * (per_sm < 1 ? 1 : per_sm);
  if (grid > nbr) grid = nbr;
  if (grid < 1) grid = 1;
  const float4* bl = reinterpret_cast<const float4*>(blocks);
  int nbr_i = (int)nbr;
  float* p0 = w.p0;
  float* p1 = w.p1;
  void* args[] = {(void*)&row_ptr, (void*)&col_idx, (void*)&bl, (void*)&nbr_i, (void*)&mv,
                  (void*)&up,      (void*)&p0,      (void*)&p1, (void*)&k_begin, (void*)&k_end};
  e = cudaLaunchCooperativeKernel(kern, dim3((unsigned)grid), dim3(256), args, 0, st);
  if (e != cudaSuccess) return cuda_status(e, "bsr_cg_coop_run: cooperative launch");
  return TRNSPARSE_OK;
}

// ---------------------------------------------------------------- sharded CG, one reduction per iteration
// Chronopoulos & Gear's formulation of preconditioned CG ("s-step methods
// and their parallel implementation", J. Comput. Appl. Math. 25, 1989): with
// u = M r and w = A u carried along, the iteration's two inner-product rounds
// of standard PCG become one, since p.Ap = delta - beta * gamma / alpha_prev
// with gamma = r.u and delta = w.u; s = A p follows the recurrence
// s = w + beta s. Per iteration k (gamma_k, delta_k, r_k.r_k known):
//   beta = gamma_k / gamma_{k-1};  p.Ap = delta_k - beta gamma_k / alpha_{k-1}
//   alpha = gamma_k / p.Ap
//   p = u + beta p;  s = w + beta s;  x += alpha p;  r -= alpha s
//   u = M r;  w = A u;  then gamma_{k+1}, delta_{k+1}, r.r in one reduction.
// In exact arithmetic these are the reference's iterates (trnsparse/
// iterative.py:53-126); the convergence test (||r|| / ||b|| after the update)
// and the |p.Ap| < 1e-30 breakdown test sit where the reference has them.
//
// One cooperative launch runs the whole solve. The SpMV input u = M r of a
// column is formed on the fly from the previous iteration's r, s and w (so
// own and halo columns need no extra pass), the owner CTA of a row writes the
// new r, s, p, x, w of that row, and the halo copies of r and s are written by
// the CTAs that form them. r, s and w are double-buffered by iteration
// parity. The exchange after the SpMV carries three partial sums and the new
// w rows the neighbours hold as halo; every rank's buffers have the same
// layout (n_alloc entries per vector), so halo destinations are element
// offsets. The peer flags double as the grid-wide barrier.
namespace tsb {
namespace {

struct CgcgWs {
  SolverStatus* st;
  Slot* slots;  // slot k: {a: p_k.Ap_k, b: gamma_k, c: delta_k, d: r_k.r_k}
  float* r[2];
  float* s[2];
  float* w[2];
  float* p;
};
constexpr int kCgcgVecs = 7;

inline size_t cgcg_head(int max_iter) { return align256(64) + align256(sizeof(Slot) * (size_t)(max_iter + 2)); }
inline size_t cgcg_ws_size(int64_t n, int max_iter) {
  return cgcg_head(max_iter) + kCgcgVecs * align256(sizeof(float) * (size_t)n);
}
inline CgcgWs cgcg_ws(void* base, int64_t n, int max_iter) {
  char* p = static_cast<char*>(base);
  CgcgWs w;
  w.st = reinterpret_cast<SolverStatus*>(p);
  w.slots = reinterpret_cast<Slot*>(p + align256(64));
  char* v = p + cgcg_head(max_iter);
  const size_t vb = align256(sizeof(float) * (size_t)n);
  for (int i = 0; i < 2; ++i) {
    w.r[i] = reinterpret_cast<float*>(v + (0 + i) * vb);
    w.s[i] = reinterpret_cast<float*>(v + (2 + i) * vb);
    w.w[i] = reinterpret_cast<float*>(v + (4 + i) * vb);
  }
  w.p = reinterpret_cast<float*>(v + 6 * vb);
  return w;
}

struct Cgcg {
  const int* row_ptr;
  const int* col_idx;
  const float4* blocks;
  int n_block_rows;
  int64_t n_own;
  const float* inv_d;  // n_alloc, halo filled; null = no preconditioner
  const float* bvec;   // n_own
  float* x;            // n_own
  CgcgWs ws;
  size_t ws_off;       // byte offset of the workspace inside every rank's peer buffer
  size_t vec_bytes;
  size_t head;
  double tol;
  int max_iter;
  PeerCtx p;           // sends: (source element, destination rank, destination element)
};

__device__ __forceinline__ float cg_m(const float* inv_d, int64_t c, float r) {
  return inv_d ? __fmul_rn(r, inv_d[c]) : r;
}

// Wait (bounded) until every rank's flag of `area` reached `seq`; return the
// rank-ordered sums of the first three partials.
// A timed-out wait yields NaN totals (the caller ends the solve).
__device__ double3 cgcg_wait(const PeerCtx& p, int area, long long seq) {
  __shared__ double3 tot;
  __shared__ int fail;
  char* mine = p.peers[p.rank];
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (threadIdx.x < p.world) {
    const bool ok = *(volatile int*)&g_device_error != DEVERR_PEER_TIMEOUT &&
                    wait_flag_geq(pc_flags(p, mine) + area * p.world + threadIdx.x, seq, 20);
    if (!ok) fail = 1;
  }
  __syncthreads();
  if (fail) return make_double3(nan(""), nan(""), nan(""));
  if (threadIdx.x == 0) {
    const volatile double* v = pc_vals(p, mine) + area * p.world * 4;
    double a = 0.0, b = 0.0, c = 0.0;
    for (int q = 0; q < p.world; ++q) {
      a += v[4 * q];
      b += v[4 * q + 1];
      c += v[4 * q + 2];
    }
    tot = make_double3(a, b, c);
  }
  __syncthreads();
  return tot;
}

// Last CTA (ticket counter `which`; one counter per kernel, whose grid size is
// fixed) publishes the three local totals of `slot` and, when
// `src` is set, the halo rows of that vector (at byte offset `vec_off` of the
// workspace) to every rank, then raises the flags.
__device__ void cgcg_publish(const Cgcg& g, int which, int area, long long seq, const Slot* slot, const float* src,
                             size_t vec_off) {
  __shared__ int last;
  __shared__ double3 part;
  const PeerCtx& p = g.p;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned t;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;\n" : "=r"(t) : "l"(pc_ticket(p, which)) : "memory");
    last = ((t + 1) % gridDim.x) == 0;
    if (last) {
      const volatile double* v = &slot->b;
      part = make_double3(v[0], v[1], v[2]);
    }
  }
  __syncthreads();
  if (!last) return;
#ifdef TSB_CG_TRACE
  if (threadIdx.x == 0) g_cg_trace[(g_cg_trace_n - 1) & 511u][4] = cgt_now();
#endif
  if (src) {
    for (int q = 0; q < p.n_sends; ++q) {
      const long long so = p.sends[3 * q], dr = p.sends[3 * q + 1], de = p.sends[3 * q + 2];
      float4* dst = reinterpret_cast<float4*>(p.peers[dr] + g.ws_off + vec_off + 4 * de);
      const volatile float4* sp = reinterpret_cast<const volatile float4*>(src + so);
      for (int i = threadIdx.x; i < p.chunk / 4; i += blockDim.x) dst[i] = make_float4(sp[i].x, sp[i].y, sp[i].z, sp[i].w);
    }
  }
  if (threadIdx.x < p.world) {
    double* v = pc_vals(p, p.peers[threadIdx.x]) + (area * p.world + p.rank) * 4;
    v[0] = part.x;
    v[1] = part.y;
    v[2] = part.z;
  }
  __syncthreads();  // the stores above happen-before each flag's release at system scope
  if (threadIdx.x < p.world) st_rel_sys(pc_flags(p, p.peers[threadIdx.x]) + area * p.world + p.rank, seq);
#ifdef TSB_CG_TRACE
  if (threadIdx.x == 0) g_cg_trace[(g_cg_trace_n - 1) & 511u][5] = cgt_now();
#endif
}

// Inputs of four consecutive columns of the on-the-fly SpMV operand.
struct Col4 {
  float4 w, s, r, d;
};

// SpMV of one block-row; the input of four consecutive columns (per lane) is
// fetched by `fetch(c)` and formed by `make(c, fetched)`. Per block the
// input's loads go out first, then the block's, then the input is formed
// (its halo stores may alias the blocks as far as the compiler knows, so they
// come after every load); the next column index is fetched ahead. Returns
// the row sums in ys[0..127].
template <bool KEEP, class Fetch, class Make>
__device__ __forceinline__ void cgcg_row_mv(const Cgcg& g, int i, float* ys, Fetch fetch, Make make) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float acc[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) acc[r] = 0.f;
  const int e = g.row_ptr[i + 1];
  int idx = g.row_ptr[i];
  int64_t j = idx < e ? g.col_idx[idx] : 0;
  for (; idx < e; ++idx) {
    const int64_t jn = idx + 1 < e ? g.col_idx[idx + 1] : 0;
    const int64_t c = j * 128 + 4 * lane;
    const Col4 in = fetch(c);
    const float4* bp = g.blocks + static_cast<int64_t>(idx) * 4096 + (w * 16) * 32 + lane;
    float4 a[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) a[r] = KEEP ? __ldg(bp + r * 32) : __ldcs(bp + r * 32);
    const float4 xv = make(c, in);
    j = jn;
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
}

// Block sum of three doubles; thread 0 adds them into slot->{b, c, d}.
__device__ __forceinline__ void cgcg_add3(double a, double b, double c, double* red, Slot* slot) {
  a = block_sum256(a, red);
  b = block_sum256(b, red);
  c = block_sum256(c, red);
  if (threadIdx.x == 0) {
    atomicAdd(&slot->b, a);
    atomicAdd(&slot->c, b);
    atomicAdd(&slot->d, c);
  }
}

// exchange steps: 0 = setup (r0 halo, ||b||^2), 1 + k = (gamma, delta, r.r)_k and w_k halo
template <bool KEEP>
__global__ void __launch_bounds__(256, 2)
cgcg_solve_kernel(Cgcg g) {
  __shared__ float ys[128];
  __shared__ double red[8];
  SolverStatus* st = g.ws.st;
  const long long seq0 = pc_seq_base(g.p);  // the epoch is fixed for the whole solve
  const int64_t halo_begin = g.n_own;
  const size_t w_off0 = g.head + 4 * g.vec_bytes, w_off1 = g.head + 5 * g.vec_bytes;

  // ---- setup part 2: ||b||^2 and the r0 halo have arrived; w0 = A u0 with u0 = M r0
  const double bb = cgcg_wait(g.p, 2, seq0 + 1).x;
  if (peer_failed()) {
    if (blockIdx.x == 0 && threadIdx.x == 0) set_done(st, 0, REASON_PEER_TIMEOUT, nan(""));
    return;
  }
  if (bb < 1e-30) {  // ||b|| < 1e-15: x = 0 (reference: zero right-hand side)
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      st->bb = bb;
      set_done(st, 0, REASON_ZERO_RHS, 0.0);
    }
    return;
  }
  {
    const float* r0 = g.ws.r[0];
    double ga = 0.0, de = 0.0, rr = 0.0;
    for (int i = blockIdx.x; i < g.n_block_rows; i += gridDim.x) {
      cgcg_row_mv<KEEP>(
          g, i, ys,
          [&](int64_t c) {
            Col4 v;
            v.r = ld4(r0 + c);
            v.d = g.inv_d ? ld4(g.inv_d + c) : make_float4(1.f, 1.f, 1.f, 1.f);
            return v;
          },
          [&](int64_t, const Col4& v) {
            return g.inv_d ? make_float4(__fmul_rn(v.r.x, v.d.x), __fmul_rn(v.r.y, v.d.y), __fmul_rn(v.r.z, v.d.z),
                                         __fmul_rn(v.r.w, v.d.w))
                           : v.r;
          });
      if (threadIdx.x < 128) {
        const int64_t row = static_cast<int64_t>(i) * 128 + threadIdx.x;
        const float r = r0[row], u = cg_m(g.inv_d, row, r), wv = ys[threadIdx.x];
        g.ws.w[0][row] = wv;
        ga += (double)r * (double)u;
        de += (double)wv * (double)u;
        rr += (double)r * (double)r;
      }
      __syncthreads();
    }
    cgcg_add3(ga, de, rr, red, &g.ws.slots[0]);
    cgcg_publish(g, 3, 0, seq0 + 2, &g.ws.slots[0], g.ws.w[0], w_off0);
  }
  double gam_prev = 0.0, alpha_prev = 0.0;
#ifdef TSB_CG_TRACE
  __shared__ unsigned cgt_slot;
#endif
  for (int k = 0;; ++k) {
    const int cur = k & 1, nxt = cur ^ 1;
#ifdef TSB_CG_TRACE
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      cgt_slot = atomicAdd(&g_cg_trace_n, 1u) & 511u;
      g_cg_trace[cgt_slot][0] = cgt_now();
    }
#endif
    const double3 t = cgcg_wait(g.p, k & 1, seq0 + 2 + k);
    CGT(1);
    if (peer_failed()) {
      if (blockIdx.x == 0 && threadIdx.x == 0) set_done(st, k, REASON_PEER_TIMEOUT, nan(""));
      return;
    }
#ifdef TSB_CG_TRACE
    if (k == 10 && threadIdx.x == 0 && blockIdx.x < 512) g_cg_cta[blockIdx.x][2] = cgt_now();
#endif
    const double gam = t.x, del = t.y, rr = t.z;
    if (k > 0) {
      const double rel = (double)(float)sqrt(rr) / sqrt(bb);
      if (rel < g.tol) {
        if (blockIdx.x == 0 && threadIdx.x == 0) set_done(st, k, REASON_CONVERGED, rel);
        return;
      }
    }
    if (k >= g.max_iter) {
      if (blockIdx.x == 0 && threadIdx.x == 0)
        set_done(st, g.max_iter, REASON_MAXITER, k > 0 ? (double)(float)sqrt(rr) / sqrt(bb) : nan(""));
      return;
    }
    const double beta_d = k > 0 ? gam / gam_prev : 0.0;
    const double pap = k > 0 ? del - beta_d * gam / alpha_prev : del;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      if (k == 0) st->bb = bb;
      g.ws.slots[k].a = pap;
    }
    if (fabs(pap) < 1e-30) {
      if (blockIdx.x == 0 && threadIdx.x == 0)
        set_done(st, g.max_iter, REASON_BREAKDOWN, k > 0 ? (double)(float)sqrt(rr) / sqrt(bb) : nan(""));
      return;
    }
    const double alpha_d = gam / pap;
    const float alpha = (float)alpha_d, beta = (float)beta_d;
    gam_prev = gam;
    alpha_prev = alpha_d;
    const float *rc = g.ws.r[cur], *sc = g.ws.s[cur], *wc = g.ws.w[cur];
    float *rn = g.ws.r[nxt], *sn = g.ws.s[nxt], *wn = g.ws.w[nxt];
    // s_k = w_k + beta s_{k-1};  r_{k+1} = r_k - alpha s_k;  u_{k+1} = M r_{k+1}
    auto form = [&](int64_t c, float* r_out, float* s_out) {
      const float s = __fadd_rn(wc[c], __fmul_rn(beta, sc[c]));
      const float r = __fsub_rn(rc[c], __fmul_rn(alpha, s));
      *s_out = s;
      *r_out = r;
      return cg_m(g.inv_d, c, r);
    };
    double ga = 0.0, de = 0.0, rr_new = 0.0;
    for (int i = blockIdx.x; i < g.n_block_rows; i += gridDim.x) {
      cgcg_row_mv<KEEP>(
          g, i, ys,
          [&](int64_t c) {
            Col4 v;
            v.w = ld4(wc + c);
            v.s = ld4(sc + c);
            v.r = ld4(rc + c);
            v.d = g.inv_d ? ld4(g.inv_d + c) : make_float4(1.f, 1.f, 1.f, 1.f);
            return v;
          },
          [&](int64_t c, const Col4& v) {
            const float wv[4] = {v.w.x, v.w.y, v.w.z, v.w.w}, sv[4] = {v.s.x, v.s.y, v.s.z, v.s.w};
            const float rv[4] = {v.r.x, v.r.y, v.r.z, v.r.w}, dv[4] = {v.d.x, v.d.y, v.d.z, v.d.w};
            float r[4], s[4], u[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              s[q] = __fadd_rn(wv[q], __fmul_rn(beta, sv[q]));
              r[q] = __fsub_rn(rv[q], __fmul_rn(alpha, s[q]));
              u[q] = g.inv_d ? __fmul_rn(r[q], dv[q]) : r[q];
            }
            if (c >= halo_begin) {  // halo copies: every CTA that needs them writes the same values
              *reinterpret_cast<float4*>(rn + c) = make_float4(r[0], r[1], r[2], r[3]);
              *reinterpret_cast<float4*>(sn + c) = make_float4(s[0], s[1], s[2], s[3]);
            }
            return make_float4(u[0], u[1], u[2], u[3]);
          });
      if (threadIdx.x < 128) {
        const int64_t row = static_cast<int64_t>(i) * 128 + threadIdx.x;
        float r, s;
        const float u = form(row, &r, &s);
        rn[row] = r;
        sn[row] = s;
        const float pk = __fadd_rn(cg_m(g.inv_d, row, rc[row]), __fmul_rn(beta, g.ws.p[row]));
        g.ws.p[row] = pk;
        g.x[row] = __fadd_rn(g.x[row], __fmul_rn(alpha, pk));
        const float wv = ys[threadIdx.x];
        wn[row] = wv;
        ga += (double)r * (double)u;
        de += (double)wv * (double)u;
        rr_new += (double)r * (double)r;
      }
      __syncthreads();
    }
    CGT(2);
#ifdef TSB_CG_TRACE
    if (k == 10 && threadIdx.x == 0 && blockIdx.x < 512) {
      g_cg_cta[blockIdx.x][0] = cgt_now();
      unsigned smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      g_cg_cta[blockIdx.x][1] = smid;
    }
#endif
    cgcg_add3(ga, de, rr_new, red, &g.ws.slots[k + 1]);
    CGT(3);
    cgcg_publish(g, 3, (k + 1) & 1, seq0 + 3 + k, &g.ws.slots[k + 1], wn, nxt ? w_off1 : w_off0);
    CGT(6);
  }
}

// Setup part 1 (ordinary launch): r0 = b (x0 = 0), ||b||^2, then the r0 halo
// and the partial to every rank (exchange step 0, area 2).
__global__ void __launch_bounds__(256) cgcg_start_kernel(Cgcg g) {
  __shared__ double red[8];
  double bb = 0.0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < g.n_own;
       i += static_cast<int64_t>(gridDim.x) * 256) {
    const float v = g.bvec[i];
    g.ws.r[0][i] = v;
    g.x[i] = 0.f;
    bb += (double)v * (double)v;
  }
  cgcg_add3(bb, 0.0, 0.0, red, &g.ws.slots[g.max_iter + 1]);
  cgcg_publish(g, 0, 2, pc_seq_base(g.p) + 1, &g.ws.slots[g.max_iter + 1], g.ws.r[0], g.head);
}

__global__ void cgcg_bump_epoch(char* const* peers, int rank, size_t comm_off, int world) {
  *reinterpret_cast<long long*>(peers[rank] + comm_off + 120 * world) += 1;
}

}  // namespace
}  // namespace tsb

extern "C" size_t trnsparse_bsr_cgcg_workspace_size(int64_t n_alloc, int max_iter) {
  return cgcg_ws_size(n_alloc < 0 ? 0 : n_alloc, max_iter < 0 ? 0 : max_iter);
}

extern "C" int trnsparse_bsr_cgcg_layout(int64_t n_alloc, int max_iter, size_t* offsets) {
  TSB_REQUIRE(offsets && n_alloc >= 0 && max_iter >= 0, "bsr_cgcg_layout: bad argument");
  const size_t head = cgcg_head(max_iter), vb = align256(sizeof(float) * (size_t)n_alloc);
  offsets[0] = 0;             // status record
  offsets[1] = align256(64);  // Slot[max_iter + 2]: {p.Ap, gamma, delta, r.r}
  for (int i = 0; i < kCgcgVecs; ++i) offsets[2 + i] = head + i * vb;  // r0 r1 s0 s1 w0 w1 p
  return TRNSPARSE_OK;
}

extern "C" int trnsparse_bsr_cgcg_solve(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                                        const int* col_idx, const float* blocks, const float* b_vec, float* x,
                                        const float* inv_d, double tol, int max_iter, int64_t n_alloc, void* ws,
                                        size_t ws_off, size_t ws_bytes, PEER_ARGS, void* stream) {
  const BsrDesc d = BSR_DESC;
  int rc = check_desc(d, "bsr_cgcg_solve");
  if (rc) return rc;
  TSB_REQUIRE(d.fast(), "bsr_cgcg_solve: needs block size 128 and block-aligned shapes");
  TSB_REQUIRE(ws && x && b_vec && max_iter >= 0 && n_alloc >= n && peers && world > 0 && rank >= 0 &&
                  rank < world && (n_sends == 0 || sends),
              "bsr_cgcg_solve: bad argument");
  TSB_REQUIRE(ws_bytes >= cgcg_ws_size(n_alloc, max_iter), "bsr_cgcg_solve: workspace too small");
  cudaStream_t st = as_stream(stream);
  Cgcg g;
  g.row_ptr = row_ptr;
  g.col_idx = col_idx;
  g.blocks = reinterpret_cast<const float4*>(blocks);
  g.n_block_rows = (int)d.block_rows();
  g.n_own = m;
  g.inv_d = inv_d;
  g.bvec = b_vec;
  g.x = x;
  g.ws = cgcg_ws(ws, n_alloc, max_iter);
  g.ws_off = ws_off;
  g.vec_bytes = align256(sizeof(float) * (size_t)n_alloc);
  g.head = cgcg_head(max_iter);
  g.tol = tol;
  g.max_iter = max_iter;
  g.p = PEER_CTX;
  TSB_REQUIRE(all_aligned({inv_d, x, g.ws.r[0], g.ws.p}), "bsr_cgcg_solve: vectors must be 16-byte aligned");
  // Clear status, slots, s_{-1} and p_{-1}. r and w are left alone: they are written before
  // they are read, and a faster peer may already have pushed this solve's r0 halo rows.
  cudaError_t e = cudaMemsetAsync(ws, 0, g.head, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(g.ws.s[0], 0, g.vec_bytes, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(g.ws.p, 0, g.vec_bytes, st);
  if (e != cudaSuccess) return cuda_status(e, "bsr_cgcg_solve: clear");
  cgcg_bump_epoch<<<1, 1, 0, st>>>(reinterpret_cast<char* const*>(peers), rank, comm_off, world);
  TSB_CHECK_LAUNCH("bsr_cgcg_solve: epoch");
  cgcg_start_kernel<<<vec_grid(m), 256, 0, st>>>(g);
  TSB_CHECK_LAUNCH("bsr_cgcg_solve: start");
  const bool keep = fits_l2(static_cast<size_t>(n_blocks) * 128 * 128 * 4);
  const void* kern = keep ? (const void*)cgcg_solve_kernel<true> : (const void*)cgcg_solve_kernel<false>;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0);
  if (e != cudaSuccess) return cuda_status(e, "bsr_cgcg_solve: occupancy");
  int64_t grid = static_cast<int64_t>(sm_count()) * (per_sm < 1 ? 1 : per_sm);
  if (grid > g.n_block_rows) grid = g.n_block_rows;
  if (grid < 1) grid = 1;
  void* args[] = {(void*)&g};
  e = cudaLaunchCooperativeKernel(kern, dim3((unsigned)grid), dim3(256), args, 0, st);
  if (e != cudaSuccess) return cuda_status(e, "bsr_cgcg_solve: cooperative launch");
  return TRNSPARSE_OK;
}

#ifdef TSB_CG_TRACE
__device__ unsigned long long tsb::g_cg_trace[512][8];
__device__ unsigned tsb::g_cg_trace_n;
__device__ unsigned long long tsb::g_cg_cta[512][4];
extern "C" __attribute__((visibility("default"))) int trnsparse_cg_cta_read(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, tsb::g_cg_cta, sizeof(tsb::g_cg_cta));
}
extern "C" __attribute__((visibility("default"))) int trnsparse_cg_trace_read(unsigned long long* host) {
  unsigned zero = 0;
  int rc = (int)cudaMemcpyFromSymbol(host, tsb::g_cg_trace, sizeof(tsb::g_cg_trace));
  cudaMemcpyToSymbol(tsb::g_cg_trace_n, &zero, sizeof(zero));
  return rc;
}
#endif
