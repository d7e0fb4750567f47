/*
 * trnsparse_b200 — C ABI of the B200 (sm_100a) sparse compute path.
 *
 * This header is the drop-in boundary that replaces the reference's
 * accelerator backend (trnsparse/nki/dispatch.py + trnsparse/nki/kernels.py).
 * Every entry point takes plain device pointers, sizes and dtype/index enums,
 * launches on the given CUDA stream (a cudaStream_t passed as void*; NULL is
 * the legacy default stream), never synchronises, and returns a
 * trnsparse_status. On failure trnsparse_last_error() returns a message for
 * the calling thread. Outputs are written, never allocated, by the library:
 * the caller owns all memory, including the scratch buffers some entry
 * points ask for (their sizes come from the matching *_workspace_size call).
 *
 * Citations "file:line" refer to the reference project trnsci/trnsparse
 * v0.6.0.
 */
#ifndef TRNSPARSE_B200_H
#define TRNSPARSE_B200_H

#include <stdint.h>
#include <stddef.h>

#if defined(__GNUC__)
#define TRNSPARSE_API __attribute__((visibility("default")))
#else
#define TRNSPARSE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status, dtypes ---------------------------------------------------- */
enum trnsparse_status {
  TRNSPARSE_OK = 0,
  TRNSPARSE_ERR_ARG = 1,         /* bad shape / size / pointer (reference: AssertionError) */
  TRNSPARSE_ERR_DTYPE = 2,       /* unsupported dtype or index type */
  TRNSPARSE_ERR_ALIGN = 3,       /* pointer alignment a kernel requires is not met */
  TRNSPARSE_ERR_CUDA = 4,        /* a CUDA runtime/driver call failed */
  TRNSPARSE_ERR_TIMEOUT = 5,     /* a bounded device-side wait gave up */
  TRNSPARSE_ERR_UNSUPPORTED = 6, /* valid request this build does not implement */
  TRNSPARSE_ERR_VALUE = 7        /* numerical precondition failed (reference: ValueError) */
};

enum trnsparse_dtype { TRNSPARSE_F32 = 0, TRNSPARSE_F64 = 1, TRNSPARSE_BF16 = 2, TRNSPARSE_F16 = 3 };
enum trnsparse_index { TRNSPARSE_I32 = 0, TRNSPARSE_I64 = 1 };

/* Message of the last failed call on this host thread ("" if none). */
TRNSPARSE_API const char* trnsparse_last_error(void);
/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
TRNSPARSE_API int trnsparse_version(void);

/* ---- CSR ---------------------------------------------------------------- */

/* out = alpha * (A @ x) [+ beta * y]   (A is m x n CSR, nnz stored entries)
 * Replaces the CPU path of trnsparse/ops.py:30-48 (`spmv`); the reference has
 * no accelerator kernel for it. `y` may be NULL (then beta is ignored), which
 * mirrors `if y is not None and beta != 0.0` at ops.py:46. `row_ptrs` and
 * `col_indices` share `index_type`; `values`, `x`, `y`, `out` share `dtype`
 * (F32 or F64). `out` must not alias x. */
TRNSPARSE_API int trnsparse_csr_spmv(int64_t m, int64_t n, int64_t nnz, int index_type, int dtype,
                       const void* row_ptrs, const void* col_indices, const void* values,
                       const void* x, double alpha, const void* y, double beta, void* out,
                       void* stream);
/* spmv with x and y in pinned HOST memory (the reference's CPU-tensor call,
 * ops.py:30-48, y = alpha A x): x is copied up in prefix pieces on a library
 * copy stream, row chunk i ([row_splits[i], row_splits[i+1]), multiples of 4
 * rows keep the vector path) runs once the first x_need[i] entries of x (the
 * chunk's largest column + 1, non-decreasing) have arrived, and its rows are
 * copied back on a second copy stream while later chunks compute. x_dev (n)
 * is device scratch; out_dev (m) is device scratch, or out_host itself, in
 * which case the chunks' kernels write y straight into the pinned host buffer
 * and no copy back is issued (measured faster: the device-to-host copies
 * otherwise compete with the x uploads). `stream` waits for the last copy:
 * after synchronising it, out_host is complete. row_splits / x_need: host
 * arrays, n_chunks <= 64. Calls on one device are issued one at a time (a
 * lock). */
TRNSPARSE_API int trnsparse_csr_spmv_host(int64_t m, int64_t n, int64_t nnz, int index_type, int dtype,
                            const void* row_ptrs, const void* col_indices, const void* values,
                            const void* x_host, double alpha, void* out_host, void* x_dev, void* out_dev,
                            int n_chunks, const int64_t* row_splits, const int64_t* x_need, void* stream);

/* OUT = alpha * (A @ B) [+ beta * C]   (B is n x k, row stride ldb; C and OUT
 * are m x k with row stride ldc / ldo). Replaces nki_spmm
 * (trnsparse/nki/dispatch.py:181-190) and the CPU path at ops.py:51-78.
 * `C` may be NULL. */
TRNSPARSE_API int trnsparse_csr_spmm(int64_t m, int64_t n, int64_t k, int64_t nnz, int index_type, int dtype,
                       const void* row_ptrs, const void* col_indices, const void* values,
                       const void* B, int64_t ldb, double alpha, const void* C, int64_t ldc,
                       double beta, void* out, int64_t ldo, void* stream);


/* Reads the device-side error word (first bounded wait that gave up, 0 if
 * none) of the current device; clears it when `clear` is non-zero. Blocks
 * until prior work on the device completes. */
TRNSPARSE_API int trnsparse_device_error(int* code, int clear);

/* ---- BSR geometry -------------------------------------------------------
 * Every BSR entry point takes the same seven leading arguments, the device
 * image of a reference BSRMatrix (trnsparse/formats.py:130-263):
 *   m, n       element shape (padding to whole blocks is implicit)
 *   b          block size
 *   n_blocks   stored blocks
 *   row_ptr    int32[ceil(m/b)+1]  block_row_ptrs
 *   col_idx    int32[n_blocks]     block_col_indices
 *   blocks     float[n_blocks*b*b] row-major blocks, contiguous
 * b == 128 with m, n multiples of 128 takes the coalesced warp-per-row-slice
 * kernels; other geometries take a generic thread-per-row kernel. */

/* out = alpha * (A @ x) [+ beta * y]: the reference's bsr_spmm with one
 * right-hand-side column (trnsparse/iterative.py:44-50 `_bsr_matvec`). */
TRNSPARSE_API int trnsparse_bsr_spmv(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                       const int* col_idx, const float* blocks, const float* x, double alpha,
                       const float* y, double beta, float* out, void* stream);

/* ---- BSR conjugate gradient (trnsparse/iterative.py:53-145) --------------
 * Device-resident PCG with the reference's control flow: zero right-hand
 * side returns (x0, 0, 0.0); |p.Ap| < 1e-30 breaks (iters = max_iter);
 * ||r||/||b|| < tol returns after that iteration. inv_d (nullable) is the
 * Jacobi preconditioner 1/diag(A) (iterative.py:129-145).
 * Workspace: trnsparse_bsr_cg_workspace_size(n, max_iter) bytes, 256-byte
 * aligned; its first 64 bytes are the status record
 *   { int32 done, iters, reason, pad; double rel; double bb; double pad[4]; }
 * (reason: 1 converged, 2 max_iter, 3 breakdown, 4 zero rhs).
 * Usage: cg_start once, then cg_iterate over consecutive ranges
 * [k_begin, k_end) up to k_end = max_iter + 1 (the last range records the
 * final status), polling `done` between ranges as often as wanted. x holds
 * x0 on entry and is updated in place. */
TRNSPARSE_API size_t trnsparse_bsr_cg_workspace_size(int64_t n, int max_iter);
TRNSPARSE_API int trnsparse_bsr_cg_start(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                           const int* col_idx, const float* blocks, const float* b_vec, const float* x,
                           int x_is_zero, const float* inv_d, int max_iter, void* ws, size_t ws_bytes,
                           void* stream);
TRNSPARSE_API int trnsparse_bsr_cg_iterate(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                             const int* col_idx, const float* blocks, float* x, const float* inv_d,
                             double tol, int max_iter, int k_begin, int k_end, void* ws, void* stream);

/* Chebyshev semi-iteration, K fixed steps (trnsparse/iterative.py:193-253).
 * alpha/beta: HOST arrays of K float32 coefficients (chebyshev_coeffs);
 * x: x0 in, x_K out; work: 2n floats of device scratch; rr_out: device
 * double receiving ||b - A x_K||^2. One fused SpMV launch per step. */
TRNSPARSE_API int trnsparse_bsr_chebyshev(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                            const int* col_idx, const float* blocks, const float* b_vec,
                            const float* alpha, const float* beta, int K, float* x, float* work,
                            double* rr_out, void* stream);

/* Richardson, x += omega (b - A x), K fixed steps (iterative.py:256-295);
 * work: n floats of device scratch; rr_out as above. */
TRNSPARSE_API int trnsparse_bsr_richardson(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                             const int* col_idx, const float* blocks, const float* b_vec, double omega,
                             int K, float* x, float* work, double* rr_out, void* stream);

/* Row-shard steps for the block-row-sharded fixed-step solvers and power
 * iteration (the reference's chebyshev_bsr / richardson_bsr /
 * power_iteration_bsr loops, iterative.py:193-340, split across ranks; the
 * caller refreshes halo columns and reduces partial sums between steps).
 * The BSR is the rank's shard: m own rows, n own + halo columns.
 *   chebyshev_step: xnext = xk + a (b - A xk) [+ bcoef (xk - xprev)]
 *                   (own rows; xk has its halo filled; richardson: momentum 0).
 *   residual_sq:    *acc += ||b - A x||^2 over the own rows.
 *   power_step:     w = A v (own rows); dots[0] += v.w, dots[1] += w.w.
 *   vec_div_norm:   y = x / fp32(sqrt(*ss)). */
TRNSPARSE_API int trnsparse_bsr_chebyshev_step(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                                  const int* col_idx, const float* blocks, const float* b_vec,
                                  const float* xk, const float* xprev, float* xnext, double a, double bcoef,
                                  int momentum, void* stream);
TRNSPARSE_API int trnsparse_bsr_residual_sq(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                               const int* col_idx, const float* blocks, const float* b_vec, const float* x,
                               double* acc, void* stream);
TRNSPARSE_API int trnsparse_bsr_power_step(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                              const int* col_idx, const float* blocks, const float* v, float* w, double* dots,
                              void* stream);
TRNSPARSE_API int trnsparse_vec_div_norm(int64_t n, const float* x, const double* ss, float* y, void* stream);

/* acc = u . v accumulated in float64 (device scalar). */
TRNSPARSE_API int trnsparse_dot(int64_t n, const float* u, const float* v, double* acc, void* stream);

/* Power iteration (trnsparse/iterative.py:298-340). Same chunked protocol as
 * CG: ranges [k_begin, k_end) up to max_iter + 1; k_begin == 0 starts from
 * v0 (normalised on the device); the status record's `rel` field holds the
 * eigenvalue; the final range (k_end == max_iter + 1) or
 * trnsparse_bsr_power_finish writes the returned eigenvector into v. */
TRNSPARSE_API size_t trnsparse_bsr_power_workspace_size(int64_t n, int max_iter);
TRNSPARSE_API int trnsparse_bsr_power_iterate(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                                const int* col_idx, const float* blocks, const float* v0, float* v,
                                double tol, int max_iter, int k_begin, int k_end, void* ws,
                                size_t ws_bytes, void* stream);
TRNSPARSE_API int trnsparse_bsr_power_finish(int64_t n, float* v, int max_iter, void* ws, void* stream);

/* ---- BSR x dense -------------------------------------------------------- */

/* C = A @ B on CUDA cores (fp32 FMA), any block size: the reference's
 * `_bsr_spmm_pytorch` (trnsparse/ops.py:162-192), which nki_bsr_spmm
 * (trnsparse/nki/dispatch.py:372-381) accelerates. B is n x k with row
 * stride ldb; C is m x k with row stride ldc (rows of empty block-rows are
 * written as zeros). */
TRNSPARSE_API int trnsparse_bsr_spmm_simt(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                            const int* col_idx, const float* blocks, const float* B, int64_t k,
                            int64_t ldb, float* C, int64_t ldc, void* stream);

/* C = A @ B on the tensor cores (tcgen05.mma, TMA, TMEM), block size 128
 * only: the hot path of the reference's bsr_spmm (trnsparse/ops.py:195-210)
 * that nki_bsr_spmm replaces on Trainium (trnsparse/nki/dispatch.py:372-381).
 *   dtype F32: 3xTF32 (hi*hi + hi*lo + lo*hi); blocks_hi/blocks_lo are the
 *              tf32 split of the blocks (trnsparse_bsr_split_tf32); B, C fp32.
 *   dtype BF16: blocks_hi and B are bf16 (blocks_lo unused).
 * c_dtype: F32, or BF16 (bf16 inputs only: each unit's fp32 accumulator is
 * rounded once in the epilogue; units of a split block-row add their rounded
 * partial sums into the cleared bf16 C).
 * plan (device memory): the work schedule written on the host by
 * trnsparse_bsr_spmm_tc_plan for this matrix's row pointers, k, bn and grid
 * (CTA count; cache it per matrix). needs_zero: that call's flag (C is
 * cleared first when a block-row is split across units).
 * C (m x k, row stride ldc elements, rows 16-byte aligned) is overwritten. bn: N tile, 128 or 256 (the plan's). Workspace:
 * trnsparse_bsr_spmm_tc_workspace_size(n, k, dtype) bytes (F32: B^T split;
 * BF16: a padded copy of B, used only when B's rows are not 16-byte aligned
 * or k < 64). */
TRNSPARSE_API size_t trnsparse_bsr_spmm_tc_workspace_size(int64_t n, int64_t k, int dtype);
TRNSPARSE_API int trnsparse_bsr_spmm_tc(int64_t m, int64_t n, int64_t n_blocks, const int* col_idx,
                          const void* blocks_hi, const void* blocks_lo, int dtype, const int* plan,
                          int grid, int needs_zero, const void* B, int64_t k, int64_t ldb, void* C,
                          int64_t ldc, int c_dtype, int bn, void* ws, size_t ws_bytes, void* stream);

/* Host-side work schedule for trnsparse_bsr_spmm_tc. row_ptr: the host copy
 * of the n_block_rows + 1 block-row pointers. Units are (block-row, run of at
 * most ~n_blocks * tiles / (3 n_ctas) of its blocks, N tile); they are
 * assigned longest first to the least-loaded of min(n_ctas, units) CTAs.
 * plan: host int32 buffer of `capacity` >= trnsparse_bsr_spmm_tc_plan_capacity
 * entries; outputs the unit count, the grid and whether C needs clearing. */
TRNSPARSE_API int64_t trnsparse_bsr_spmm_tc_plan_capacity(int64_t n_block_rows, int64_t n_blocks, int64_t k,
                                                          int bn, int n_ctas);
TRNSPARSE_API int trnsparse_bsr_spmm_tc_plan(int64_t n_block_rows, const int* row_ptr, int64_t k, int bn,
                                             int n_ctas, int* plan, int64_t capacity, int* n_units,
                                             int* grid, int* needs_zero);

/* hi = tf32(src), lo = tf32(src - hi), elementwise over `count` floats
 * (round to nearest, ties away). Used once per BSR matrix for the F32
 * tensor-core path. hi NULL: only lo = tf32(src - src with its low 13 mantissa
 * bits cleared), for passing src itself as blocks_hi (a kind::tf32 MMA reads
 * only the top 10 mantissa bits of an fp32 operand); one extra copy of the
 * blocks instead of two. */
TRNSPARSE_API int trnsparse_bsr_split_tf32(int64_t count, const float* src, float* hi, float* lo, void* stream);

/* C = (A o mask) @ B with the Schwarz screening mask applied inside the
 * tensor-core kernel (3xTF32, fp32 in/out): the reference's screened_spmm
 * (trnsparse/ops.py:213-277; nki_screened_spmm, trnsparse/nki/dispatch.py:
 * 487-494, kernels.py:86-155). A is M x K (row stride lda), B is K x N
 * (ldb), C is M x N (ldc), all row-major fp32; lda, ldq, ldc multiples of 4
 * and C 16-byte aligned (C is written by TMA stores).
 *   bounds_kind 1: `bounds` is the length-M diag_integrals vector (M == K);
 *                  mask[i,j] = sqrt|d_i| * sqrt|d_j| > fp32(sqrt(threshold)).
 *   bounds_kind 2: `bounds` is the M x K pair-bound matrix Q (row stride ldq)
 *                  of screening.py's schwarz_bounds; mask = Q > fp32(sqrt(thr))
 *                  (screen_quartets, screening.py:29-40).
 * K chunks with no surviving pair issue no MMA. One persistent CTA per SM
 * takes an equal share of the (128-row x N-tile output tile, 128-wide K
 * block) pairs; tiles shared by two CTAs are reduce-added into a cleared C.
 * Workspace:
 * trnsparse_screened_spmm_workspace_size(K, N) bytes (B^T split). */
TRNSPARSE_API size_t trnsparse_screened_spmm_workspace_size(int64_t K, int64_t N);
TRNSPARSE_API int trnsparse_screened_spmm(int64_t M, int64_t K, int64_t N, const float* A, int64_t lda,
                            const float* bounds, int bounds_kind, int64_t ldq, double threshold,
                            const float* B, int64_t ldb, float* C, int64_t ldc, void* ws,
                            size_t ws_bytes, void* stream);

/* Block-sparse attention forward: O = softmax(Q K^T * scale) V restricted to
 * the stored blocks of a BSR mask (pattern only), per head: the reference's
 * block_sparse_attention_tiled (trnsparse/ops.py:549-625; two-pass CPU form
 * ops.py:280-357; nki_bsr_attn_tiled, trnsparse/nki/dispatch.py:580).
 * Q, K, V, O: heads contiguous (heads, seq, head_dim) row-major tensors of
 * `dtype` (F32 or BF16); softmax and accumulation in fp32. The mask has
 * seq/block_size block-rows; rows of an empty block-row, and rows past the
 * last whole block, are zero. head_dim <= 256. */
TRNSPARSE_API int trnsparse_bsr_attention(int64_t heads, int64_t seq, int64_t head_dim, int block_size,
                            const int* block_row_ptr, const int* block_col_idx, const void* Q,
                            const void* K, const void* V, void* O, int dtype, double scale,
                            void* stream);

/* Block-sparse attention backward (reference: _block_sparse_attn_backward,
 * trnsparse/ops.py:360-473; nki_bsr_attn_bwd, trnsparse/nki/dispatch.py:813):
 * dQ, dK, dV of O = softmax(Q K^T scale) V over the stored blocks, by the
 * Flash-delta identity dS = P (dO V^T - rowsum(dO o O)). Layout and dtypes as
 * trnsparse_bsr_attention; head_dim <= 128. block_col_ptr / block_row_idx:
 * the mask's transposed pattern (ceil(seq/b) + 1 column pointers; for each
 * key block, the query blocks that store it); max_col_blocks: the largest
 * number of query blocks storing one key block (more than 8 splits it over
 * CTAs). Workspace: trnsparse_bsr_attention_backward_workspace_size(...)
 * bytes (row max, row sum, delta; fp32 dK/dV accumulators for bf16 when a
 * key block is split). Rows that get no gradient are zero. */
TRNSPARSE_API size_t trnsparse_bsr_attention_backward_workspace_size(int64_t heads, int64_t seq, int64_t head_dim,
                                                         int dtype, int max_col_blocks);
TRNSPARSE_API int trnsparse_bsr_attention_backward(int64_t heads, int64_t seq, int64_t head_dim, int block_size,
                                      const int* block_row_ptr, const int* block_col_idx,
                                      const int* block_col_ptr, const int* block_row_idx, int max_col_blocks,
                                      const void* Q, const void* K, const void* V, const void* O, const void* dO,
                                      void* dQ, void* dK, void* dV, int dtype, double scale, void* ws,
                                      size_t ws_bytes, void* stream);

/* Tensor-core form of trnsparse_bsr_attention for bf16, block size 128,
 * head_dim 64 or 128, seq a multiple of 128: tcgen05 S = Q K^T and O += P V
 * with TMEM accumulators in one pass (an online softmax whose running max
 * moves only when a block's max exceeds it by 2^8; numerator and denominator
 * share it, so O equals the reference's exp(s - max) / sum @ V up to
 * rounding). */
TRNSPARSE_API int trnsparse_bsr_attention_tc(int64_t heads, int64_t seq, int64_t head_dim, const int* block_row_ptr,
                               const int* block_col_idx, const void* Q, const void* K, const void* V,
                               void* O, double scale, void* stream);
/* As trnsparse_bsr_attention_tc; lse (nullable, fp32 [heads * seq]) receives
 * each row's log-sum-exp in base-2 units of the scaled scores,
 * log2(sum_j exp2(s_j * scale * log2(e))), which the tensor-core backward takes. */
TRNSPARSE_API int trnsparse_bsr_attention_tc_lse(int64_t heads, int64_t seq, int64_t head_dim,
                                   const int* block_row_ptr, const int* block_col_idx, const void* Q,
                                   const void* K, const void* V, void* O, float* lse, double scale, void* stream);

/* Tensor-core backward (bf16, block 128, head_dim 64/128, seq % 128 == 0) of
 * the reference's _block_sparse_attn_backward (trnsparse/ops.py:360-473).
 * The plan (host, int32) lists row units (query block, range of
 * block_col_idx), column units (key block, range of block_row_idx of the
 * transposed pattern) and aux entries (blocks with no stored partner, and
 * blocks split over several units, whose partial sums go through fp32
 * workspace slots); plan == NULL only fills counts = {row units, column
 * units, aux entries, slots}. split bounds the partner blocks per unit. */
TRNSPARSE_API int trnsparse_bsr_attention_backward_tc_plan(int64_t n_block_rows, int64_t n_block_cols,
                                             const int* block_row_ptr, const int* block_col_ptr, int split,
                                             int* plan, int64_t plan_capacity, int64_t* counts);
TRNSPARSE_API size_t trnsparse_bsr_attention_backward_tc_workspace_size(int64_t heads, int64_t seq, int64_t head_dim,
                                                          int64_t n_slots);
/* plan: the device copy of the plan above (16-byte aligned). lse: the
 * forward's trnsparse_bsr_attention_tc_lse output, or NULL (then the forward
 * is rerun for it, into dQ as scratch). */
TRNSPARSE_API int trnsparse_bsr_attention_backward_tc(int64_t heads, int64_t seq, int64_t head_dim,
                                        const int* block_row_ptr, const int* block_col_idx,
                                        const int* block_row_idx, const int* plan, int n_row_units,
                                        int n_col_units, int n_aux, int n_slots, const void* Q, const void* K,
                                        const void* V, const void* O, const void* dO, const float* lse, void* dQ,
                                        void* dK, void* dV, double scale, void* ws, size_t ws_bytes, void* stream);

/* ---- block-row-sharded CG (one process per GPU) --------------------------
 * The multi-GPU form of cg_bsr (trnsparse/iterative.py:53-126; the
 * reference itself has no multi-device code). A rank owns n_own rows; its
 * BSR geometry has m = n_own rows and n = n_ext columns, columns >= n_own
 * being halo copies of rows owned by other ranks. Workspace vectors are
 * n_ext long (trnsparse_bsr_cg_workspace_size(n_ext, max_iter)); offsets[6]
 * receives the byte offsets of {status, slots, r, p_even, p_odd, Ap}. Slot k
 * (32 bytes) holds {p.Ap, r0.z0 (k = 0), r.r, r.z} for iteration k. Per
 * iteration k the caller runs phase 0 (fused SpMV + p update), sums slot k's
 * first double over ranks, runs phase 1 (x, r update), sums slot k's last two
 * doubles over ranks and refreshes the halo part of r. dist_start needs the
 * sum of status.bb and slot 0's second double over ranks before phase 0 of
 * iteration 0. inv_d must hold the halo's inverse diagonal too. */
TRNSPARSE_API int trnsparse_bsr_cg_layout(int64_t n, int max_iter, size_t* offsets);
TRNSPARSE_API int trnsparse_bsr_cg_dist_start(int64_t n_own, int64_t n_ext, const float* b_vec, const float* inv_d,
                                int max_iter, void* ws, size_t ws_bytes, void* stream);
TRNSPARSE_API int trnsparse_bsr_cg_dist_phase(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                                const int* col_idx, const float* blocks, float* x, const float* inv_d,
                                double tol, int max_iter, int k, int phase, void* ws, void* stream);

/* ---- peer memory for the sharded solvers (NVLink, one process per GPU) ---
 * No reference counterpart (the reference has no multi-device code); used by
 * the block-row-sharded CG instead of small NCCL collectives. peer_alloc
 * returns a zeroed device buffer and its 64-byte CUDA IPC handle; other ranks
 * open it with peer_open. peer_comm_bytes(world) is the size of the exchange
 * area a buffer must reserve at `comm_off`. peer_reduce_push (one CTA):
 * stores the halo rows listed in `sends` (int64 triples: source element
 * offset in `src`, destination rank, destination byte offset in that rank's
 * buffer; `chunk` floats each) and the local partials *my_a, *my_b into every
 * peer, raises this rank's flag, waits (bounded) for all peers' flags for
 * (epoch * stride + step + 1), then overwrites *my_a, *my_b with the sums
 * over ranks in rank order. `peers` is a DEVICE array of `world` buffer
 * addresses (this rank's own at index `rank`). area is 0, 1 or 2; two
 * consecutive exchanges must use different areas (the sharded CG uses 2 for
 * its setup exchange and alternates 0 / 1 per iteration); call
 * peer_bump_epoch once per solve on every rank. */
TRNSPARSE_API size_t trnsparse_peer_comm_bytes(int world);
TRNSPARSE_API int trnsparse_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
TRNSPARSE_API int trnsparse_peer_open(const void* ipc_handle, void** ptr);
TRNSPARSE_API int trnsparse_peer_close(void* ptr);
TRNSPARSE_API int trnsparse_peer_free(void* ptr);
TRNSPARSE_API int trnsparse_peer_bump_epoch(void* mine, size_t comm_off, int world, void* stream);
TRNSPARSE_API int trnsparse_peer_reduce_push(void* const* peers, int world, int rank, size_t comm_off, double* my_a,
                               double* my_b, int area, long long stride, long long step,
                               const float* src, const long long* sends, int n_sends, int chunk,
                               void* stream);

/* Sharded CG with the exchanges fused into the solver kernels (no reference
 * counterpart; multi-GPU form of iterative.py:53-126). Same workspace and
 * iteration protocol as trnsparse_bsr_cg_dist_*, but the workspace must lie
 * at offset 0 of this rank's trnsparse_peer_alloc buffer and no host-side
 * reduction or halo exchange is needed: the last CTA of each kernel stores the
 * rank's partial sums (and, after the x/r update, the halo rows of r listed in
 * `sends`, `b` floats each) into every peer's buffer and raises a flag; the
 * next kernel waits (bounded) for all flags and sums in rank order. Block size
 * 128, block-aligned shapes. `peers` is a device array of the world's buffer
 * addresses. Every rank must make the same sequence of calls. */
TRNSPARSE_API int trnsparse_bsr_cg_fused_start(int64_t n_own, int64_t n_ext, int b, const float* b_vec,
                                 const float* inv_d, int max_iter, void* ws, size_t ws_bytes,
                                 void* const* peers, int world, int rank, size_t comm_off,
                                 const long long* sends, int n_sends, void* stream);
TRNSPARSE_API int trnsparse_bsr_cg_fused_phase(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                                 const int* col_idx, const float* blocks, float* x, const float* inv_d,
                                 double tol, int max_iter, int k, int phase, void* ws, void* const* peers,
                                 int world, int rank, size_t comm_off, const long long* sends, int n_sends,
                                 void* stream);

/* The fused sharded CG in one cooperative launch for iterations k_begin ..
 * k_end (k == max_iter only records the final status): every iteration's
 * two phases run back to back inside the kernel, the peer flags serving as
 * the grid-wide barrier. Same buffers, protocol and requirements as
 * trnsparse_bsr_cg_fused_*; start with trnsparse_bsr_cg_fused_start. */
TRNSPARSE_API int trnsparse_bsr_cg_coop_run(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                               const int* col_idx, const float* blocks, float* x, const float* inv_d,
                               double tol, int max_iter, int k_begin, int k_end, void* ws, void* const* peers,
                               int world, int rank, size_t comm_off, const long long* sends, int n_sends,
                               void* stream);

/* Sharded Jacobi-PCG with one reduction per iteration (Chronopoulos-Gear
 * recurrences; the same iterates as the reference's cg_bsr in exact
 * arithmetic, trnsparse/iterative.py:53-126), whole solve in one
 * cooperative launch after a small start kernel, exchanges over the peer
 * buffers of trnsparse_peer_* (CUDA IPC, one NVLink box). Every rank's
 * workspace holds n_alloc entries per vector (the largest n_ext of all
 * ranks), laid out per trnsparse_bsr_cgcg_layout, at byte offset ws_off of its
 * peer buffer; sends: n_sends triples (source element, destination rank,
 * destination element) of the b-row halo chunks this rank owes. x0 = 0;
 * inv_d (n_ext, halo filled) or null. Status record and slots as for the
 * other CG entry points (slot k: p.Ap, gamma, delta, r.r). */
TRNSPARSE_API size_t trnsparse_bsr_cgcg_workspace_size(int64_t n_alloc, int max_iter);
TRNSPARSE_API int trnsparse_bsr_cgcg_layout(int64_t n_alloc, int max_iter, size_t* offsets /* 9 */);
TRNSPARSE_API int trnsparse_bsr_cgcg_solve(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                               const int* col_idx, const float* blocks, const float* b_vec, float* x,
                               const float* inv_d, double tol, int max_iter, int64_t n_alloc, void* ws,
                               size_t ws_off, size_t ws_bytes, void* const* peers, int world, int rank,
                               size_t comm_off, const long long* sends, int n_sends, void* stream);

/* Allocation-free PCG. No counterpart in the reference: it exists for
 * callers that cannot allocate device memory (code running inside an
 * allocator or pool callback, or hosts with a fixed up-front memory budget).
 * Runs the same solve as trnsparse_bsr_cg_start + trnsparse_bsr_cg_iterate
 * over [0, max_iter + 1), but its scratch is a fixed 64 MiB array inside the
 * library, held on every GPU that loads the library until exit, instead of a
 * caller workspace; sizes whose trnsparse_bsr_cg_workspace_size exceeds that
 * are rejected with TRNSPARSE_ERR_ARG. The array belongs to the library's
 * device module: the driver creates it (64 MiB) when that module is first
 * loaded on a device, which, under CUDA's default lazy loading, is the first
 * call of ANY library function on that device. A caller that must not
 * allocate later should make one library call per device at start-up (this
 * entry point included: its first call on a device also looks up the array's
 * device address with cudaGetSymbolAddress), before any allocator callback
 * or stream capture. The address is kept per device for the life of the
 * process; do not call this entry point after cudaDeviceReset, which reloads
 * the module. All calls share the one array, so calls that
 * overlap on the GPU (other streams, other host threads) race; run them one
 * after another. status_out (nullable, device, 64 bytes) receives the final
 * status record described above. Calls no allocating routine. */
TRNSPARSE_API int trnsparse_bsr_cg_noalloc(int64_t m, int64_t n, int b, int64_t n_blocks, const int* row_ptr,
                             const int* col_idx, const float* blocks, const float* b_vec, float* x,
                             int x_is_zero, const float* inv_d, double tol, int max_iter,
                             void* status_out, void* stream);

/* ---- device-side format construction --------------------------------
 * BSRMatrix.from_dense (trnsparse/formats.py:184-221): a block is kept iff
 * max |v| over the block (zero-padded past the matrix edge) exceeds the
 * threshold; kept blocks in row-major block order. Two calls: _count fills
 * block_row_ptr (int64 [ceil(m/b) + 1], device) and keeps the block slots in
 * ws; the caller reads block_row_ptr's last entry (the block count),
 * allocates, and _fill writes blocks (n_blocks x b x b, A's dtype) and
 * block_col_idx (int64). threshold: already rounded to A's dtype. A: row-major
 * m x n with leading dimension lda (elements); dtype F32 or BF16. */
TRNSPARSE_API size_t trnsparse_bsr_from_dense_workspace_size(int64_t m, int64_t n, int block_size);
TRNSPARSE_API int trnsparse_bsr_from_dense_count(int64_t m, int64_t n, const void* A, int64_t lda, int dtype,
                                   int block_size, float threshold, long long* block_row_ptr, void* ws,
                                   size_t ws_bytes, void* stream);
TRNSPARSE_API int trnsparse_bsr_from_dense_fill(int64_t m, int64_t n, const void* A, int64_t lda, int dtype,
                                  int block_size, void* blocks, long long* block_col_idx, const void* ws,
                                  void* stream);
/* CSR from_dense (formats.py:269-278): entries with |v| > threshold, row by
 * row in column order. _count fills row_ptr (int64 [m + 1]); _fill writes
 * values (A's dtype) and col_idx (int64). */
TRNSPARSE_API size_t trnsparse_csr_from_dense_workspace_size(int64_t m);
TRNSPARSE_API int trnsparse_csr_from_dense_count(int64_t m, int64_t n, const void* A, int64_t lda, int dtype,
                                   float threshold, long long* row_ptr, void* ws, size_t ws_bytes,
                                   void* stream);
TRNSPARSE_API int trnsparse_csr_from_dense_fill(int64_t m, int64_t n, const void* A, int64_t lda, int dtype,
                                  float threshold, const long long* row_ptr, void* values, long long* col_idx,
                                  void* stream);
/* The same count, also writing a bit mask of the kept entries (uint32 words,
 * trnsparse_csr_from_dense_mask_bytes(m, n) bytes: bit c % 32 of word
 * r * ceil(n / 32) + c / 32 for entry (r, c)); _fill_masked then gathers only
 * the kept values instead of reading every row again (fewer bytes while the
 * density stays below roughly one entry in eight 32-byte sectors). Same
 * output as _fill. */
TRNSPARSE_API size_t trnsparse_csr_from_dense_mask_bytes(int64_t m, int64_t n);
TRNSPARSE_API int trnsparse_csr_from_dense_count_mask(int64_t m, int64_t n, const void* A, int64_t lda, int dtype,
                                        float threshold, long long* row_ptr, uint32_t* mask, void* ws,
                                        size_t ws_bytes, void* stream);
TRNSPARSE_API int trnsparse_csr_from_dense_fill_masked(int64_t m, int64_t n, const void* A, int64_t lda, int dtype,
                                         const long long* row_ptr, const uint32_t* mask, void* values,
                                         long long* col_idx, void* stream);
/* COOMatrix.to_csr (formats.py:104-124): entries ordered by (row, col),
 * entries with equal (row, col) in input order (a stable sort). rows, cols:
 * int64 device arrays of nnz entries (nnz < 2^32, n < 2^31); values of dtype
 * F32, F64, BF16 or F16. Outputs: row_ptr (int64 [m + 1]), cols_out (int64),
 * values_out. Synchronises the stream once to report out-of-range indices
 * (TRNSPARSE_ERR_ARG). */
TRNSPARSE_API size_t trnsparse_coo_to_csr_workspace_size(int64_t m, int64_t nnz);
TRNSPARSE_API int trnsparse_coo_to_csr(int64_t m, int64_t n, int64_t nnz, const long long* rows,
                         const long long* cols, const void* values, int dtype, long long* row_ptr,
                         long long* cols_out, void* values_out, void* ws, size_t ws_bytes, void* stream);

/* ---- CSR value gradient ------------------------------------------------
 * out[e] = alpha * sum_t G[row_e, t] * X[col_e, t] over the stored entries e
 * of A (row_ptrs/col_indices, index_type I32/I64; G m x k, X n x k,
 * row-major, dtype F32/F64): the adjoint of alpha * A @ X with respect to A's
 * values. The reference gets it from torch autograd through the
 * materialised product (nki/dispatch.py:154-178, dA = (dC @ B^T) projected on
 * the pattern); here it is one sampled dense-dense product over the pattern. */
TRNSPARSE_API int trnsparse_csr_sddmm(int64_t m, int64_t n, int64_t k, int64_t nnz, int index_type, int dtype,
                        const void* row_ptrs, const void* col_indices, const void* G, int64_t ldg,
                        const void* X, int64_t ldx, double alpha, void* out, void* stream);

/* ---- block gradients on the tensor cores ------------------------------
 * 128 x 128 output tiles of X Y^T, X (mx x K, row stride ldx) and Y
 * (my x K, ldy) row-major, dtype F32 (3xTF32) or BF16 (fp32 accumulation):
 *   tiles != NULL: packed. tiles holds n_tiles (i, j) int32 pairs (device);
 *     tile u = X[128 i : 128 i + 128] . Y[128 j : 128 j + 128]^T goes to rows
 *     [128 u, 128 u + 128) of `out` (128 columns, row stride ldo): the BSR
 *     block gradient dblocks[k] = dC_i B_j^T of the reference's
 *     _BSRSpMMFunction.backward (trnsparse/nki/dispatch.py:331-369).
 *   tiles == NULL: dense. out (out_rows x out_cols <= mx x my, ldo) = X Y^T,
 *     optionally masked: mask_kind 1, bounds = diagonal integrals d (square):
 *     keep fl(sqrt|d_r| sqrt|d_c|) > fp32(sqrt(threshold)); mask_kind 2,
 *     bounds = pair-bound matrix Q (row stride ldq): keep Q[r, c] >
 *     fp32(sqrt(threshold)). The screened dA = (dC B^T) o mask of
 *     _ScreenedSpMMFunction.backward (nki/dispatch.py:447-484).
 * out: F32 or BF16, 16-byte aligned rows. Rows/columns past X's or Y's edge
 * read as zero. Workspace: trnsparse_nt_tc_workspace_size(mx, my, K, dtype)
 * bytes (F32: the tf32 hi/lo split of X and Y; BF16: padded copies, used
 * only when an operand's rows are not 16-byte aligned or K < 64). */
TRNSPARSE_API size_t trnsparse_nt_tc_workspace_size(int64_t mx, int64_t my, int64_t K, int dtype);
TRNSPARSE_API int trnsparse_nt_tc(int64_t mx, int64_t my, int64_t K, int dtype, const void* X, int64_t ldx,
                    const void* Y, int64_t ldy, const int* tiles, int64_t n_tiles, void* out, int64_t ldo,
                    int out_dtype, int64_t out_rows, int64_t out_cols, int mask_kind, const float* bounds,
                    int64_t ldq, double threshold, void* ws, size_t ws_bytes, void* stream);

/* ---- transposes (autograd adjoints and spmv_symmetric) ----------------
 * Transposed structure of a CSR matrix on the device: the reference builds
 * A^T through a host COO round trip (trnsparse/ops.py:146-154
 * sparse_transpose) and the strict triangle of spmv_symmetric through a
 * coalesced COO tensor (ops.py:81-104). row_ptr/col_idx: index_type I32 or
 * I64. strict != 0 leaves the diagonal entries out (square A only). Outputs:
 * row_ptr_t (int64 [n + 1]), col_t (int64, the source row of each entry of
 * A^T) and perm (int64, the index in A of each entry of A^T); entries of A^T
 * are ordered by (row of A^T, column of A^T) with the first row_ptr_t[n]
 * slots of col_t/perm used. No host synchronisation. The values of A^T are
 * gathered per call with trnsparse_gather (values[perm]), so in-place updates
 * of A's values never see a stale transpose. The same call on a BSR
 * matrix's block pointers gives the transposed block pattern. */
TRNSPARSE_API size_t trnsparse_csr_transpose_workspace_size(int64_t m, int64_t n, int64_t nnz);
TRNSPARSE_API int trnsparse_csr_transpose(int64_t m, int64_t n, int64_t nnz, int index_type, const void* row_ptr,
                            const void* col_idx, int strict, long long* row_ptr_t, long long* col_t,
                            long long* perm, void* ws, size_t ws_bytes, void* stream);
/* dst[p] = src[idx[p]], elements of 2, 4 or 8 bytes (CSR values of A^T). */
TRNSPARSE_API int trnsparse_gather(int64_t count, int elem_bytes, const void* src, const long long* idx, void* dst,
                     void* stream);
/* dst block p = transpose of src block idx[p], b x b blocks of 2- or 4-byte
 * elements: the blocks of A^T in its block order (the reference's autograd
 * transposes every stored block for dB = A^T dC, nki/dispatch.py:331-369). */
TRNSPARSE_API int trnsparse_bsr_blocks_transpose(int64_t count, int b, int elem_bytes, const void* src,
                                   const long long* idx, void* dst, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TRNSPARSE_B200_H */
