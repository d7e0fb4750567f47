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

/* OUT = alpha * (A @ B) [+ beta * C]   (B is n x k, row stride ldb; C and OUT
 * are m x k with row stride ldc / ldo). Replaces nki_spmm
 * (trnsparse/nki/dispatch.py:181-190) and the CPU path at ops.py:51-78.
 * `C` may be NULL. */
TRNSPARSE_API int trnsparse_csr_spmm(int64_t m, int64_t n, int64_t k, int64_t nnz, int index_type, int dtype,
                       const void* row_ptrs, const void* col_indices, const void* values,
                       const void* B, int64_t ldb, double alpha, const void* C, int64_t ldc,
                       double beta, void* out, int64_t ldo, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TRNSPARSE_B200_H */
