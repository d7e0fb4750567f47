"""trnsparse_b200 — B200 (sm_100a) implementation of trnsparse's sparse compute path.

Drop-in for the reference trnsci/trnsparse v0.6.0 public API
(trnsparse/__init__.py:10-66): same names, signatures and semantics, with the
hot ops (spmv, spmm, bsr_spmm, screened_spmm, block_sparse_attention_tiled and
the BSR solvers) running as hand-written CUDA kernels behind the C ABI in
include/trnsparse_b200.h. There is no CPU compute path.
"""

__version__ = "0.6.0"

from .backend import HAS_NKI, get_backend, set_backend
from .formats import BSRMatrix, COOMatrix, CSRMatrix, eye_sparse, from_dense, from_scipy
from .iterative import (
    bsr_diagonal,
    cg_bsr,
    chebyshev_bsr,
    chebyshev_coeffs,
    jacobi_preconditioner_bsr,
    power_iteration_bsr,
    richardson_bsr,
)
from .ops import (
    block_sparse_attention_tiled,
    bsr_spmm,
    nnz_per_row,
    screened_spmm,
    sparse_add,
    sparse_scale,
    sparse_transpose,
    spmm,
    spmv,
    spmv_symmetric,
)
from .screening import density_screen, schwarz_bounds, screen_quartets, sparsity_stats

__all__ = [
    "CSRMatrix",
    "COOMatrix",
    "BSRMatrix",
    "from_dense",
    "from_scipy",
    "eye_sparse",
    "spmv",
    "spmm",
    "spmv_symmetric",
    "bsr_spmm",
    "screened_spmm",
    "block_sparse_attention_tiled",
    "sparse_add",
    "sparse_scale",
    "sparse_transpose",
    "nnz_per_row",
    "schwarz_bounds",
    "screen_quartets",
    "density_screen",
    "sparsity_stats",
    "cg_bsr",
    "chebyshev_bsr",
    "chebyshev_coeffs",
    "richardson_bsr",
    "power_iteration_bsr",
    "jacobi_preconditioner_bsr",
    "bsr_diagonal",
    "HAS_NKI",
    "set_backend",
    "get_backend",
]
