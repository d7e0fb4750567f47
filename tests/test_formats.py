"""Host-side format semantics, checked bit-exactly against the reference's outputs."""

from __future__ import annotations

import pytest
import torch

import trnsparse_b200 as ts
from conftest import golden_cases, golden_names


@pytest.mark.parametrize("name", golden_names("spmv") + golden_names("spmm"))
def test_csr_from_dense_structure(name):
    c = golden_cases()[name]
    csr = ts.from_dense(c["dense"])
    d = c["csr"]
    assert torch.equal(csr.values, d["values"])
    assert torch.equal(csr.col_indices, d["col_indices"])
    assert torch.equal(csr.row_ptrs, d["row_ptrs"])
    assert csr.col_indices.dtype == d["col_indices"].dtype and csr.row_ptrs.dtype == d["row_ptrs"].dtype
    assert torch.equal(csr.to_dense(), c["dense"])


@pytest.mark.parametrize("name", golden_names("bsr_spmm"))
def test_bsr_from_dense_structure(name):
    c = golden_cases()[name]
    d = c["bsr"]
    if "dense" not in c:
        pytest.skip("fixture stores structure only")
    bsr = ts.BSRMatrix.from_dense(c["dense"], block_size=d["block_size"], threshold=c["threshold"])
    assert torch.equal(bsr.blocks, d["blocks"])
    assert torch.equal(bsr.block_col_indices, d["block_col_indices"])
    assert torch.equal(bsr.block_row_ptrs, d["block_row_ptrs"])
    assert bsr.block_col_indices.dtype == torch.long and bsr.block_row_ptrs.dtype == torch.long
    assert bsr.shape == d["shape"]
    assert torch.equal(bsr.to_dense(), c["to_dense"])


def test_bsr_threshold_structure_128():
    c = golden_cases()["bsr_b128_threshold"]
    d = c["bsr"]
    bsr = ts.BSRMatrix(d["blocks"], d["block_col_indices"], d["block_row_ptrs"], d["shape"], d["block_size"])
    dense = bsr.to_dense()
    again = ts.BSRMatrix.from_dense(dense, block_size=128, threshold=c["threshold"])
    assert torch.equal(again.block_col_indices, d["block_col_indices"])
    assert torch.equal(again.block_row_ptrs, d["block_row_ptrs"])


def test_empty_and_density():
    bsr = ts.BSRMatrix.from_dense(torch.zeros(16, 16), block_size=8)
    assert bsr.n_blocks == 0 and bsr.density == 0.0
    assert torch.equal(bsr.to_dense(), torch.zeros(16, 16))


def test_coo_roundtrip_and_transpose_structure():
    torch.manual_seed(0)
    A = torch.randn(9, 7)
    A[A.abs() < 0.8] = 0
    csr = ts.from_dense(A)
    assert torch.equal(csr.to_coo().to_csr().to_dense(), A)
    assert torch.equal(ts.sparse_transpose(csr).to_dense(), A.T)
    assert torch.equal(ts.sparse_add(csr, csr, 1.0, 2.0).to_dense(), 3.0 * A)
    assert torch.equal(ts.sparse_scale(csr, 3.0).to_dense(), 3.0 * A)
    assert ts.nnz_per_row(csr).tolist() == (A != 0).sum(1).tolist()


def test_eye_and_scipy():
    sp = pytest.importorskip("scipy.sparse")
    I = ts.eye_sparse(5)
    assert torch.equal(I.to_dense(), torch.eye(5))
    M = sp.random(10, 8, density=0.3, random_state=0, format="csr")
    c = ts.from_scipy(M)
    assert c.values.dtype == torch.float32 and c.col_indices.dtype == torch.long
    assert torch.allclose(c.to_dense(), torch.tensor(M.toarray(), dtype=torch.float32))


def test_backend_is_cuda_only():
    assert ts.HAS_NKI is False
    assert ts.get_backend() == "cuda"
    ts.set_backend("auto")
    with pytest.raises(ValueError):
        ts.set_backend("pytorch")


def test_workload_shapes():
    from trnsparse_b200 import workloads as w

    A = w.poisson2d_csr(64)
    assert A.nnz == 5 * 64 * 64 - 4 * 64 and A.row_ptrs.dtype == torch.int32
    d = A.to_dense()
    assert torch.equal(d, d.T) and torch.all(d.diagonal() == 4)
    m = w.sliding_window_mask()  # 128 block-rows: window of 8 plus 2 global columns
    assert m.n_blocks == sum(len({j for j in range(i + 1) if i - j < 8 or j < 2}) for i in range(128)) == 1235
    A5, b5 = w.block_pentadiagonal_spd(8, b=16)
    D = A5.to_dense()
    assert torch.allclose(D, D.T) and torch.linalg.eigvalsh(D.double()).min() > 0


def test_public_api_matches_reference_names():
    """The 30 names of the reference's trnsparse/__init__.py:36-66 are all exported."""
    ref = ["CSRMatrix", "COOMatrix", "BSRMatrix", "from_dense", "from_scipy", "eye_sparse", "spmv", "spmm",
           "spmv_symmetric", "bsr_spmm", "screened_spmm", "block_sparse_attention_tiled", "sparse_add",
           "sparse_scale", "sparse_transpose", "nnz_per_row", "schwarz_bounds", "screen_quartets", "density_screen",
           "sparsity_stats", "cg_bsr", "chebyshev_bsr", "chebyshev_coeffs", "richardson_bsr", "power_iteration_bsr",
           "jacobi_preconditioner_bsr", "bsr_diagonal", "HAS_NKI", "set_backend", "get_backend"]
    assert sorted(ts.__all__) == sorted(ref)
    for n in ref:
        assert hasattr(ts, n)


def test_threshold_rounds_to_the_matrix_dtype():
    """The device builders compare in the matrix dtype, as torch does with a
    Python scalar: the float32 0.1 is not > 0.1, the bf16 0.1 is not > 0.1."""
    from trnsparse_b200.formats import _threshold_in

    for dt in (torch.float32, torch.bfloat16):
        v = torch.tensor([0.1, 0.2, 1e-3], dtype=dt)
        for thr in (0.1, 0.15, 1e-3, 0.0, -1.0):
            t = _threshold_in(dt, thr)
            assert torch.equal(v.abs() > thr, v.float().abs() > t)


def test_spmv_pipeline_plan():
    """Host plan of the pinned-host spmv pipeline: row chunks of whole 64-row
    groups covering [0, m), and per chunk the x prefix its columns reach,
    non-decreasing (a chunk never waits for less than an earlier one)."""
    from trnsparse_b200 import ops, workloads as w

    A = w.poisson2d_csr(64)  # 4096 rows, band +-64
    for K in (1, 3, 4, 7):
        nch, splits, need = ops._spmv_pipe_plan(A.row_ptrs, A.col_indices, A.shape[0], K)
        s = splits.tolist()
        assert s[0] == 0 and s[-1] == A.shape[0] and nch == len(s) - 1
        assert all(b > a and a % 64 == 0 for a, b in zip(s, s[1:]))
        nd = need.tolist()
        assert nd == sorted(nd) and nd[-1] == A.shape[1]
        for i in range(nch):
            lo, hi = int(A.row_ptrs[s[i]]), int(A.row_ptrs[s[i + 1]])
            assert nd[i] >= int(A.col_indices[lo:hi].max()) + 1
    # rows without entries need nothing more than the rows before them
    E = ts.CSRMatrix(values=torch.ones(2), col_indices=torch.tensor([5, 7]),
                     row_ptrs=torch.tensor([0, 1] + [1] * 200 + [2]), shape=(202, 10))
    nch, splits, need = ops._spmv_pipe_plan(E.row_ptrs, E.col_indices, 202, 4)
    assert need.tolist() == [6, 6, 6, 8][:nch]
