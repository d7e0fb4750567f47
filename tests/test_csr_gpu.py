"""CSR spmv / spmm on the GPU (through the C ABI) against the oracle and golden vectors.

Tolerance: fp32 results within 1e-5 relative Frobenius error of the
reference (float64 runs within 1e-12).
"""

from __future__ import annotations

import pytest
import torch

import oracle
import trnsparse_b200 as ts
from conftest import golden_cases, golden_names, rel_fro

pytestmark = pytest.mark.gpu
TOL32 = 1e-5


def _csr(d, index_dtype=None, device="cuda"):
    it = index_dtype or d["row_ptrs"].dtype
    return ts.CSRMatrix(
        values=d["values"].to(device),
        col_indices=d["col_indices"].to(device=device, dtype=it),
        row_ptrs=d["row_ptrs"].to(device=device, dtype=it),
        shape=d["shape"],
    )


@pytest.mark.parametrize("index_dtype", [torch.int64, torch.int32])
@pytest.mark.parametrize("name", golden_names("spmv"))
def test_spmv_golden(name, index_dtype):
    c = golden_cases()[name]
    A = _csr(c["csr"], index_dtype)
    y = None if c["y"] is None else c["y"].cuda()
    got = ts.spmv(A, c["x"].cuda(), alpha=c["alpha"], y=y, beta=c["beta"])
    assert got.is_cuda and got.shape == c["out"].shape and got.dtype == c["out"].dtype
    assert rel_fro(got, c["out"]) <= TOL32
    torch.testing.assert_close(got.cpu(), c["out"], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("index_dtype", [torch.int64, torch.int32])
@pytest.mark.parametrize("name", golden_names("spmm"))
def test_spmm_golden(name, index_dtype):
    c = golden_cases()[name]
    A = _csr(c["csr"], index_dtype)
    C = None if c["C"] is None else c["C"].cuda()
    got = ts.spmm(A, c["B"].cuda(), alpha=c["alpha"], C=C, beta=c["beta"])
    assert rel_fro(got, c["out"]) <= TOL32
    torch.testing.assert_close(got.cpu(), c["out"], atol=1e-5, rtol=1e-5)


def test_host_inputs_return_host_tensors():
    c = golden_cases()["spmv_alpha_beta"]
    A = ts.from_dense(torch.tensor([[2.0, 0.0], [0.0, 3.0]]))
    got = ts.spmv(A, torch.tensor([1.0, 1.0]), alpha=2.0, y=torch.tensor([10.0, 20.0]), beta=0.5)
    assert got.device.type == "cpu"
    assert got.tolist() == c["out"].tolist() == [9.0, 16.0]
    I = ts.eye_sparse(2)
    out = ts.spmm(I, torch.ones(2, 3), alpha=2.0, C=torch.ones(2, 3) * 10, beta=0.5)
    assert torch.all(out == 7.0)


def _random_csr(m, n, density, seed, dtype=torch.float32, long_rows=()):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(m, n, generator=g, dtype=dtype)
    A[torch.rand(m, n, generator=g) > density] = 0
    for r in long_rows:
        A[r] = torch.randn(n, generator=g, dtype=dtype)
    return A


@pytest.mark.parametrize("dtype,tol", [(torch.float32, TOL32), (torch.float64, 1e-12)])
def test_ragged_rows_and_dtypes(dtype, tol):
    # long dense rows overflow a CTA's staging buffer and exercise the warp-per-row path
    A = _random_csr(3000, 20000, 0.0004, 3, dtype, long_rows=(5, 1500, 2999))
    csr = ts.from_dense(A)
    x = torch.randn(20000, dtype=dtype)
    y = torch.randn(3000, dtype=dtype)
    ref = oracle.csr_spmv(csr.row_ptrs, csr.col_indices, csr.values, csr.shape, x, 1.5, y, -0.5)
    got = ts.spmv(csr, x.cuda(), alpha=1.5, y=y.cuda(), beta=-0.5)
    assert rel_fro(got, ref) <= tol
    B = torch.randn(20000, 12, dtype=dtype)
    ref = oracle.csr_spmm(csr.row_ptrs, csr.col_indices, csr.values, csr.shape, B)
    got = ts.spmm(csr, B.cuda())
    assert rel_fro(got, ref) <= tol


def test_misaligned_operands_take_scalar_path():
    A = _random_csr(500, 300, 0.05, 4)
    csr = ts.from_dense(A)
    # shift values/indices by one element so nothing is 16-byte aligned
    vals = torch.cat([torch.zeros(1), csr.values]).cuda()[1:]
    cols = torch.cat([torch.zeros(1, dtype=torch.long), csr.col_indices]).cuda()[1:]
    mis = ts.CSRMatrix(values=vals, col_indices=cols, row_ptrs=csr.row_ptrs.cuda(), shape=csr.shape)
    # device_layout makes contiguous copies; pass through the C ABI directly to keep the offsets
    from trnsparse_b200 import _lib

    x = torch.randn(300).cuda()
    out = torch.empty(500, device="cuda")
    rp = mis.row_ptrs
    _lib.call("trnsparse_csr_spmv", 500, 300, mis.nnz, _lib.I64, _lib.F32, rp.data_ptr(), cols.data_ptr(),
              vals.data_ptr(), x.data_ptr(), 1.0, None, 0.0, out.data_ptr(), _lib.stream_handle(out.device))
    ref = oracle.csr_spmv(csr.row_ptrs, csr.col_indices, csr.values, csr.shape, x.cpu())
    assert rel_fro(out, ref) <= TOL32
    assert vals.data_ptr() % 16 != 0


def test_empty_matrix():
    csr = ts.CSRMatrix(values=torch.zeros(0), col_indices=torch.zeros(0, dtype=torch.long),
                       row_ptrs=torch.zeros(7, dtype=torch.long), shape=(6, 4))
    y = torch.randn(6)
    got = ts.spmv(csr, torch.randn(4).cuda(), alpha=2.0, y=y.cuda(), beta=3.0)
    torch.testing.assert_close(got.cpu(), 3.0 * y)
    assert torch.count_nonzero(ts.spmm(csr, torch.randn(4, 5).cuda())) == 0


def test_errors_are_loud():
    csr = ts.eye_sparse(4)
    with pytest.raises(AssertionError):
        ts.spmv(csr, torch.randn(5).cuda())
    with pytest.raises(RuntimeError):
        ts.spmv(csr, torch.randn(4, dtype=torch.float64).cuda())


def test_config2_full_size_poisson():
    """Config 2 at full size: 2048^2-grid Poisson, int32 indices, alpha=2; spmm with k=32."""
    from trnsparse_b200 import workloads as w

    A = w.poisson2d_csr(2048)
    x = w.poisson_rhs(A.shape[0])
    ref = oracle.csr_spmv(A.row_ptrs, A.col_indices, A.values, A.shape, x, 2.0)
    got = ts.spmv(A, x.cuda(), alpha=2.0)
    assert rel_fro(got, ref) <= 1e-6
    # the stencil rows have exact small-integer weights: row sums are exact
    ones = torch.ones(A.shape[0], device="cuda")
    rs = ts.spmv(A, ones)
    exact = oracle.csr_spmv(A.row_ptrs, A.col_indices, A.values, A.shape, torch.ones(A.shape[0]))
    assert torch.equal(rs.cpu(), exact) and int((exact == 0).sum()) == (2046 * 2046)
    B = w.poisson_rhs(A.shape[0], 32)
    ref = oracle.csr_spmm(A.row_ptrs, A.col_indices, A.values, A.shape, B)
    got = ts.spmm(A, B.cuda())
    assert rel_fro(got, ref) <= 1e-6


@pytest.mark.parametrize("index_dtype", [torch.int32, torch.int64])
def test_spmv_pinned_host_pipeline(index_dtype):
    """A pinned host x on a large matrix takes the chunked pipeline (x up, row
    chunks computed as their columns arrive, rows back on a second stream):
    same values as the device-resident call, including a band matrix whose
    row chunks reach far-away columns and a row chunk with no entries."""
    from trnsparse_b200 import ops
    from trnsparse_b200 import workloads as w

    A = w.poisson2d_csr(1024, index_dtype=index_dtype)  # 1,048,576 rows
    x = w.poisson_rhs(A.shape[0])
    ref = ts.spmv(A, x.cuda(), alpha=2.0).cpu()
    got = ts.spmv(A, x.pin_memory(), alpha=2.0)
    assert not got.is_cuda and ops._SPMV_PIPE_MIN_ROWS <= A.shape[0]
    torch.testing.assert_close(got, ref, rtol=1e-6, atol=1e-6)
    # first and last columns in every row, an empty middle: every chunk waits for all of x
    n = 1 << 19
    rp = torch.zeros(n + 1, dtype=torch.int64)
    keep = torch.ones(n, dtype=torch.bool)
    keep[n // 3: n // 3 + 100000] = False
    counts = keep.long() * 2
    rp[1:] = torch.cumsum(counts, 0)
    ci = torch.stack([torch.zeros(n, dtype=torch.long), torch.full((n,), n - 1)], 1)[keep].reshape(-1)
    vals = torch.randn(ci.numel(), generator=torch.Generator().manual_seed(8))
    B = ts.CSRMatrix(values=vals, col_indices=ci.to(index_dtype), row_ptrs=rp.to(index_dtype), shape=(n, n))
    xb = torch.randn(n, generator=torch.Generator().manual_seed(9))
    torch.testing.assert_close(ts.spmv(B, xb.pin_memory()), ts.spmv(B, xb.cuda()).cpu(), rtol=1e-6, atol=1e-6)
    assert ts._lib.device_error() == 0


# ---------------------------------------------------------------- spmv_symmetric (ops.py:81-104)
@pytest.mark.parametrize("name", golden_names("spmv_symmetric"))
def test_spmv_symmetric_golden(name):
    c = golden_cases()[name]
    A = _csr(c["csr"], torch.int32)
    got = ts.spmv_symmetric(A, c["x"].cuda(), alpha=c["alpha"])
    assert got.is_cuda
    assert rel_fro(got, c["out"]) <= TOL32
    host = ts.spmv_symmetric(_csr(c["csr"], device="cpu"), c["x"], alpha=c["alpha"])
    assert host.device.type == "cpu" and rel_fro(host, c["out"]) <= TOL32


def test_spmv_symmetric_sees_in_place_updates():
    """The strict-triangle transpose caches only the structure: an in-place change
    of A.values is used by the next call (the reference rebuilds it every call)."""
    c = golden_cases()["spmv_sym_upper"]
    d = c["csr"]
    A = _csr(d, torch.int32)
    x = c["x"].cuda()
    ts.spmv_symmetric(A, x)
    A.values.mul_(-2.0)
    A.values[::7] += 1.0
    want = oracle.csr_spmv_symmetric(d["row_ptrs"], d["col_indices"], A.values.cpu(), d["shape"], c["x"])
    assert rel_fro(ts.spmv_symmetric(A, x), want) <= TOL32


def test_csr_transpose_structure_on_device():
    """trnsparse_csr_transpose gives the stable (column, row) order bit for bit."""
    from trnsparse_b200 import workloads as w
    from trnsparse_b200.ops import _transpose_structure

    A = w.poisson2d_csr(64)
    g = torch.Generator().manual_seed(3)
    D = torch.randn(300, 211, generator=g) * (torch.rand(300, 211, generator=g) < 0.05)
    D[:, 17] = 0.0
    D[40] = torch.randn(211, generator=g)
    for M, strict in ((A, False), (A, True), (ts.from_dense(D), False)):
        m, n = M.shape
        rpt, colt, perm, nnz_t = _transpose_structure(M.row_ptrs, M.col_indices, m, n, strict, {},
                                                      torch.device("cuda"))
        rows = torch.repeat_interleave(torch.arange(m), (M.row_ptrs[1:] - M.row_ptrs[:-1]).long())
        cols = M.col_indices.long()
        keep = torch.nonzero(rows != cols).squeeze(1) if strict else torch.arange(rows.numel())
        order = keep[torch.argsort(cols[keep] * m + rows[keep], stable=True)]
        want_rp = torch.zeros(n + 1, dtype=torch.long)
        want_rp[1:] = torch.cumsum(torch.bincount(cols[keep], minlength=n), 0)
        assert nnz_t == order.numel()
        assert torch.equal(perm.cpu(), order)
        assert torch.equal(colt.cpu().long(), rows[order])
        assert torch.equal(rpt.cpu().long(), want_rp)
