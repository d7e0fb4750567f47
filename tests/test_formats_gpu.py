"""Device-side format construction (csrc/formats.cu) against the host path:
BSRMatrix.from_dense (formats.py:184-221), CSR from_dense (formats.py:269-278)
and COOMatrix.to_csr (formats.py:104-124). Structure and values bit-exact."""

from __future__ import annotations

import pytest
import torch

import oracle
import trnsparse_b200 as ts

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> torch.Tensor:
    t = t.detach().cpu().contiguous()
    return t.view({2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()])


def _block_sparse_dense(m, n, b, p_keep, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(m, n, generator=g)
    mb, nbc = -(-m // b), -(-n // b)
    keep = torch.rand(mb, nbc, generator=g) < p_keep
    mask = keep.repeat_interleave(b, 0).repeat_interleave(b, 1)[:m, :n]
    return (A * mask).to(dtype)


@pytest.mark.parametrize("m,n,b,thr,dtype", [
    (2048, 2048, 128, 0.0, torch.float32),
    (300, 517, 128, 0.0, torch.float32),
    (96, 200, 16, 0.0, torch.float32),
    (64, 64, 8, 1.5, torch.float32),
    (250, 130, 32, 0.1, torch.bfloat16),
    (256, 256, 128, -1.0, torch.float32),
])
def test_bsr_from_dense_device_matches_host(m, n, b, thr, dtype):
    A = _block_sparse_dense(m, n, b, 0.3, seed=m + n + b, dtype=dtype)
    if m >= 64:
        A[3, 5] = float("nan")      # drops its block (torch.amax propagates NaN)
        A[m - 1, n - 1] = 0.1       # compared in A's dtype
    d = ts.BSRMatrix.from_dense(A.cuda(), block_size=b, threshold=thr)
    blocks, cols, ptrs = oracle.bsr_from_dense(A, block_size=b, threshold=thr)
    assert d.blocks.is_cuda and d.block_row_ptrs.dtype == torch.int64
    assert torch.equal(d.block_row_ptrs.cpu(), ptrs)
    assert torch.equal(d.block_col_indices.cpu(), cols)
    assert d.blocks.dtype == dtype and d.blocks.shape == blocks.shape
    assert torch.equal(_bits(d.blocks), _bits(blocks))
    h = ts.BSRMatrix.from_dense(A, block_size=b, threshold=thr)  # host path, same answer
    assert torch.equal(h.block_row_ptrs, ptrs) and torch.equal(_bits(h.blocks), _bits(blocks))


def test_bsr_from_dense_device_edge_cases():
    z = ts.BSRMatrix.from_dense(torch.zeros(100, 60, device="cuda"), block_size=32)
    assert z.n_blocks == 0 and z.block_row_ptrs.tolist() == [0, 0, 0, 0, 0]
    e = ts.BSRMatrix.from_dense(torch.zeros(0, 60, device="cuda"), block_size=32)
    assert e.n_blocks == 0 and e.block_row_ptrs.tolist() == [0]
    # a transposed (non-contiguous) view
    A = _block_sparse_dense(256, 384, 128, 0.5, seed=9)
    d = ts.BSRMatrix.from_dense(A.cuda().t(), block_size=128)
    blocks, cols, ptrs = oracle.bsr_from_dense(A.t().contiguous(), block_size=128)
    assert torch.equal(d.block_row_ptrs.cpu(), ptrs) and torch.equal(d.blocks.cpu(), blocks)
    # the device-built matrix feeds the kernels directly
    B = torch.randn(256, 64, device="cuda")
    torch.testing.assert_close(ts.bsr_spmm(d, B), A.t().cuda() @ B, rtol=1e-5, atol=1e-4)
    assert ts._lib.device_error() == 0


@pytest.mark.parametrize("m,n,thr,dtype,zero_frac,offset", [
    (1000, 700, 0.0, torch.float32, 0.7, 0),
    (333, 4099, 0.5, torch.float32, 0.7, 0),
    (64, 64, 0.1, torch.bfloat16, 0.7, 0),
    (1, 100000, 1.0, torch.float32, 0.7, 0),
    # sparse results take the masked fill (the count pass's bit mask, gathered values)
    (777, 3001, 0.0, torch.float32, 0.98, 0),
    (300, 1000, 0.0, torch.bfloat16, 0.99, 0),
    (257, 999, 0.2, torch.float32, 0.98, 1),  # rows not 16-byte aligned: one element per lane
])
def test_csr_from_dense_device_matches_host(m, n, thr, dtype, zero_frac, offset):
    g = torch.Generator().manual_seed(m * 7 + n)
    A = torch.randn(m, n + offset, generator=g)
    A[torch.rand(m, n + offset, generator=g) < zero_frac] = 0.0
    A[0, 0] = float("nan")
    A[m // 2, n // 3] = float("inf")
    A[m - 1, n - 1] = 0.1
    if m > 10:
        A[5] = 0.0  # an empty row
    A = A.to(dtype)
    Ad = A.cuda()[:, offset:]
    A = A[:, offset:]
    c = ts.from_dense(Ad, threshold=thr)
    vals, cols, ptrs = oracle.csr_from_dense(A.contiguous(), threshold=thr)
    assert c.values.is_cuda and c.row_ptrs.dtype == torch.int64 and c.col_indices.dtype == torch.int64
    assert torch.equal(c.row_ptrs.cpu(), ptrs)
    assert torch.equal(c.col_indices.cpu(), cols)
    assert torch.equal(_bits(c.values), _bits(vals))
    assert ts._lib.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.bfloat16, torch.float16])
def test_coo_to_csr_device_stable_order(dtype):
    """Rows of 0, 1, 32, 33, 2048, 2049 and 5000 entries (warp sort, CTA
    sort, CTA sort + merge passes), duplicate (row, col) entries keep their
    input order."""
    g = torch.Generator().manual_seed(17)
    m, n = 40, 3000
    lens = [0, 1, 32, 33, 2048, 2049, 5000] + [int(x) for x in torch.randint(0, 50, (m - 7,), generator=g)]
    rows = torch.cat([torch.full((L,), r, dtype=torch.long) for r, L in enumerate(lens)])
    cols = torch.randint(0, n, (rows.numel(),), generator=g)
    cols[::7] = cols[0]  # many duplicates
    perm = torch.randperm(rows.numel(), generator=g)
    rows, cols = rows[perm], cols[perm]
    vals = torch.randn(rows.numel(), generator=g).to(dtype)
    coo = ts.COOMatrix(values=vals.cuda(), row_indices=rows.cuda(), col_indices=cols.cuda(), shape=(m, n))
    c = coo.to_csr()
    order = torch.argsort(rows * n + cols, stable=True)
    counts = torch.bincount(rows, minlength=m)
    ptrs = torch.zeros(m + 1, dtype=torch.long)
    ptrs[1:] = torch.cumsum(counts, 0)
    assert torch.equal(c.row_ptrs.cpu(), ptrs)
    assert torch.equal(c.col_indices.cpu(), cols[order])
    assert torch.equal(_bits(c.values), _bits(vals[order]))
    # duplicates add up in to_dense (summation order is the library's: compare with a tolerance)
    if dtype in (torch.float32, torch.float64):
        torch.testing.assert_close(c.to_dense().cpu().double(),
                                   ts.COOMatrix(vals, rows, cols, (m, n)).to_csr().to_dense().double(),
                                   rtol=1e-4, atol=1e-4)


def test_coo_to_csr_device_rejects_out_of_range():
    coo = ts.COOMatrix(values=torch.ones(3, device="cuda"), row_indices=torch.tensor([0, 5, 1], device="cuda"),
                       col_indices=torch.tensor([0, 1, 2], device="cuda"), shape=(4, 4))
    with pytest.raises(AssertionError):
        coo.to_csr()
    empty = ts.COOMatrix(values=torch.ones(0, device="cuda"), row_indices=torch.zeros(0, dtype=torch.long, device="cuda"),
                         col_indices=torch.zeros(0, dtype=torch.long, device="cuda"), shape=(3, 3))
    assert empty.to_csr().row_ptrs.tolist() == [0, 0, 0, 0]
