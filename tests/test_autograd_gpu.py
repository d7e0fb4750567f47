"""Gradients of the sparse products against dense PyTorch autograd on the
same inputs (fp32: 1e-5 relative Frobenius error on each gradient).

The reference's CPU path builds its products from differentiable torch ops,
so gradients reach the dense operands and the stored values; the device
implementation provides the same through autograd Functions whose backward
runs the device kernels on the transposed operand."""

from __future__ import annotations

import pytest
import torch

import trnsparse_b200 as ts
from conftest import rel_fro

pytestmark = pytest.mark.gpu


def _csr(seed, m=300, n=260, density=0.05):
    g = torch.Generator().manual_seed(seed)
    D = torch.randn(m, n, generator=g) * (torch.rand(m, n, generator=g) < density)
    return D, ts.from_dense(D)


@pytest.mark.parametrize("k", [0, 1, 24])
def test_csr_product_gradients(k):
    D, A = _csr(1)
    g = torch.Generator().manual_seed(2)
    X = torch.randn(D.shape[1], k, generator=g) if k else torch.randn(D.shape[1], generator=g)
    Y = torch.randn(D.shape[0], k, generator=g) if k else torch.randn(D.shape[0], generator=g)
    Xd, Yd = X.cuda().requires_grad_(True), Y.cuda().requires_grad_(True)
    A.values = A.values.clone().requires_grad_(True)
    out = ts.spmm(A, Xd, alpha=1.5, C=Yd, beta=0.5) if k else ts.spmv(A, Xd, alpha=1.5, y=Yd, beta=0.5)
    G = torch.randn(out.shape, generator=g).cuda()
    out.backward(G)
    # dense reference with the same pattern
    Dd = D.cuda().requires_grad_(True)
    X2, Y2 = X.cuda().requires_grad_(True), Y.cuda().requires_grad_(True)
    ref = 1.5 * (Dd @ X2) + 0.5 * Y2
    ref.backward(G)
    assert rel_fro(out, ref) <= 1e-5
    assert rel_fro(Xd.grad, X2.grad) <= 1e-5 and rel_fro(Yd.grad, Y2.grad) <= 1e-6
    rows = torch.repeat_interleave(torch.arange(D.shape[0]), A.row_ptrs[1:] - A.row_ptrs[:-1])
    assert rel_fro(A.values.grad, Dd.grad.cpu()[rows, A.col_indices.long()]) <= 1e-5


@pytest.mark.parametrize("b,k", [(128, 48), (32, 16)])
def test_bsr_spmm_gradients(b, k):
    g = torch.Generator().manual_seed(5)
    D = torch.randn(3 * b + 17, 2 * b + 5, generator=g)
    D[b : 2 * b] = 0.0  # an empty block-row
    A = ts.BSRMatrix.from_dense(D, block_size=b)
    A.blocks = A.blocks.clone().requires_grad_(True)
    B = torch.randn(D.shape[1], k, generator=g).cuda().requires_grad_(True)
    out = ts.bsr_spmm(A, B)
    G = torch.randn(out.shape, generator=g).cuda()
    out.backward(G)
    Dd = D.cuda().requires_grad_(True)
    B2 = B.detach().clone().requires_grad_(True)
    ref = Dd @ B2
    ref.backward(G)
    assert rel_fro(out, ref) <= 1e-5
    assert rel_fro(B.grad, B2.grad) <= 1e-5
    # block gradients are the dense gradient restricted to each stored block
    rp, ci = A.block_row_ptrs.tolist(), A.block_col_indices.tolist()
    dD = torch.zeros((len(rp) - 1) * b, -(-D.shape[1] // b) * b)
    dD[: D.shape[0], : D.shape[1]] = Dd.grad.cpu()
    want = torch.stack([dD[i * b:(i + 1) * b, ci[kk] * b:(ci[kk] + 1) * b]
                        for i in range(len(rp) - 1) for kk in range(rp[i], rp[i + 1])])
    assert rel_fro(A.blocks.grad, want) <= 1e-5


@pytest.mark.parametrize("kind", [1, 2])
def test_screened_spmm_gradients(kind):
    g = torch.Generator().manual_seed(7)
    n, k = 256, 40
    r = torch.rand(n, 3, generator=g) * 6.0
    G2 = torch.exp(-0.5 * torch.cdist(r, r) ** 2)
    Q = ts.schwarz_bounds(G2) if kind == 2 else torch.diagonal(G2).clone() * torch.rand(n, generator=g)
    thr = 1e-3
    A = (torch.randn(n, n, generator=g)).cuda().requires_grad_(True)
    B = torch.randn(n, k, generator=g).cuda().requires_grad_(True)
    out = ts.screened_spmm(A, Q.cuda(), B, thr)
    Gr = torch.randn(out.shape, generator=g).cuda()
    out.backward(Gr)
    t = float(torch.tensor(thr ** 0.5, dtype=torch.float32))
    if kind == 1:
        q = torch.sqrt(torch.abs(Q.cuda()))
        mask = (q.unsqueeze(1) * q.unsqueeze(0) > t).float()
    else:
        mask = (Q.cuda() > t).float()
    A2, B2 = A.detach().clone().requires_grad_(True), B.detach().clone().requires_grad_(True)
    ref = (A2 * mask) @ B2
    ref.backward(Gr)
    assert rel_fro(out, ref) <= 1e-5
    assert rel_fro(A.grad, A2.grad) <= 1e-5 and rel_fro(B.grad, B2.grad) <= 1e-5


# ---------------------------------------------------------------- against the reference's own backward
def test_spmm_gradients_golden():
    """Golden vectors from the reference's _SpMMFunction.backward (nki/dispatch.py:154-178)."""
    from conftest import golden_cases

    c = golden_cases()["spmm_bwd"]
    d = c["csr"]
    A = ts.CSRMatrix(values=d["values"].clone().requires_grad_(True), col_indices=d["col_indices"],
                     row_ptrs=d["row_ptrs"], shape=d["shape"])
    B = c["B"].cuda().requires_grad_(True)
    ts.spmm(A, B).backward(c["dC"].cuda())
    rows = torch.repeat_interleave(torch.arange(d["shape"][0]), d["row_ptrs"][1:] - d["row_ptrs"][:-1])
    assert rel_fro(A.values.grad, c["dA_dense"][rows, d["col_indices"]]) <= 1e-5
    assert rel_fro(B.grad, c["dB"]) <= 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_bsr_spmm_gradients_golden(dtype):
    """Golden vectors from the reference's _BSRSpMMFunction.backward (nki/dispatch.py:331-369):
    fp32 within 1e-5, bf16 operands within 2e-2."""
    from conftest import golden_cases

    c = golden_cases()["bsr_bwd"]
    d = c["bsr"]
    A = ts.BSRMatrix(blocks=d["blocks"].to(dtype).cuda().requires_grad_(True),
                     block_col_indices=d["block_col_indices"], block_row_ptrs=d["block_row_ptrs"],
                     shape=d["shape"], block_size=d["block_size"])
    B = c["B"].to(dtype).cuda().requires_grad_(True)
    ts.bsr_spmm(A, B).backward(c["dC"].to(dtype).cuda())
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    assert rel_fro(A.blocks.grad, c["dblocks"]) <= tol
    assert rel_fro(B.grad, c["dB"]) <= tol


def test_screened_spmm_gradients_golden():
    """Golden vectors from the reference's _ScreenedSpMMFunction.backward (nki/dispatch.py:447-484)."""
    from conftest import golden_cases

    c = golden_cases()["screened_bwd"]
    A = c["A"].cuda().requires_grad_(True)
    B = c["B"].cuda().requires_grad_(True)
    ts.screened_spmm(A, c["diag"].cuda(), B, c["threshold"]).backward(c["dC"].cuda())
    assert rel_fro(A.grad, c["dA"]) <= 1e-5
    assert rel_fro(B.grad, c["dB"]) <= 1e-5


def test_bsr_transpose_cache_has_one_slot():
    """In-place updates of A.blocks (an optimizer step) replace the cached transpose
    instead of adding a copy per step, and the gradient follows the new values."""
    import oracle

    g = torch.Generator().manual_seed(9)
    D = torch.randn(256, 256, generator=g)
    A = ts.BSRMatrix.from_dense(D, block_size=128)
    A.blocks = A.blocks.cuda().requires_grad_(True)
    B = torch.randn(256, 8, generator=g).cuda().requires_grad_(True)
    for step in range(3):
        B.grad = None
        dC = torch.randn(256, 8, generator=g).cuda()
        ts.bsr_spmm(A, B).backward(dC)
        blk = A.blocks.detach().cpu()
        _, dB = oracle.bsr_spmm_backward(blk, A.block_col_indices, A.block_row_ptrs, A.shape, 128,
                                         B.detach().cpu(), dC.cpu())
        assert rel_fro(B.grad, dB) <= 1e-5, step
        with torch.no_grad():
            A.blocks.mul_(0.5)
        assert sum(1 for k in A._dev if isinstance(k, tuple) and k[0] == "bsr_transpose") == 1
