"""screened_spmm on the tensor cores against the reference's golden outputs
and the CPU oracle (fp32, 3xTF32: 1e-5 relative Frobenius error; fully
screened inputs must give exact zeros)."""

from __future__ import annotations

import pytest
import torch

import oracle
import trnsparse_b200 as ts
from conftest import golden_cases, golden_names, rel_fro

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", golden_names("screened_spmm"))
def test_screened_golden(name):
    c = golden_cases()[name]
    got = ts.screened_spmm(c["A"].cuda(), c["diag"].cuda(), c["B"].cuda(), c["threshold"])
    if c["out"].abs().max() == 0:
        assert torch.count_nonzero(got) == 0
    else:
        assert rel_fro(got, c["out"]) <= 1e-5
    assert ts._lib.device_error() == 0


def _fock(n, k, seed, sort=False):
    g = torch.Generator().manual_seed(seed)
    r = torch.rand(n, 3, generator=g, dtype=torch.float64) * 40.0
    if sort:
        r = r[torch.argsort(r[:, 0])]
    Q = torch.sqrt(torch.exp(-0.5 * torch.cdist(r, r) ** 2).float())
    A = Q * torch.randn(n, n, generator=g)
    B = torch.randn(n, k, generator=g)
    return A, Q, B


@pytest.mark.parametrize("n,k,sort", [(512, 96, False), (640, 256, True), (300, 40, True),
                                      # N in (256, 512]: both 256-wide N tiles in one work unit
                                      (896, 512, False), (300, 300, True)])
def test_screened_pair_bounds(n, k, sort):
    A, Q, B = _fock(n, k, seed=n, sort=sort)
    ref = oracle.screened_spmm_pair(A, Q, B, 1e-10)
    got = ts.screened_spmm(A.cuda(), Q.cuda(), B.cuda(), 1e-10)
    assert rel_fro(got, ref) <= 1e-5


def test_screened_vector_form_and_host_tensors():
    torch.manual_seed(5)
    n = 384
    A = torch.randn(n, n)
    d = torch.rand(n) ** 4  # many small bounds -> many screened pairs
    B = torch.randn(n, 64)
    ref = oracle.screened_spmm(A, d, B, 0.05)
    got = ts.screened_spmm(A, d, B, 0.05)
    assert got.device.type == "cpu" and rel_fro(got, ref) <= 1e-5


@pytest.mark.parametrize("k", [32, 400])
def test_screened_block_skip_exact_zero_rows(k):
    n = 512
    A = torch.randn(n, n)
    d = torch.ones(n)
    d[:256] = 1e-12  # rows/cols 0..255 screened against everything
    B = torch.randn(n, k)
    got = ts.screened_spmm(A.cuda(), d.cuda(), B.cuda(), 1e-6).cpu()
    assert torch.count_nonzero(got[:256]) == 0
    assert rel_fro(got, oracle.screened_spmm(A, d, B, 1e-6)) <= 1e-5


def test_screened_rejects_bad_shapes():
    with pytest.raises(AssertionError):
        ts.screened_spmm(torch.randn(4, 5).cuda(), torch.rand(4).cuda(), torch.randn(5, 2).cuda(), 0.1)


def test_config3_full_size():
    """Config 3 at full size: n=8192 Fock-like pair bounds, N=512, threshold 1e-10."""
    from trnsparse_b200 import workloads as w

    A, Q, B, diag, thr = w.fock_like()
    ref = oracle.screened_spmm_pair(A, Q, B, thr)
    got = ts.screened_spmm(A.cuda(), Q.cuda(), B.cuda(), thr)
    assert rel_fro(got, ref) <= 1e-5
    # the mask itself is bit-exact against screen_quartets
    assert int(oracle.screen_quartets(Q, thr).sum()) == int(ts.screen_quartets(Q.cuda(), thr).sum())
