"""bsr_spmm / BSR SpMV on the GPU against the oracle and the reference's golden outputs.

fp32 tolerance: 1e-5 relative Frobenius error.
"""

from __future__ import annotations

import pytest
import torch

import oracle
import trnsparse_b200 as ts
from conftest import golden_cases, golden_names, rel_fro

pytestmark = pytest.mark.gpu
TOL32 = 1e-5


def _bsr(d):
    return ts.BSRMatrix(d["blocks"], d["block_col_indices"], d["block_row_ptrs"], d["shape"], d["block_size"])


@pytest.mark.parametrize("name", golden_names("bsr_spmm"))
def test_bsr_spmm_golden(name):
    c = golden_cases()[name]
    A = _bsr(c["bsr"])
    got = ts.bsr_spmm(A, c["B"].cuda())
    assert got.shape == c["out"].shape
    if c["out"].abs().max() == 0:
        assert torch.count_nonzero(got) == 0
    else:
        assert rel_fro(got, c["out"]) <= TOL32


@pytest.mark.parametrize("name", golden_names("bsr_spmm"))
def test_bsr_matvec_golden(name):
    c = golden_cases()[name]
    d = c["bsr"]
    A = _bsr(d)
    x = c["B"][:, :1].contiguous()
    ref = oracle.bsr_spmm(d["blocks"], d["block_col_indices"], d["block_row_ptrs"], d["shape"], d["block_size"], x)
    got = ts.bsr_spmm(A, x.cuda())
    if ref.abs().max() == 0:
        assert torch.count_nonzero(got) == 0
    else:
        assert rel_fro(got, ref) <= TOL32


def test_host_in_host_out():
    c = golden_cases()["bsr_b8_unaligned"]
    got = ts.bsr_spmm(_bsr(c["bsr"]), c["B"])
    assert got.device.type == "cpu"
    assert rel_fro(got, c["out"]) <= TOL32


def test_config1_bsr_spmm_full_size():
    from trnsparse_b200 import workloads as w

    A, B = w.bsr_random_grid()
    ref = oracle.bsr_spmm(A.blocks, A.block_col_indices, A.block_row_ptrs, A.shape, A.block_size, B)
    got = ts.bsr_spmm(A, B.cuda())
    assert rel_fro(got, ref) <= TOL32


def test_config5_matvec_full_size():
    from trnsparse_b200 import workloads as w

    A, b = w.block_pentadiagonal_spd()
    # vectorised float64 check of the same product: blocks x gathered slices
    rows = A.block_rows()
    xs = b.double().view(-1, 128)[A.block_col_indices]
    y = torch.zeros(A.shape[0] // 128, 128, dtype=torch.float64)
    y.index_add_(0, rows, torch.bmm(A.blocks.double(), xs.unsqueeze(2)).squeeze(2))
    got = ts.bsr_spmm(A, b.cuda().unsqueeze(1)).squeeze(1)
    assert rel_fro(got, y.reshape(-1)) <= 1e-6
