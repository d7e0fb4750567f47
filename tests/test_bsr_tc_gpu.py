"""Tensor-core (tcgen05) bsr_spmm against the oracle, the golden vectors and
the independent CUDA-core kernel.

Tolerances: fp32 (3xTF32) 1e-5 relative Frobenius error; bf16 operands with
fp32 accumulation 2e-2 against the fp32 oracle on the same (bf16-rounded)
inputs.
"""

from __future__ import annotations

import pytest
import torch

import oracle
import trnsparse_b200 as ts
from trnsparse_b200.ops import bsr_spmm_cuda_core
from conftest import rel_fro

pytestmark = pytest.mark.gpu


def _random_bsr(mb, nb, p, seed, b=128, dtype=torch.float32, shape=None):
    g = torch.Generator().manual_seed(seed)
    present = torch.rand(mb, nb, generator=g) < p
    present[0, 0] = True
    rows, cols = present.nonzero(as_tuple=True)
    blocks = torch.randn(rows.numel(), b, b, generator=g).to(dtype)
    ptrs = torch.zeros(mb + 1, dtype=torch.long)
    ptrs[1:] = torch.cumsum(present.sum(1), 0)
    return ts.BSRMatrix(blocks, cols.clone(), ptrs, shape or (mb * b, nb * b), b)


def _ref(A, B):
    return oracle.bsr_spmm(A.blocks.float(), A.block_col_indices, A.block_row_ptrs, A.shape, A.block_size, B.float())


def test_tc_single_block_known_product():
    A = ts.BSRMatrix(torch.eye(128).unsqueeze(0) * 2.0, torch.tensor([0]), torch.tensor([0, 1]), (128, 128), 128)
    B = torch.arange(128 * 32, dtype=torch.float32).reshape(128, 32) / 64.0
    got = ts.bsr_spmm(A, B.cuda()).cpu()
    assert torch.equal(got, 2.0 * B)  # exact: powers of two and small integers
    assert ts._lib.device_error() == 0


@pytest.mark.parametrize("k", [8, 16, 40, 64, 100, 128, 200, 256, 384, 512, 700])
def test_tc_fp32_widths(k):
    A = _random_bsr(3, 4, 0.6, seed=k)
    B = torch.randn(A.shape[1], k, generator=torch.Generator().manual_seed(100 + k))
    got = ts.bsr_spmm(A, B.cuda())
    assert rel_fro(got, _ref(A, B)) <= 1e-5
    assert ts._lib.device_error() == 0


def test_tc_unaligned_shape_and_empty_rows():
    torch.manual_seed(7)
    D = torch.randn(300, 260)
    D[128:256] = 0.0  # empty block-row 1
    A = ts.BSRMatrix.from_dense(D, block_size=128)
    B = torch.randn(260, 48)
    got = ts.bsr_spmm(A, B.cuda())
    assert rel_fro(got, D @ B) <= 1e-5
    assert torch.count_nonzero(got[128:256]) == 0


def test_tc_matches_cuda_core_scaled():
    A = _random_bsr(24, 24, 0.25, seed=3)
    B = torch.randn(A.shape[1], 256, generator=torch.Generator().manual_seed(4))
    Bd = B.cuda()
    tc = ts.bsr_spmm(A, Bd)
    cc = bsr_spmm_cuda_core(A, Bd)
    assert rel_fro(tc, cc) <= 1e-5
    assert rel_fro(tc, _ref(A, B)) <= 1e-5


def test_tc_config1():
    from trnsparse_b200 import workloads as w

    A, B = w.bsr_random_grid()
    got = ts.bsr_spmm(A, B.cuda())
    assert rel_fro(got, _ref(A, B)) <= 1e-5
    got2 = ts.bsr_spmm(A, B.cuda())  # cached split / units reused
    assert rel_fro(got, got2) <= 1e-6


@pytest.mark.parametrize("k", [64, 256, 300, 512])
def test_tc_bf16(k):
    A = _random_bsr(4, 4, 0.5, seed=11, dtype=torch.bfloat16)
    B = torch.randn(A.shape[1], k, generator=torch.Generator().manual_seed(12)).to(torch.bfloat16)
    got = ts.bsr_spmm(A, B.cuda())
    assert got.dtype == torch.bfloat16
    assert rel_fro(got.float(), _ref(A, B)) <= 2e-2
    assert ts._lib.device_error() == 0


@pytest.mark.parametrize("dtype,k", [(torch.bfloat16, 40), (torch.bfloat16, 100), (torch.bfloat16, 600),
                                     (torch.float32, 100), (torch.float32, 600)])
def test_tc_whole_row_units(dtype, k):
    """Enough busy block-rows that every unit is a whole block-row (plain TMA stores,
    bf16 C written by the epilogue for bf16 inputs): ragged m, n and k, empty rows,
    k below one 64-column box (padded B copy) and several N tiles."""
    A = _random_bsr(200, 6, 0.3, seed=k, dtype=dtype, shape=(200 * 128 - 37, 6 * 128 - 5))
    empty = (A.block_row_ptrs[1:] == A.block_row_ptrs[:-1]).nonzero().flatten().tolist()
    assert len(empty) > 0 and 200 - len(empty) >= 148
    B = torch.randn(A.shape[1], k, generator=torch.Generator().manual_seed(k)).to(dtype)
    got = ts.bsr_spmm(A, B.cuda())
    assert got.dtype == dtype and got.shape == (A.shape[0], k)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    assert rel_fro(got.float(), _ref(A, B)) <= tol
    for r in empty[:5]:
        assert torch.count_nonzero(got[r * 128:(r + 1) * 128]) == 0
    assert ts._lib.device_error() == 0
