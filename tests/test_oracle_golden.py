"""Pin the CPU oracle against the reference's own outputs (golden fixtures).

The fixtures were produced by running the reference trnsci/trnsparse v0.6.0
(tests/golden/make_golden.py). Known answers from the reference's tests are
checked literally as well.
"""

from __future__ import annotations

import pytest
import torch

import oracle
from conftest import golden_cases, golden_names


def _bsr(c):
    d = c["bsr"]
    return (d["blocks"], d["block_col_indices"], d["block_row_ptrs"], d["shape"], d["block_size"])


@pytest.mark.parametrize("name", golden_names("spmv"))
def test_spmv(name):
    c = golden_cases()[name]
    d = c["csr"]
    got = oracle.csr_spmv(d["row_ptrs"], d["col_indices"], d["values"], d["shape"], c["x"], c["alpha"], c["y"], c["beta"])
    torch.testing.assert_close(got, c["out"], atol=0, rtol=0)
    vals, cols, ptrs = oracle.csr_from_dense(c["dense"])
    assert torch.equal(vals, d["values"]) and torch.equal(cols, d["col_indices"]) and torch.equal(ptrs, d["row_ptrs"])


def test_spmv_known_answer():
    c = golden_cases()["spmv_alpha_beta"]
    assert c["out"].tolist() == [9.0, 16.0]  # reference tests/test_ops.py:25-32


@pytest.mark.parametrize("name", golden_names("spmm"))
def test_spmm(name):
    c = golden_cases()[name]
    d = c["csr"]
    got = oracle.csr_spmm(d["row_ptrs"], d["col_indices"], d["values"], d["shape"], c["B"], c["alpha"], c["C"], c["beta"])
    torch.testing.assert_close(got, c["out"], atol=0, rtol=0)


def test_spmm_known_answer():
    assert torch.all(golden_cases()["spmm_alpha_beta"]["out"] == 7.0)  # tests/test_ops.py:61-67


@pytest.mark.parametrize("name", golden_names("spmv_symmetric"))
def test_spmv_symmetric(name):
    c = golden_cases()[name]
    d = c["csr"]
    got = oracle.csr_spmv_symmetric(d["row_ptrs"], d["col_indices"], d["values"], d["shape"], c["x"], c["alpha"])
    torch.testing.assert_close(got, c["out"], atol=0, rtol=0)


def test_spmv_symmetric_known_answer():
    c = golden_cases()["spmv_sym_known"]
    assert c["out"].tolist() == [6.0, 13.0, 19.0]  # reference tests/test_ops.py:70-79 (A @ x of the full matrix)


def test_nnz_per_row_known_answer():
    c = golden_cases()["nnz_per_row"]
    _, _, ptrs = oracle.csr_from_dense(c["dense"])
    assert (ptrs[1:] - ptrs[:-1]).tolist() == c["out"].tolist() == [2, 0, 3]


@pytest.mark.parametrize("name", golden_names("bsr_spmm"))
def test_bsr(name):
    c = golden_cases()[name]
    d = c["bsr"]
    got = oracle.bsr_spmm(*_bsr(c), c["B"])
    torch.testing.assert_close(got, c["out"], atol=0, rtol=0)
    if "dense" in c:
        blocks, cols, ptrs = oracle.bsr_from_dense(c["dense"], d["block_size"], c["threshold"])
        assert torch.equal(blocks, d["blocks"]) and torch.equal(cols, d["block_col_indices"])
        assert torch.equal(ptrs, d["block_row_ptrs"])
        assert torch.equal(oracle.bsr_to_dense(*_bsr(c)), c["to_dense"])


def test_bsr_empty_is_zero():
    assert torch.count_nonzero(golden_cases()["bsr_b8_empty"]["out"]) == 0  # tests/test_bsr.py:95-101


def test_screen_known():
    c = golden_cases()["screen_known"]
    m = oracle.screen_quartets(c["Q"], c["threshold"])
    assert torch.equal(m, c["out"])
    assert m[0, 0].item() is True and m[0, 1].item() is False  # tests/test_screening.py:16-21


def test_schwarz():
    c = golden_cases()["schwarz_random"]
    Q = oracle.schwarz_bounds(c["G"])
    assert torch.equal(Q, c["Q"])
    assert torch.equal(oracle.screen_quartets(Q, c["threshold"]), c["mask"])


@pytest.mark.parametrize("name", golden_names("screened_spmm"))
def test_screened(name):
    c = golden_cases()[name]
    got = oracle.screened_spmm(c["A"], c["diag"], c["B"], c["threshold"])
    torch.testing.assert_close(got, c["out"], atol=0, rtol=0)


def test_screened_huge_threshold_is_exact_zero():
    assert torch.count_nonzero(golden_cases()["screened_huge"]["out"]) == 0


@pytest.mark.parametrize("name", golden_names("attention"))
def test_attention(name):
    c = golden_cases()[name]
    got = oracle.block_sparse_attention(c["Q"], c["K"], c["V"], c["block_row_ptrs"], c["block_col_indices"], c["block_size"])
    torch.testing.assert_close(got, c["out"], atol=0, rtol=0)


@pytest.mark.parametrize("name", golden_names("cg") + golden_names("cg_jacobi"))
def test_cg(name):
    c = golden_cases()[name]
    inv_d = oracle.jacobi_inv_diag(_bsr(c)) if c["op"] == "cg_jacobi" else None
    x, it, rel = oracle.cg_bsr(_bsr(c), c["b"], tol=c["tol"], max_iter=c["max_iter"], inv_d=inv_d)
    torch.testing.assert_close(x, c["x"], atol=0, rtol=0)
    assert it == c["iters"] and rel == c["rel"]
    if c["op"] == "cg_jacobi":
        assert torch.equal(oracle.bsr_diagonal(*_bsr(c)), c["diag"])


def test_cg_known_answers():
    z = golden_cases()["cg_zero_rhs"]
    assert z["iters"] == 0 and z["rel"] == 0.0 and torch.count_nonzero(z["x"]) == 0  # tests/test_iterative.py:80-87
    assert golden_cases()["cg_identity"]["iters"] <= 2  # tests/test_iterative.py:28-38


def test_chebyshev_coeffs():
    c = golden_cases()["cheb_coeffs"]
    a, b = oracle.chebyshev_coeffs(c["lam_min"], c["lam_max"], c["K"])
    assert torch.equal(a, c["alpha"]) and torch.equal(b, c["beta"])
    assert abs(a[0].item() - 1.0 / 50.5) < 1e-5 and abs(b[0].item()) < 1e-6  # tests/test_iterative.py:197-207


def test_chebyshev_richardson_power():
    c = golden_cases()["chebyshev"]
    x, _, rel = oracle.chebyshev_bsr(_bsr(c), c["b"], c["lam_min"], c["lam_max"], K=c["K"])
    torch.testing.assert_close(x, c["x"], atol=0, rtol=0)
    assert rel == c["rel"]
    c = golden_cases()["richardson"]
    x, _, rel = oracle.richardson_bsr(_bsr(c), c["b"], c["omega"], K=c["K"])
    torch.testing.assert_close(x, c["x"], atol=0, rtol=0)
    c = golden_cases()["power"]
    lam, v, it = oracle.power_iteration_bsr(_bsr(c), c["v0"], max_iter=c["max_iter"], tol=c["tol"])
    assert lam == c["lam"] and it == c["iters"]
    torch.testing.assert_close(v, c["v"], atol=0, rtol=0)


@pytest.mark.parametrize("name", golden_names("attention_bwd"))
def test_attention_backward(name):
    c = golden_cases()[name]
    dQ, dK, dV = oracle.block_sparse_attention_backward(c["Q"], c["K"], c["V"], c["O"], c["dO"], c["block_row_ptrs"],
                                                        c["block_col_indices"], c["block_size"])
    for got, ref in ((dQ, c["dQ"]), (dK, c["dK"]), (dV, c["dV"])):
        torch.testing.assert_close(got, ref, atol=0, rtol=0)


def test_csr_spmm_backward_golden():
    c = golden_cases()["spmm_bwd"]
    dA, dB = oracle.csr_spmm_backward(c["dense"], c["B"], c["dC"])
    torch.testing.assert_close(dA, c["dA_dense"], atol=0, rtol=0)
    torch.testing.assert_close(dB, c["dB"], atol=0, rtol=0)


def test_bsr_spmm_backward_golden():
    c = golden_cases()["bsr_bwd"]
    dblk, dB = oracle.bsr_spmm_backward(*_bsr(c), c["B"], c["dC"])
    torch.testing.assert_close(dblk, c["dblocks"], atol=0, rtol=0)
    torch.testing.assert_close(dB, c["dB"], atol=0, rtol=0)


def test_screened_spmm_backward_golden():
    c = golden_cases()["screened_bwd"]
    dA, dB = oracle.screened_spmm_backward(c["A"], c["diag"], c["B"], c["threshold"], c["dC"])
    torch.testing.assert_close(dA, c["dA"], atol=0, rtol=0)
    torch.testing.assert_close(dB, c["dB"], atol=0, rtol=0)
