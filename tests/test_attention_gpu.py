"""block_sparse_attention_tiled on the GPU against the reference's golden
outputs and the CPU oracle.

fp32: atol/rtol 1e-4 (the reference's own tiled-vs-naive tolerance,
tests/test_attention.py:96-148). bf16 I/O with fp32 softmax: 2e-2 relative
Frobenius error against the oracle on the fp32-upcast inputs.
"""

from __future__ import annotations

import pytest
import torch

import oracle
import trnsparse_b200 as ts
from trnsparse_b200 import workloads as w
from conftest import golden_cases, golden_names, rel_fro

pytestmark = pytest.mark.gpu


class _Mask:
    def __init__(self, rp, ci, b, seq):
        self.block_row_ptrs, self.block_col_indices, self.block_size, self.shape = rp, ci, b, (seq, seq)


@pytest.mark.parametrize("name", golden_names("attention"))
def test_attention_golden(name):
    c = golden_cases()[name]
    seq = c["Q"].shape[0]
    m = _Mask(c["block_row_ptrs"], c["block_col_indices"], c["block_size"], seq)
    got = ts.block_sparse_attention_tiled(c["Q"].cuda(), c["K"].cuda(), c["V"].cuda(), m)
    torch.testing.assert_close(got.cpu(), c["out"], atol=1e-4, rtol=1e-4)


def test_attention_host_tensors_and_bsr_mask():
    c = golden_cases()["attn_local"]
    mask = ts.BSRMatrix(torch.ones(int(c["block_row_ptrs"][-1]), 128, 128), c["block_col_indices"],
                        c["block_row_ptrs"], (256, 256), 128)
    got = ts.block_sparse_attention_tiled(c["Q"], c["K"], c["V"], mask)
    assert got.device.type == "cpu"
    torch.testing.assert_close(got, c["out"], atol=1e-4, rtol=1e-4)


def test_attention_batched_bf16_sliding_window():
    heads, seq, hd = 3, 2048, 128
    mask = w.sliding_window_mask(seq=seq)
    Q, K, V = w.attention_inputs(heads=heads, seq=seq, hd=hd, seed=3)
    got = ts.block_sparse_attention_tiled(Q.cuda(), K.cuda(), V.cuda(), mask)
    assert got.dtype == torch.bfloat16 and got.shape == Q.shape
    for h in range(heads):
        ref = oracle.block_sparse_attention(Q[0, h].float(), K[0, h].float(), V[0, h].float(),
                                            mask.block_row_ptrs, mask.block_col_indices, 128)
        assert rel_fro(got[0, h].float(), ref) <= 2e-2


def test_attention_custom_scale_and_ragged_seq():
    torch.manual_seed(0)
    seq, hd, b = 200, 48, 64  # 3 whole blocks, 8 trailing rows outside the mask
    Q, K, V = (torch.randn(seq, hd) for _ in range(3))
    rp = torch.tensor([0, 1, 3, 5])
    ci = torch.tensor([0, 0, 1, 1, 2])
    m = _Mask(rp, ci, b, seq)
    got = ts.block_sparse_attention_tiled(Q.cuda(), K.cuda(), V.cuda(), m, scale=0.3).cpu()
    ref = oracle.block_sparse_attention(Q, K, V, rp, ci, b, scale=0.3)
    torch.testing.assert_close(got, ref, atol=1e-4, rtol=1e-4)
    assert torch.count_nonzero(got[192:]) == 0


def test_attention_backward_matches_dense_autograd():
    torch.manual_seed(1)
    seq, hd, b = 256, 32, 128
    c = golden_cases()["attn_global"]
    rp, ci = torch.tensor([0, 1, 3]), torch.tensor([0, 0, 1])
    m = _Mask(rp, ci, b, seq)
    Q, K, V = (torch.randn(seq, hd, device="cuda", requires_grad=True) for _ in range(3))
    out = ts.block_sparse_attention_tiled(Q, K, V, m)
    g = torch.randn_like(out)
    out.backward(g)
    Q2, K2, V2 = (t.detach().clone().requires_grad_(True) for t in (Q, K, V))
    dense = torch.zeros(seq, seq, dtype=torch.bool, device="cuda")
    dense[:128, :128] = True
    dense[128:, :] = True
    S = (Q2 @ K2.T) * hd**-0.5
    P = torch.softmax(S.masked_fill(~dense, float("-inf")), dim=-1)
    (P @ V2).backward(g)
    for a, r in ((Q.grad, Q2.grad), (K.grad, K2.grad), (V.grad, V2.grad)):
        torch.testing.assert_close(a, r, atol=1e-4, rtol=1e-4)
    assert c is not None


@pytest.mark.parametrize("hd,heads,seq", [(128, 2, 1024), (64, 3, 768), (128, 1, 128)])
def test_attention_tensor_core_vs_cuda_core_and_oracle(hd, heads, seq):
    from trnsparse_b200.ops import _attn_forward

    mask = w.sliding_window_mask(seq=seq, window=3, n_global=1)
    Q, K, V = w.attention_inputs(heads=heads, seq=seq, hd=hd, seed=hd + seq)
    Qd, Kd, Vd = Q.cuda(), K.cuda(), V.cuda()
    tc = _attn_forward(Qd, Kd, Vd, mask, hd**-0.5)
    cc = _attn_forward(Qd, Kd, Vd, mask, hd**-0.5, cuda_cores=True)
    assert ts._lib.device_error() == 0
    assert rel_fro(tc.float(), cc.float()) <= 2e-2
    for h in range(heads):
        ref = oracle.block_sparse_attention(Q[0, h].float(), K[0, h].float(), V[0, h].float(),
                                            mask.block_row_ptrs, mask.block_col_indices, 128)
        assert rel_fro(tc[0, h].float(), ref) <= 2e-2


def test_attention_tensor_core_empty_block_row():
    seq, hd = 384, 128
    rp = torch.tensor([0, 1, 1, 3])  # block-row 1 empty
    ci = torch.tensor([0, 0, 2])
    m = _Mask(rp, ci, 128, seq)
    Q, K, V = w.attention_inputs(heads=2, seq=seq, hd=hd, seed=9)
    got = ts.block_sparse_attention_tiled(Q.cuda(), K.cuda(), V.cuda(), m).cpu()
    assert torch.count_nonzero(got[0, :, 128:256]) == 0
    for h in range(2):
        ref = oracle.block_sparse_attention(Q[0, h].float(), K[0, h].float(), V[0, h].float(), rp, ci, 128)
        assert rel_fro(got[0, h].float(), ref) <= 2e-2


@pytest.mark.parametrize("scale", [0.9, -0.7])
def test_attention_tensor_core_moving_max(scale):
    """Key blocks of growing magnitude move the running row max on many steps,
    so the in-TMEM rescale of the output runs; a negative scale flips the
    max/min roles."""
    from trnsparse_b200.ops import _attn_forward

    seq, hd = 1024, 64
    mask = w.sliding_window_mask(seq=seq, window=5, n_global=1)
    Q, K, V = w.attention_inputs(heads=2, seq=seq, hd=hd, seed=21)
    gain = torch.repeat_interleave(torch.linspace(0.1, 3.0, seq // 128), 128).view(1, 1, seq, 1)
    K = (K.float() * gain).to(torch.bfloat16)
    tc = _attn_forward(Q.cuda(), K.cuda(), V.cuda(), mask, scale)
    assert ts._lib.device_error() == 0
    for h in range(2):
        ref = oracle.block_sparse_attention(Q[0, h].float(), K[0, h].float(), V[0, h].float(),
                                            mask.block_row_ptrs, mask.block_col_indices, 128, scale=scale)
        assert rel_fro(tc[0, h].float().cpu(), ref) <= 2e-2


@pytest.mark.parametrize("name", golden_names("attention_bwd"))
def test_attention_backward_golden(name):
    """Backward kernels (stats, dQ row-first, dK/dV column-first) against the
    reference's _block_sparse_attn_backward outputs (fp32, 1e-4)."""
    c = golden_cases()[name]
    m = _Mask(c["block_row_ptrs"], c["block_col_indices"], c["block_size"], c["Q"].shape[0])
    Q, K, V = (c[k].cuda().requires_grad_(True) for k in ("Q", "K", "V"))
    out = ts.block_sparse_attention_tiled(Q, K, V, m)
    out.backward(c["dO"].cuda())
    for got, ref in ((Q.grad, c["dQ"]), (K.grad, c["dK"]), (V.grad, c["dV"])):
        torch.testing.assert_close(got.cpu(), ref, atol=1e-4, rtol=1e-4)
    assert ts._lib.device_error() == 0


def test_attention_backward_bf16_heads_and_ragged():
    """bf16 with leading head dimensions (2e-2 relative Frobenius against the
    fp32 oracle on the same bf16 inputs), and an fp32 ragged case (seq not a
    multiple of the block: the trailing rows get zero gradient)."""
    seq, hd = 512, 128
    mask = w.sliding_window_mask(seq=seq, window=2, n_global=1)
    Q, K, V = w.attention_inputs(heads=2, seq=seq, hd=hd, seed=40)
    dO = torch.randn(1, 2, seq, hd, generator=torch.Generator().manual_seed(41)).to(torch.bfloat16)
    Qd, Kd, Vd = (t.cuda().requires_grad_(True) for t in (Q, K, V))
    ts.block_sparse_attention_tiled(Qd, Kd, Vd, mask).backward(dO.cuda())
    for h in range(2):
        args = [t[0, h].float() for t in (Q, K, V)]
        O = oracle.block_sparse_attention(*args, mask.block_row_ptrs, mask.block_col_indices, 128)
        refs = oracle.block_sparse_attention_backward(*args, O, dO[0, h].float(), mask.block_row_ptrs,
                                                      mask.block_col_indices, 128)
        for got, ref in zip((Qd.grad, Kd.grad, Vd.grad), refs):
            assert got.dtype == torch.bfloat16
            assert rel_fro(got[0, h].float(), ref) <= 2e-2
    # ragged fp32
    torch.manual_seed(3)
    seq, hd, b = 200, 48, 64
    rp, ci = torch.tensor([0, 1, 3, 5]), torch.tensor([0, 0, 1, 1, 2])
    m = _Mask(rp, ci, b, seq)
    Q, K, V, dO = (torch.randn(seq, hd) for _ in range(4))
    Qd, Kd, Vd = (t.cuda().requires_grad_(True) for t in (Q, K, V))
    ts.block_sparse_attention_tiled(Qd, Kd, Vd, m, scale=0.3).backward(dO.cuda())
    O = oracle.block_sparse_attention(Q, K, V, rp, ci, b, scale=0.3)
    refs = oracle.block_sparse_attention_backward(Q, K, V, O, dO, rp, ci, b, scale=0.3)
    for got, ref in zip((Qd.grad, Kd.grad, Vd.grad), refs):
        torch.testing.assert_close(got.cpu(), ref, atol=1e-4, rtol=1e-4)
    assert torch.count_nonzero(Qd.grad[192:]) == 0
    assert ts._lib.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_attention_backward_split_global_columns(dtype):
    """A key block stored by more than 8 query blocks (a global-token column
    of a 21-block mask) is split over several dK/dV CTAs that add into fp32
    accumulators; checked against the fp32 oracle (1e-4 for fp32, 2e-2
    relative Frobenius for bf16)."""
    seq, hd, b = 21 * 64, 64, 64
    mask = w.sliding_window_mask(seq=seq, b=b, window=2, n_global=1)
    g = torch.Generator().manual_seed(77)
    Q, K, V, dO = (torch.randn(seq, hd, generator=g).to(dtype) for _ in range(4))
    Qd, Kd, Vd = (t.cuda().requires_grad_(True) for t in (Q, K, V))
    ts.block_sparse_attention_tiled(Qd, Kd, Vd, mask).backward(dO.cuda())
    args = [t.float() for t in (Q, K, V)]
    O = oracle.block_sparse_attention(*args, mask.block_row_ptrs, mask.block_col_indices, b)
    refs = oracle.block_sparse_attention_backward(*args, O, dO.float(), mask.block_row_ptrs,
                                                  mask.block_col_indices, b)
    for got, ref in zip((Qd.grad, Kd.grad, Vd.grad), refs):
        assert got.dtype == dtype
        if dtype == torch.float32:
            torch.testing.assert_close(got.cpu(), ref, atol=1e-4, rtol=1e-4)
        else:
            assert rel_fro(got.float().cpu(), ref) <= 2e-2
    assert ts._lib.device_error() == 0


def _tc_backward_case(hd, heads, seq, rp, ci, seed):
    g = torch.Generator().manual_seed(seed)
    Q, K, V, dO = (torch.randn(1, heads, seq, hd, generator=g).to(torch.bfloat16) for _ in range(4))
    m = _Mask(rp, ci, 128, seq)
    return m, Q, K, V, dO


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("split", [16, 3])
def test_attention_backward_tensor_core_vs_oracle(hd, split, monkeypatch):
    """tcgen05 backward (bf16, block 128) against the fp32 oracle on the same
    bf16 inputs, 2e-2 relative Frobenius: global-token columns stored by more
    query blocks than `split` (partial sums through fp32 slots), an empty
    block-row (zero dQ) and a key block no query block stores (zero dK, dV)."""
    from trnsparse_b200 import ops

    monkeypatch.setattr(ops, "_ATTN_BWD_SPLIT", split)
    seq, heads = 128 * 20, 2
    mt = seq // 128
    keep = torch.zeros(mt, mt, dtype=torch.bool)
    for i in range(mt):
        for j in range(mt):
            keep[i, j] = j <= i and (i - j < 3 or j < 2)
    keep[5, :] = False      # empty block-row
    keep[:, 7] = False      # key block stored by no query block
    rows, cols = keep.nonzero(as_tuple=True)
    rp = torch.zeros(mt + 1, dtype=torch.int64)
    rp[1:] = torch.cumsum(torch.bincount(rows, minlength=mt), 0)
    m, Q, K, V, dO = _tc_backward_case(hd, heads, seq, rp, cols, 90 + hd)
    Qd, Kd, Vd = (t.cuda().requires_grad_(True) for t in (Q, K, V))
    ts.block_sparse_attention_tiled(Qd, Kd, Vd, m).backward(dO.cuda())
    assert ts._lib.device_error() == 0
    for h in range(heads):
        args = [t[0, h].float() for t in (Q, K, V)]
        O = oracle.block_sparse_attention(*args, rp, cols, 128)
        refs = oracle.block_sparse_attention_backward(*args, O, dO[0, h].float(), rp, cols, 128)
        for got, ref in zip((Qd.grad, Kd.grad, Vd.grad), refs):
            assert got.dtype == torch.bfloat16
            assert rel_fro(got[0, h].float(), ref) <= 2e-2
    assert torch.count_nonzero(Qd.grad[0, :, 5 * 128:6 * 128]) == 0
    assert torch.count_nonzero(Kd.grad[0, :, 7 * 128:8 * 128]) == 0
    assert torch.count_nonzero(Vd.grad[0, :, 7 * 128:8 * 128]) == 0


def test_attention_backward_tensor_core_lse_and_cuda_core_agree():
    """The tensor-core backward with the forward's saved log-sum-exp, with the
    log-sum-exp recomputed (lse=None) and the CUDA-core backward agree
    (bf16 outputs, 1e-2 relative Frobenius)."""
    from trnsparse_b200 import ops

    seq, hd = 128 * 12, 128
    mask = w.sliding_window_mask(seq=seq, window=4, n_global=1)
    Q, K, V = (t.cuda() for t in w.attention_inputs(heads=3, seq=seq, hd=hd, seed=61))
    dO = torch.randn(Q.shape, generator=torch.Generator().manual_seed(62)).to(torch.bfloat16).cuda()
    scale = 0.11
    O, lse = ops._attn_forward(Q, K, V, mask, scale, want_lse=True)
    assert lse is not None and lse.shape == (3 * seq,)
    a = ops._attn_backward(Q, K, V, O, dO, mask, scale, lse=lse)
    b = ops._attn_backward(Q, K, V, O, dO, mask, scale, lse=None)
    c = ops._attn_backward(Q, K, V, O, dO, mask, scale, cuda_cores=True)
    assert ts._lib.device_error() == 0
    for x, y, z in zip(a, b, c):
        assert rel_fro(x.float(), y.float()) <= 1e-2
        assert rel_fro(x.float(), z.float()) <= 1e-2


def test_attention_config4_full_size():
    """The benchmarked shape (config 4: 16 heads x seq 16384 x head_dim 128, bf16,
    causal window of 8 blocks plus 2 global blocks, 1,235 blocks per head):
    forward heads 0 and 15 and the backward (dQ, dK, dV) of head 15 against the
    fp32 oracle on the fp32-upcast inputs, 2e-2 relative Frobenius. The
    backward splits each global column's 128 partner query blocks into 8
    units, as the bench runs it."""
    mask = w.sliding_window_mask()
    assert mask.n_blocks == 1235 and mask.shape == (16384, 16384)
    Q, K, V = w.attention_inputs()
    assert Q.shape == (1, 16, 16384, 128) and Q.dtype == torch.bfloat16
    dO = torch.randn(Q.shape, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    Qd, Kd, Vd = (t.cuda().requires_grad_(True) for t in (Q, K, V))
    out = ts.block_sparse_attention_tiled(Qd, Kd, Vd, mask)
    out.backward(dO.cuda())
    assert ts._lib.device_error() == 0
    rp, ci = mask.block_row_ptrs, mask.block_col_indices
    for h in (0, 15):
        args = [t[0, h].float() for t in (Q, K, V)]
        O = oracle.block_sparse_attention(*args, rp, ci, 128)
        assert rel_fro(out[0, h].detach().float(), O) <= 2e-2, h
        if h == 15:
            refs = oracle.block_sparse_attention_backward(*args, O, dO[0, h].float(), rp, ci, 128)
            for name, got, ref in zip("QKV", (Qd.grad, Kd.grad, Vd.grad), refs):
                assert rel_fro(got[0, h].float(), ref) <= 2e-2, name
