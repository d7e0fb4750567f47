"""Generate tests/golden/golden.pt by running the reference trnsci/trnsparse.

Run in the build container, where the reference source tree is importable:

    TRNSPARSE_REF=<path to the reference checkout> python tests/golden/make_golden.py

Every case stores its seeded inputs and the reference's own outputs (its
PyTorch CPU path: `nki` is absent, so HAS_NKI is False). The fixtures pin the
CPU oracle in ``oracle/`` and are the golden vectors the GPU parity tests
compare against. Sizes are kept small so the file stays a few MB.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import torch

REF = os.environ.get("TRNSPARSE_REF")
if not REF:
    sys.exit("set TRNSPARSE_REF to the reference checkout")
sys.path.insert(0, REF)
sys.path.insert(0, str(Path(REF) / "examples"))
import trnsparse  # noqa: E402
import block_sparse_attention as attn_demo  # noqa: E402

assert not trnsparse.HAS_NKI

OUT = Path(__file__).resolve().parent / "golden.pt"
cases: dict[str, dict] = {}


def csr_dict(c):
    return {"values": c.values, "col_indices": c.col_indices, "row_ptrs": c.row_ptrs, "shape": tuple(c.shape)}


def bsr_dict(b):
    return {
        "blocks": b.blocks,
        "block_col_indices": b.block_col_indices,
        "block_row_ptrs": b.block_row_ptrs,
        "shape": tuple(b.shape),
        "block_size": b.block_size,
    }


# ---------------------------------------------------------------- CSR formats + spmv/spmm
def add_spmv(name, A, x, alpha=1.0, y=None, beta=0.0):
    csr = trnsparse.from_dense(A)
    out = trnsparse.spmv(csr, x, alpha=alpha, y=y, beta=beta)
    cases[name] = {"op": "spmv", "dense": A, "csr": csr_dict(csr), "x": x, "alpha": alpha, "y": y, "beta": beta, "out": out}


def add_spmm(name, A, B, alpha=1.0, C=None, beta=0.0):
    csr = trnsparse.from_dense(A)
    out = trnsparse.spmm(csr, B, alpha=alpha, C=C, beta=beta)
    cases[name] = {"op": "spmm", "dense": A, "csr": csr_dict(csr), "B": B, "alpha": alpha, "C": C, "beta": beta, "out": out}


add_spmv("spmv_identity", torch.eye(4), torch.tensor([1.0, 2.0, 3.0, 4.0]))
add_spmv("spmv_alpha_beta", torch.tensor([[2.0, 0.0], [0.0, 3.0]]), torch.tensor([1.0, 1.0]), 2.0,
         torch.tensor([10.0, 20.0]), 0.5)
torch.manual_seed(42)
A = torch.randn(100, 100)
A[torch.abs(A) < 1.5] = 0.0
add_spmv("spmv_large_sparse", A, torch.randn(100))
torch.manual_seed(11)
A = torch.randn(300, 257)
A[torch.rand(300, 257) > 0.03] = 0.0
A[17] = 0.0  # an empty row
A[200, :] = torch.randn(257)  # a dense row
add_spmv("spmv_ragged_ab", A, torch.randn(257), -1.5, torch.randn(300), 0.25)
add_spmm("spmm_alpha_beta", torch.eye(2), torch.ones(2, 3), 2.0, torch.ones(2, 3) * 10, 0.5)
torch.manual_seed(12)
A = torch.randn(200, 137)
A[torch.rand(200, 137) > 0.05] = 0.0
add_spmm("spmm_unaligned", A, torch.randn(137, 64))
torch.manual_seed(13)
A = torch.randn(150, 90)
A[torch.rand(150, 90) > 0.1] = 0.0
add_spmm("spmm_odd_cols_ab", A, torch.randn(90, 7), 0.75, torch.randn(150, 7), -2.0)
A = torch.tensor([[1.0, 0.0, 2.0], [0.0, 0.0, 0.0], [3.0, 4.0, 5.0]])
cases["nnz_per_row"] = {"op": "nnz_per_row", "dense": A, "out": trnsparse.nnz_per_row(trnsparse.from_dense(A))}


# spmv_symmetric: one stored triangle of a symmetric matrix (ops.py:81-104)
def add_spmv_sym(name, A, x, alpha=1.0):
    csr = trnsparse.from_dense(A)
    out = trnsparse.spmv_symmetric(csr, x, alpha=alpha, uplo="upper")
    cases[name] = {"op": "spmv_symmetric", "dense": A, "csr": csr_dict(csr), "x": x, "alpha": alpha, "out": out}


Ak = torch.tensor([[4.0, 1.0, 0.0], [1.0, 3.0, 2.0], [0.0, 2.0, 5.0]])
add_spmv_sym("spmv_sym_known", torch.triu(Ak), torch.tensor([1.0, 2.0, 3.0]))
torch.manual_seed(21)
S = torch.randn(257, 257)
S[torch.rand(257, 257) > 0.04] = 0.0
S = torch.triu(S + S.t())
S[31] = 0.0  # an empty row
S[100, 100] = 0.0  # a row without its diagonal entry
add_spmv_sym("spmv_sym_upper", S, torch.randn(257))
add_spmv_sym("spmv_sym_alpha", S, torch.randn(257), alpha=-0.75)

# ---------------------------------------------------------------- BSR
def block_random(mb, nb, b, dens, seed):
    torch.manual_seed(seed)
    A = torch.zeros(mb * b, nb * b)
    mask = torch.rand(mb, nb) < dens
    for i in range(mb):
        for j in range(nb):
            if mask[i, j]:
                A[i * b : (i + 1) * b, j * b : (j + 1) * b] = torch.randn(b, b)
    return A


def add_bsr(name, A, b, B, threshold=0.0):
    bsr = trnsparse.BSRMatrix.from_dense(A, block_size=b, threshold=threshold)
    out = trnsparse.bsr_spmm(bsr, B)
    case = {"op": "bsr_spmm", "bsr": bsr_dict(bsr), "B": B, "threshold": threshold, "out": out}
    if b < 128:  # small cases also pin the format round trip
        case.update(dense=A, to_dense=bsr.to_dense())
    cases[name] = case


add_bsr("bsr_b8_vs_dense", block_random(3, 3, 8, 0.5, 5), 8, torch.randn(24, 16))
torch.manual_seed(6)
add_bsr("bsr_b8_unaligned", torch.randn(20, 14), 8, torch.randn(14, 10))
add_bsr("bsr_b8_sparse", block_random(5, 5, 8, 0.1, 7), 8, torch.randn(40, 12))
add_bsr("bsr_b8_empty", torch.zeros(16, 16), 8, torch.randn(16, 8))
torch.manual_seed(42)
add_bsr("bsr_b128_2x3", block_random(2, 3, 128, 0.5, 42), 128, torch.randn(384, 64))
torch.manual_seed(43)
A = block_random(3, 2, 128, 0.7, 43)
A[:, 5] *= 1e-3
add_bsr("bsr_b128_threshold", A, 128, torch.randn(256, 40), threshold=0.5)

# ---------------------------------------------------------------- screening / screened_spmm
Qk = torch.tensor([[1.0, 0.5], [0.5, 1.0]])
cases["screen_known"] = {"op": "screen_quartets", "Q": Qk, "threshold": 0.3, "out": trnsparse.screen_quartets(Qk, 0.3)}
torch.manual_seed(5)
Gd = torch.rand(40, 40) * 1e-3
cases["schwarz_random"] = {"op": "schwarz", "G": Gd, "Q": trnsparse.schwarz_bounds(Gd),
                           "mask": trnsparse.screen_quartets(trnsparse.schwarz_bounds(Gd), 1e-4), "threshold": 1e-4}


def add_screened(name, n, N, thr, seed, diag_scale=1.0, shift=0.0):
    torch.manual_seed(seed)
    A = torch.randn(n, n)
    diag = torch.abs(torch.randn(n)) * diag_scale + shift
    B = torch.randn(n, N)
    out = trnsparse.screened_spmm(A, diag, B, threshold=thr)
    cases[name] = {"op": "screened_spmm", "A": A, "diag": diag, "B": B, "threshold": thr, "out": out}


add_screened("screened_thr0", 64, 16, 0.0, 0, shift=0.1)
add_screened("screened_huge", 64, 16, 1e30, 1)
add_screened("screened_parity", 64, 16, 0.5, 2, diag_scale=4.0)
add_screened("screened_256", 256, 96, 0.5, 3, diag_scale=2.0)

# ---------------------------------------------------------------- attention (fp32)
def add_attn(name, seq, hd, b, mask, seed=10):
    torch.manual_seed(seed)
    Q, K, V = torch.randn(seq, hd), torch.randn(seq, hd), torch.randn(seq, hd)
    mb = trnsparse.BSRMatrix.from_dense(mask.float(), block_size=b)
    out = trnsparse.block_sparse_attention_tiled(Q, K, V, mb)
    naive = attn_demo.block_sparse_attention(Q, K, V, mb)
    cases[name] = {"op": "attention", "Q": Q, "K": K, "V": V, "block_row_ptrs": mb.block_row_ptrs,
                   "block_col_indices": mb.block_col_indices, "block_size": b, "out": out,
                   "naive_maxdiff": float((out - naive).abs().max())}


add_attn("attn_local", 256, 32, 128, attn_demo._local_window_mask(256, 128, 1))
add_attn("attn_dilated", 256, 32, 128, attn_demo._dilated_mask(256, 128, 2))
add_attn("attn_global", 384, 32, 128, attn_demo._global_token_mask(384, 128, 1, 1))
add_attn("attn_hd256", 256, 256, 128, attn_demo._local_window_mask(256, 128, 1))
add_attn("attn_hd128_causal", 384, 128, 128, torch.tril(torch.ones(384, 384, dtype=torch.bool)), seed=14)
m = torch.zeros(384, 384, dtype=torch.bool)
m[:128, :128] = True
m[256:, 128:] = True  # block-row 1 is empty -> zero output rows
add_attn("attn_empty_row", 384, 64, 128, m, seed=15)

# ---------------------------------------------------------------- attention backward (fp32)
from trnsparse.ops import _block_sparse_attn_backward  # noqa: E402


def add_attn_bwd(name, seq, hd, b, mask, seed):
    torch.manual_seed(seed)
    Q, K, V, dO = (torch.randn(seq, hd) for _ in range(4))
    mb = trnsparse.BSRMatrix.from_dense(mask.float(), block_size=b)
    O = trnsparse.block_sparse_attention_tiled(Q, K, V, mb)
    dQ, dK, dV = _block_sparse_attn_backward(Q, K, V, O, dO, mb, hd**-0.5)
    cases[name] = {"op": "attention_bwd", "Q": Q, "K": K, "V": V, "O": O, "dO": dO,
                   "block_row_ptrs": mb.block_row_ptrs, "block_col_indices": mb.block_col_indices,
                   "block_size": b, "dQ": dQ, "dK": dK, "dV": dV}


add_attn_bwd("attn_bwd_local", 256, 32, 128, attn_demo._local_window_mask(256, 128, 1), seed=31)
add_attn_bwd("attn_bwd_global", 384, 64, 128, attn_demo._global_token_mask(384, 128, 1, 1), seed=32)
add_attn_bwd("attn_bwd_empty_row", 384, 32, 128, m, seed=33)

# ---------------------------------------------------------------- solvers
def spd(n, b, seed):
    torch.manual_seed(seed)
    M = torch.randn(n, n)
    Ad = M @ M.T + n * torch.eye(n)
    return Ad, trnsparse.BSRMatrix.from_dense(Ad, block_size=b)


Ad, Ab = spd(128, 128, 1)
torch.manual_seed(21)
b = torch.randn(128)
x, it, rel = trnsparse.cg_bsr(Ab, b, tol=1e-8, max_iter=256)
cases["cg_spd128"] = {"op": "cg", "bsr": bsr_dict(Ab), "b": b, "tol": 1e-8, "max_iter": 256, "x": x, "iters": it, "rel": rel}
Ad, Ab = spd(256, 64, 2)
torch.manual_seed(22)
b = torch.randn(256)
Mj = trnsparse.jacobi_preconditioner_bsr(Ab)
x, it, rel = trnsparse.cg_bsr(Ab, b, tol=1e-7, max_iter=100, M=Mj)
cases["cg_jacobi256"] = {"op": "cg_jacobi", "bsr": bsr_dict(Ab), "b": b, "tol": 1e-7, "max_iter": 100, "x": x,
                         "iters": it, "rel": rel, "diag": trnsparse.bsr_diagonal(Ab)}
x, it, rel = trnsparse.cg_bsr(Ab, torch.zeros(256), tol=1e-7, max_iter=100)
cases["cg_zero_rhs"] = {"op": "cg", "bsr": bsr_dict(Ab), "b": torch.zeros(256), "tol": 1e-7, "max_iter": 100, "x": x,
                        "iters": it, "rel": rel}
Ie = trnsparse.BSRMatrix.from_dense(torch.eye(128), block_size=128)
torch.manual_seed(23)
b = torch.randn(128)
x, it, rel = trnsparse.cg_bsr(Ie, b, tol=1e-8, max_iter=50)
cases["cg_identity"] = {"op": "cg", "bsr": bsr_dict(Ie), "b": b, "tol": 1e-8, "max_iter": 50, "x": x, "iters": it, "rel": rel}
al, be = trnsparse.chebyshev_coeffs(1.0, 100.0, 10)
cases["cheb_coeffs"] = {"op": "cheb_coeffs", "lam_min": 1.0, "lam_max": 100.0, "K": 10, "alpha": al, "beta": be}
Ad, Ab = spd(128, 128, 9)
torch.manual_seed(24)
b = torch.randn(128)
lam = torch.linalg.eigvalsh(Ad)
x, K, rel = trnsparse.chebyshev_bsr(Ab, b, lam.min().item(), lam.max().item(), K=30)
cases["chebyshev"] = {"op": "chebyshev", "bsr": bsr_dict(Ab), "b": b, "lam_min": lam.min().item(),
                      "lam_max": lam.max().item(), "K": 30, "x": x, "rel": rel}
x, K, rel = trnsparse.richardson_bsr(Ab, b, omega=2.0 / (lam.min().item() + lam.max().item()), K=30)
cases["richardson"] = {"op": "richardson", "bsr": bsr_dict(Ab), "b": b, "omega": 2.0 / (lam.min().item() + lam.max().item()),
                       "K": 30, "x": x, "rel": rel}
torch.manual_seed(25)
v0 = torch.randn(128)
lam_p, v, it = trnsparse.power_iteration_bsr(Ab, v0=v0, max_iter=200, tol=1e-6)
cases["power"] = {"op": "power", "bsr": bsr_dict(Ab), "v0": v0, "max_iter": 200, "tol": 1e-6, "lam": lam_p, "v": v,
                  "iters": it, "eig_max": lam.max().item()}

# ---------------------------------------------------------------- autograd backward formulas
# The reference's backward passes live in its autograd Functions
# (trnsparse/nki/dispatch.py); their forward needs the NKI toolchain, so the
# backward staticmethods are called directly with a context object holding
# what the forward would have saved.
from trnsparse.nki import dispatch as _dispatch  # noqa: E402


class _Ctx:
    def __init__(self, saved, needs, **kw):
        self.saved_tensors = saved
        self.needs_input_grad = needs
        self.__dict__.update(kw)


torch.manual_seed(31)
Db = torch.randn(3 * 128, 2 * 128)
Db[128:256] = 0.0  # an empty block-row
Db[0:128, 128:256] = 0.0  # a missing off-diagonal block
bsr_b = trnsparse.BSRMatrix.from_dense(Db, block_size=128)
Bb = torch.randn(256, 16)
dCb = torch.randn(384, 16)
ctx = _Ctx((bsr_b.blocks, bsr_b.block_col_indices, bsr_b.block_row_ptrs, Bb),
           (True, False, False, False, False, True), A_shape=bsr_b.shape, A_block_size=128)
gblk, _, _, _, _, gB = _dispatch._BSRSpMMFunction.backward(ctx, dCb)
cases["bsr_bwd"] = {"op": "bsr_spmm_backward", "bsr": bsr_dict(bsr_b), "B": Bb, "dC": dCb, "dblocks": gblk, "dB": gB}

torch.manual_seed(32)
n_s = 256
r_s = torch.rand(n_s, 3) * 6.0
diag_s = torch.exp(-0.5 * torch.cdist(r_s, r_s) ** 2).diagonal().clone() * torch.rand(n_s)
A_s = torch.randn(n_s, n_s)
B_s = torch.randn(n_s, 24)
dC_s = torch.randn(n_s, 24)
Q_s = torch.sqrt(torch.abs(diag_s))
mask_s = (Q_s.unsqueeze(-1) * Q_s.unsqueeze(0)) > (1e-3) ** 0.5
ctx = _Ctx((A_s, B_s, mask_s), (True, False, False, True))
gA, _, _, gB = _dispatch._ScreenedSpMMFunction.backward(ctx, dC_s)
cases["screened_bwd"] = {"op": "screened_spmm_backward", "A": A_s, "diag": diag_s, "B": B_s, "threshold": 1e-3,
                         "dC": dC_s, "dA": gA, "dB": gB}

torch.manual_seed(33)
Dm = torch.randn(200, 137)
Dm[torch.rand(200, 137) > 0.05] = 0.0
Bm = torch.randn(137, 24)
dCm = torch.randn(200, 24)
ctx = _Ctx((Dm, Bm), (True, True))
gA, gB = _dispatch._SpMMFunction.backward(ctx, dCm)
cases["spmm_bwd"] = {"op": "spmm_backward", "dense": Dm, "csr": csr_dict(trnsparse.from_dense(Dm)), "B": Bm,
                     "dC": dCm, "dA_dense": gA, "dB": gB}


def _compact(v):
    if isinstance(v, torch.Tensor):
        return v.detach().clone().contiguous()
    if isinstance(v, dict):
        return {k: _compact(x) for k, x in v.items()}
    return v


torch.save(_compact(cases), OUT)
print(f"wrote {len(cases)} cases to {OUT} ({OUT.stat().st_size / 1e6:.2f} MB)")
