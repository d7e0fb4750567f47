"""The allocation-free CG entry point against the workspace-based one.

trnsparse_bsr_cg_noalloc serves callers that cannot allocate device memory
(for example code running inside an allocator callback, or a host with a
fixed memory budget): it keeps its scratch in a fixed array inside the
library. This test calls it through the C ABI twice in a row (the second
call must not see leftovers of the first) and compares each solution with
cg_bsr's, which runs the same solver on a caller workspace, at the 1e-5
relative Frobenius tolerance of the other solver tests. It lives in its own
file, collected last, and needs no state from other tests.
"""

from __future__ import annotations

import pytest
import torch

import trnsparse_b200 as ts
from trnsparse_b200 import _lib, workloads
from trnsparse_b200.ops import _bsr_geometry

pytestmark = pytest.mark.gpu


def _status(st):
    st = st.cpu()
    done, iters, reason = st[:12].view(torch.int32).tolist()
    return done, iters, reason, st[16:24].view(torch.float64).item()


def _noalloc(A, b, x0, inv_d, tol, max_iter):
    dev = b.device
    x = torch.zeros_like(b) if x0 is None else x0.clone()
    status = torch.zeros(64, dtype=torch.uint8, device=dev)
    _lib.call("trnsparse_bsr_cg_noalloc", *_bsr_geometry(A, dev), b.data_ptr(), x.data_ptr(), 1 if x0 is None else 0,
              _lib.ptr(inv_d), float(tol), max_iter, status.data_ptr(), _lib.stream_handle(dev))
    return (x,) + _status(status)


def _workspace(A, b, x0, inv_d, tol, max_iter):
    """The same solve through trnsparse_bsr_cg_start/_iterate on a caller workspace."""
    dev = b.device
    x = torch.zeros_like(b) if x0 is None else x0.clone()
    nbytes = _lib.raw("trnsparse_bsr_cg_workspace_size")(b.numel(), max_iter)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    geo = _bsr_geometry(A, dev)
    s = _lib.stream_handle(dev)
    _lib.call("trnsparse_bsr_cg_start", *geo, b.data_ptr(), x.data_ptr(), 1 if x0 is None else 0, _lib.ptr(inv_d),
              max_iter, ws.data_ptr(), nbytes, s)
    _lib.call("trnsparse_bsr_cg_iterate", *geo, x.data_ptr(), _lib.ptr(inv_d), float(tol), max_iter, 0,
              max_iter + 1, ws.data_ptr(), s)
    return (x,) + _status(ws[:64])


@pytest.mark.parametrize("block_rows,max_iter,tol,jacobi,start", [
    (64, 30, 0.0, True, "zero"),
    (32, 100, 1e-6, True, "zero"),
    (32, 100, 1e-6, True, "x0"),      # x0 != 0: the r = b - A x0 start
    (32, 60, 1e-6, False, "zero"),    # no preconditioner (inv_d NULL)
    (16, 40, 0.0, False, "x0"),
])
def test_noalloc_matches_workspace_cg(block_rows, max_iter, tol, jacobi, start):
    A, b = workloads.block_pentadiagonal_spd(block_rows)
    bd = b.cuda()
    inv_d = ts.jacobi_preconditioner_bsr(A)._trnsparse_inv_d.cuda().float().contiguous() if jacobi else None
    x0 = torch.randn(b.shape, generator=torch.Generator().manual_seed(3)).cuda() if start == "x0" else None
    x_ref, done_ref, it_ref, reason_ref, rel_ref = _workspace(A, bd, x0, inv_d, tol, max_iter)
    # the public API agrees with the workspace solve it wraps
    M = ts.jacobi_preconditioner_bsr(A) if jacobi else None
    x_api, it_api, _ = ts.cg_bsr(A, bd, x0=x0, tol=tol, max_iter=max_iter, M=M)
    assert it_api == it_ref
    for _ in range(2):  # two calls in a row share the scratch array
        x, done, iters, reason, rel = _noalloc(A, bd, x0, inv_d, tol, max_iter)
        assert done == done_ref == 1 and iters == it_ref and reason == reason_ref
        err = (torch.linalg.norm(x.double() - x_ref.double()) / torch.linalg.norm(x_ref.double())).item()
        assert err <= 1e-5
        assert abs(rel - rel_ref) <= 1e-5 * max(abs(rel_ref), 1e-30) + 1e-12


def test_noalloc_rejects_oversize():
    A, b = workloads.block_pentadiagonal_spd(4)
    big_n = 8 << 20  # 8M unknowns need more than the fixed scratch
    with pytest.raises(AssertionError, match="scratch"):
        _lib.call("trnsparse_bsr_cg_noalloc", big_n, big_n, 128, 0, 0, 0, 0, 0, 0, 1, None, 0.0, 10, None, None)
