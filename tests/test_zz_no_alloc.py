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


def _noalloc(A, b, inv_d, tol, max_iter):
    dev = b.device
    x = torch.zeros_like(b)
    status = torch.zeros(64, dtype=torch.uint8, device=dev)
    _lib.call("trnsparse_bsr_cg_noalloc", *_bsr_geometry(A, dev), b.data_ptr(), x.data_ptr(), 1,
              _lib.ptr(inv_d), float(tol), max_iter, status.data_ptr(), _lib.stream_handle(dev))
    st = status.cpu()
    done, iters = st[:8].view(torch.int32).tolist()
    return x, done, iters, st[16:24].view(torch.float64).item()


@pytest.mark.parametrize("block_rows,max_iter,tol", [(64, 30, 0.0), (32, 100, 1e-6)])
def test_noalloc_matches_workspace_cg(block_rows, max_iter, tol):
    A, b = workloads.block_pentadiagonal_spd(block_rows)
    M = ts.jacobi_preconditioner_bsr(A)
    bd = b.cuda()
    inv_d = M._trnsparse_inv_d.cuda().float().contiguous()
    x_ref, it_ref, rel_ref = ts.cg_bsr(A, bd, tol=tol, max_iter=max_iter, M=M)
    for _ in range(2):  # two calls in a row share the scratch array
        x, done, iters, rel = _noalloc(A, bd, inv_d, tol, max_iter)
        assert done == 1 and iters == it_ref
        err = (torch.linalg.norm(x.double() - x_ref.double()) / torch.linalg.norm(x_ref.double())).item()
        assert err <= 1e-5
        assert abs(rel - rel_ref) <= 1e-5 * max(abs(rel_ref), 1e-30) + 1e-12


def test_noalloc_rejects_oversize():
    A, b = workloads.block_pentadiagonal_spd(4)
    big_n = 8 << 20  # 8M unknowns need more than the fixed scratch
    with pytest.raises(AssertionError, match="scratch"):
        _lib.call("trnsparse_bsr_cg_noalloc", big_n, big_n, 128, 0, 0, 0, 0, 0, 0, 1, None, 0.0, 10, None, None)
