"""BSR iterative solvers on B200 (reference: trnsparse/iterative.py).

``cg_bsr`` (with or without the Jacobi preconditioner), ``chebyshev_bsr``,
``richardson_bsr`` and ``power_iteration_bsr`` run fully on the device: each
iteration is one fused SpMV launch (CG adds one vector launch), all scalars
(alpha, beta, inner products, the convergence test) stay in device memory,
and the host only polls a status word between chunks of iterations. The
control flow and return values are the reference's. CG with an arbitrary
user preconditioner (a callable or a dense inverse) runs the reference's
host-driven loop with the device SpMV as the matvec.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

from . import _lib
from .formats import BSRMatrix
from .ops import _back, _bsr_geometry, _dev_of, _on, bsr_spmm

_STATUS_BYTES = 64


def _status(ws: torch.Tensor) -> tuple[int, int, int, float]:
    """(done, iters, reason, rel) from a solver workspace's status record."""
    head = ws[:_STATUS_BYTES].cpu()
    ints = head[:16].view(torch.int32).tolist()
    rel = head[16:24].view(torch.float64).item()
    return ints[0], ints[1], ints[2], rel


def bsr_diagonal(A: BSRMatrix) -> torch.Tensor:
    """Main diagonal of a BSR matrix (reference: iterative.py:22-41).

    Taken from the diagonal blocks (block-row i, block-column i); zero where
    no diagonal block is stored. Returned on the device of ``A.blocks``.
    """
    m, _ = A.shape
    b = A.block_size
    mt = (m + b - 1) // b
    out = torch.zeros(mt * b, dtype=A.dtype, device=A.blocks.device)
    if A.n_blocks:
        rows = A.block_rows()
        cols = A.block_col_indices.to(torch.long).cpu()
        diag = (rows == cols).nonzero(as_tuple=True)[0]
        # first diagonal block of each block-row (the reference breaks on the first match)
        seen: dict[int, int] = {}
        for k in diag.tolist():
            seen.setdefault(int(rows[k]), k)
        if seen:
            br = torch.tensor(list(seen.keys()), dtype=torch.long)
            ks = torch.tensor(list(seen.values()), dtype=torch.long, device=A.blocks.device)
            d = torch.diagonal(A.blocks[ks], dim1=-2, dim2=-1)  # (nd, b)
            idx = (br.unsqueeze(1) * b + torch.arange(b)).reshape(-1).to(A.blocks.device)
            out[idx] = d.reshape(-1)
    return out[:m]


def jacobi_preconditioner_bsr(A: BSRMatrix) -> Callable[[torch.Tensor], torch.Tensor]:
    """``M(r) = r / diag(A)`` (reference: iterative.py:129-145).

    Raises ValueError on a near-zero diagonal entry. The returned callable
    carries its inverse diagonal so ``cg_bsr`` can fuse it into the device
    iteration.
    """
    d = bsr_diagonal(A)
    if torch.any(d.abs() < 1e-15):
        raise ValueError("Jacobi preconditioner: diagonal has near-zero entries")
    inv_d = 1.0 / d

    def precond(r: torch.Tensor) -> torch.Tensor:
        return r * inv_d.to(r.device)

    precond._trnsparse_inv_d = inv_d  # type: ignore[attr-defined]
    return precond


def _matvec(A: BSRMatrix) -> Callable[[torch.Tensor], torch.Tensor]:
    def mv(x: torch.Tensor) -> torch.Tensor:
        return bsr_spmm(A, x.unsqueeze(1)).squeeze(1)

    return mv


def cg_bsr(
    A: BSRMatrix,
    b: torch.Tensor,
    x0: torch.Tensor | None = None,
    tol: float = 1e-6,
    max_iter: int = 1000,
    M: Callable[[torch.Tensor], torch.Tensor] | torch.Tensor | None = None,
) -> tuple[torch.Tensor, int, float]:
    """Preconditioned CG for SPD ``A`` (reference: iterative.py:53-126).

    Returns ``(x, iters, rel_residual)``; ``x`` is on ``b``'s device.
    """
    x, iters, rel, _ = _cg_bsr_device(A, b, x0, tol, max_iter, M)
    return x, iters, rel


def _inv_diag_on(M, dev: torch.device) -> torch.Tensor:
    """The Jacobi preconditioner's inverse diagonal as float32 on ``dev``,
    copied once per device and kept on the callable (the callable is built
    for one matrix; its inverse diagonal never changes)."""
    cache = M.__dict__.setdefault("_trnsparse_inv_d_dev", {})
    t = cache.get(str(dev))
    if t is None:
        t = cache[str(dev)] = _on(M._trnsparse_inv_d, dev, torch.float32)
    return t


def _cg_executed(ws: torch.Tensor, n: int, max_iter: int) -> int:
    """Iterations that did work: the last k whose p.Ap slot was written (the
    reference's loop may break early on |p.Ap| < 1e-30)."""
    import ctypes

    offs = (ctypes.c_size_t * 9)()
    _lib.call("trnsparse_bsr_cg_layout", n, max_iter, offs)
    pap = ws[offs[1] : offs[1] + 32 * (max_iter + 1)].view(torch.float64).view(-1, 4)[:, 0]
    nz = (pap != 0).nonzero()
    return int(nz[-1].item()) + 1 if nz.numel() else 0


def _cg_bsr_device(A, b, x0, tol, max_iter, M) -> tuple[torch.Tensor, int, float, int]:
    """cg_bsr plus the number of iterations that did work (-1 on the host loop).

    Block size 128, square block-aligned A, x0 = 0: the whole solve is one
    cooperative launch (``trnsparse_bsr_cg_fused_start`` + ``_coop_run`` on a
    one-rank peer world whose buffer is a plain workspace): every iteration's
    two phases run inside the kernel and it returns once the reference's loop
    would have stopped (converged, or |p.Ap| < 1e-30), so no launch is spent
    after the end. The arithmetic is that of the two-launch iteration. Other
    shapes, or an x0, go through ``trnsparse_bsr_cg_start`` / ``_iterate``.
    """
    inv_d = None
    fused = M is None or (callable(M) and hasattr(M, "_trnsparse_inv_d"))
    if not fused or b.dtype != torch.float32 or A.dtype != torch.float32:
        x, it, rel = _cg_host_loop(A, b, x0, tol, max_iter, M)
        return x, it, rel, -1
    dev = _dev_of(b, x0)
    n = b.shape[0]
    geo = _bsr_geometry(A, dev)
    if M is not None:
        inv_d = _inv_diag_on(M, dev)
    bd = _on(b, dev, torch.float32)
    x = (x0.to(device=dev, dtype=torch.float32).clone() if x0 is not None
         else torch.zeros(n, dtype=torch.float32, device=dev))
    ws_bytes = _lib.raw("trnsparse_bsr_cg_workspace_size")(n, max_iter)
    s = _lib.stream_handle(dev)
    m_, n_ = A.shape
    whole = x0 is None and A.block_size == 128 and m_ == n_ == n and n % 128 == 0 and max_iter >= 1
    with torch.cuda.device(dev):
        if whole:
            comm_off = (ws_bytes + 255) // 256 * 256
            ws = torch.zeros(comm_off + _lib.raw("trnsparse_peer_comm_bytes")(1), dtype=torch.uint8, device=dev)
            peers = torch.full((1,), ws.data_ptr(), dtype=torch.int64, device=dev)  # a fill, no host copy
            sends = torch.zeros(3, dtype=torch.int64, device=dev)
            peer = (peers.data_ptr(), 1, 0, comm_off, sends.data_ptr(), 0)
            _lib.call("trnsparse_bsr_cg_fused_start", n, n, 128, bd.data_ptr(), _lib.ptr(inv_d), max_iter,
                      ws.data_ptr(), ws_bytes, *peer, s)
            _lib.call("trnsparse_bsr_cg_coop_run", *geo, x.data_ptr(), _lib.ptr(inv_d), float(tol), max_iter, 0,
                      max_iter, ws.data_ptr(), *peer, s)
            done, iters, reason, rel = _status(ws)
            if reason == 5:
                raise RuntimeError("cg_bsr: a bounded device wait timed out (device error word set)")
            return _back(x, b), iters, rel, _cg_executed(ws, n, max_iter)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        _lib.call("trnsparse_bsr_cg_start", *geo, bd.data_ptr(), x.data_ptr(), 1 if x0 is None else 0,
                  _lib.ptr(inv_d), max_iter, ws.data_ptr(), ws_bytes, s)
        # Iterations go out in chunks; the host reads the status record of a
        # chunk (an async copy into pinned memory) while the next chunk is
        # already queued, so the device never waits for the host and at most
        # one chunk of launches is issued after the solve has ended (they exit
        # at once on the status word).
        head = torch.empty(_STATUS_BYTES, dtype=torch.uint8, pin_memory=True)
        stream = torch.cuda.current_stream(dev)
        k, chunk = 0, 8

        def launch(k0: int) -> int:
            k1 = min(k0 + chunk, max_iter + 1)
            _lib.call("trnsparse_bsr_cg_iterate", *geo, x.data_ptr(), _lib.ptr(inv_d), float(tol), max_iter, k0,
                      k1, ws.data_ptr(), s)
            return k1

        k = launch(k)
        while True:
            head.copy_(ws[:_STATUS_BYTES], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
            if k <= max_iter:
                k = launch(k)
            ev.synchronize()
            if head[:4].view(torch.int32).item() or k > max_iter:
                break
            chunk = min(2 * chunk, 64)
        done, iters, _reason, rel = _status(ws)
    return _back(x, b), iters, rel, _cg_executed(ws, n, max_iter)


def _cg_host_loop(A, b, x0, tol, max_iter, M):
    """Reference control flow with host scalars; matvec on the device."""
    dev = _dev_of(b, x0)
    mv = _matvec(A)
    n = b.shape[0]
    if M is None:
        precond = None
    elif callable(M):
        precond = M
    else:
        Md = M.to(dev)

        def precond(r):
            return torch.mv(Md, r)

    bd = b.to(dev)
    x = x0.to(dev).clone() if x0 is not None else torch.zeros(n, dtype=b.dtype, device=dev)
    r = bd - mv(x)
    b_norm = torch.linalg.norm(bd).item()
    if b_norm < 1e-15:
        return _back(x, b), 0, 0.0
    z = precond(r) if precond is not None else r.clone()
    p = z.clone()
    rz = torch.dot(r, z).item()
    r_norm = float("nan")
    for k in range(max_iter):
        Ap = mv(p)
        pAp = torch.dot(p, Ap).item()
        if abs(pAp) < 1e-30:
            break
        alpha = rz / pAp
        x = x + alpha * p
        r = r - alpha * Ap
        r_norm = torch.linalg.norm(r).item()
        rel = r_norm / b_norm
        if rel < tol:
            return _back(x, b), k + 1, rel
        z = precond(r) if precond is not None else r
        rz_new = torch.dot(r, z).item()
        p = z + (rz_new / rz) * p
        rz = rz_new
    return _back(x, b), max_iter, r_norm / b_norm


def chebyshev_coeffs(lam_min: float, lam_max: float, K: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Momentum-form Chebyshev step coefficients (reference: iterative.py:148-190).

    Recurrence in float64 (Barrett et al. 1994, Templates, Alg. 2.1, momentum
    form), returned as float32 tensors of length K.
    """
    c = (lam_max - lam_min) / 2.0
    d = (lam_max + lam_min) / 2.0
    alpha = torch.zeros(K, dtype=torch.float64)
    beta = torch.zeros(K, dtype=torch.float64)
    a_prev = 1.0 / d
    if K > 0:
        alpha[0] = a_prev
    for k in range(1, K):
        bt = (c * a_prev / 2.0) ** 2
        a_new = 1.0 / (d - bt / a_prev)
        alpha[k] = a_new
        beta[k] = a_new * bt / a_prev
        a_prev = a_new
    return alpha.float(), beta.float()


def _fixed_step_solver(name, A, b, x0, extra_args, K):
    import ctypes

    dev = _dev_of(b, x0)
    n = b.shape[0]
    geo = _bsr_geometry(A, dev)
    bd = _on(b, dev, torch.float32)
    x = (x0.to(device=dev, dtype=torch.float32).clone() if x0 is not None
         else torch.zeros(n, dtype=torch.float32, device=dev))
    work = torch.empty(2 * n + 64, dtype=torch.float32, device=dev)
    rr = torch.zeros(1, dtype=torch.float64, device=dev)
    b_norm = torch.linalg.norm(bd).item()
    with torch.cuda.device(dev):
        _lib.call(name, *geo, bd.data_ptr(), *extra_args, K, x.data_ptr(), work.data_ptr(), rr.data_ptr(),
                  _lib.stream_handle(dev))
    r_norm = float(torch.sqrt(rr).float().item())
    return _back(x, b), K, r_norm / max(b_norm, 1e-15)


def chebyshev_bsr(
    A: BSRMatrix,
    b: torch.Tensor,
    lam_min: float,
    lam_max: float,
    K: int = 50,
    x0: torch.Tensor | None = None,
) -> tuple[torch.Tensor, int, float]:
    """K-step Chebyshev semi-iteration (reference: iterative.py:193-253); returns (x, K, rel)."""
    import ctypes

    alpha, beta = chebyshev_coeffs(lam_min, lam_max, K)
    fa = (ctypes.c_float * max(K, 1))(*alpha.tolist())
    fb = (ctypes.c_float * max(K, 1))(*beta.tolist())
    return _fixed_step_solver("trnsparse_bsr_chebyshev", A, b, x0, (fa, fb), K)


def richardson_bsr(
    A: BSRMatrix,
    b: torch.Tensor,
    omega: float,
    K: int = 100,
    x0: torch.Tensor | None = None,
) -> tuple[torch.Tensor, int, float]:
    """K-step Richardson ``x += omega (b - A x)`` (reference: iterative.py:256-295)."""
    return _fixed_step_solver("trnsparse_bsr_richardson", A, b, x0, (float(omega),), K)


def power_iteration_bsr(
    A: BSRMatrix,
    v0: torch.Tensor | None = None,
    max_iter: int = 100,
    tol: float = 1e-9,
) -> tuple[float, torch.Tensor, int]:
    """Dominant eigenpair by power iteration (reference: iterative.py:298-340).

    Without ``v0`` the start vector is ``torch.randn(n)`` from the global CPU
    generator, as in the reference. Returns ``(eigenvalue, v, iters)``.
    """
    n = A.shape[0]
    if v0 is None:
        v0 = torch.randn(n, dtype=A.dtype)
    dev = _dev_of(v0)
    geo = _bsr_geometry(A, dev)
    v0d = _on(v0, dev, torch.float32)
    v = torch.empty(n, dtype=torch.float32, device=dev)
    ws_bytes = _lib.raw("trnsparse_bsr_power_workspace_size")(n, max_iter)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    s = _lib.stream_handle(dev)
    with torch.cuda.device(dev):
        k = 0
        chunk = 8
        while True:
            k_end = min(k + chunk, max_iter + 1)
            _lib.call("trnsparse_bsr_power_iterate", *geo, v0d.data_ptr(), v.data_ptr(), float(tol), max_iter, k, k_end,
                      ws.data_ptr(), ws_bytes, s)
            k = k_end
            done, iters, reason, lam = _status(ws)
            if done or k > max_iter:
                break
            chunk *= 2
        if done and k <= max_iter:
            _lib.call("trnsparse_bsr_power_finish", n, v.data_ptr(), max_iter, ws.data_ptr(), s)
    if reason == 3:  # ||A v|| < 1e-30: the reference returns (0.0, v, k + 1)
        lam = 0.0
    return float(lam), _back(v, v0), iters
