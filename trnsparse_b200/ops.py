"""Sparse operations on B200 (reference API: trnsparse/ops.py).

Every hot-path op keeps the reference's signature and semantics and runs on
the GPU through the C ABI (``_lib.call``). Dense operands may live on the
host or on the GPU: host inputs are copied to the current CUDA device and
the result is copied back, so code written for the reference's CPU path gets
the same (host) tensors back; CUDA inputs stay on the device. There is no CPU
compute path and no backend switch.
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _lib
from .formats import BSRMatrix, COOMatrix, CSRMatrix


def _dev_of(*ts: torch.Tensor | None) -> torch.device:
    for t in ts:
        if t is not None and t.is_cuda:
            return t.device
    return _lib.require_cuda()


def _on(t: torch.Tensor | None, dev: torch.device, dtype: torch.dtype | None = None) -> torch.Tensor | None:
    if t is None:
        return None
    if t.device != dev or (dtype is not None and t.dtype != dtype):
        t = t.to(device=dev, dtype=dtype, non_blocking=t.is_pinned() if t.device.type == "cpu" else False)
    return t.contiguous()


def _back(out: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
    """Return ``out`` on ``like``'s device; host results land in pinned memory."""
    if like.is_cuda:
        return out
    host = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    host.copy_(out, non_blocking=True)
    torch.cuda.current_stream(out.device).synchronize()
    return host


# ---------------------------------------------------------------------------
# CSR
# ---------------------------------------------------------------------------


def spmv(
    A: CSRMatrix,
    x: torch.Tensor,
    alpha: float = 1.0,
    y: torch.Tensor | None = None,
    beta: float = 0.0,
) -> torch.Tensor:
    """``alpha * A @ x (+ beta * y)`` (reference: trnsparse/ops.py:30-48).

    ``beta * y`` is added only when ``y is not None and beta != 0.0``. A 2-D
    ``x`` is treated as a dense right-hand side (as ``sparse @ x`` would).
    Differentiable in ``A.values``, ``x`` and ``y`` (as the reference's torch
    path is); the backward runs the transposed product on the device.
    """
    m, n = A.shape
    assert x.shape[0] == n, f"Dimension mismatch: A is {A.shape}, x is {x.shape}"
    if x.dim() == 2:
        return spmm(A, x, alpha=alpha, C=y, beta=beta)
    if _needs_grad(A.values, x, y):
        use_y = y is not None and beta != 0.0
        return _CsrProductFn.apply(A.values, x, y if use_y else None, A, float(alpha), float(beta))
    return _spmv_impl(A, x, alpha, y, beta)


_SPMV_PIPE_CHUNKS = 4          # row / x chunks of the host-buffer pipeline (4 measured best of 4-32)
_SPMV_DIRECT_Y = os.environ.get("TRNSPARSE_SPMV_DIRECT_Y", "1") != "0"
_SPMV_PIPE_MIN_ROWS = 1 << 18  # smaller products are not worth splitting


def _spmv_pipe_plan(row_ptrs: torch.Tensor, col_indices: torch.Tensor, m: int, K: int):
    """Row chunks (multiples of 64 rows, about m / K each) and, per chunk, the
    prefix of x it needs (its largest column + 1, made non-decreasing):
    ``(n_chunks, splits int64 [n_chunks + 1], need int64 [n_chunks])`` on the host."""
    rp = row_ptrs.long()
    rstep = (-(-m // K) + 63) // 64 * 64
    splits = list(range(0, m, rstep)) + [m]
    bounds = rp[torch.tensor(splits, device=rp.device)].tolist()
    need, top = [], 0
    for i in range(len(splits) - 1):
        lo, hi = bounds[i], bounds[i + 1]
        if hi > lo:
            top = max(top, int(col_indices[lo:hi].max().item()) + 1)
        need.append(top)
    return len(splits) - 1, torch.tensor(splits, dtype=torch.int64), torch.tensor(need, dtype=torch.int64)


def _spmv_pipelined(A: CSRMatrix, lay: dict, x: torch.Tensor, alpha: float, dev: torch.device) -> torch.Tensor:
    """``alpha * A @ x`` for a pinned host ``x`` through ``trnsparse_csr_spmv_host``:
    x goes up in pieces, each row chunk's product starts once the x entries
    its columns reach have arrived, and its rows come back while later chunks
    still compute, so both PCIe directions and the kernel overlap."""
    m, n = A.shape
    K = _SPMV_PIPE_CHUNKS
    key = ("spmv_pipe", K)
    plan = lay.get(key)
    if plan is None:
        plan = _spmv_pipe_plan(lay["row_ptrs"], lay["col_indices"], m, K)
        lay[key] = plan
    nch, splits, need = plan
    xd = torch.empty(n, dtype=A.dtype, device=dev)
    host = torch.empty(m, dtype=A.dtype, pin_memory=True)
    st = torch.cuda.current_stream(dev)
    # _SPMV_DIRECT_Y: the row chunks' kernels write y straight into the pinned host buffer
    # (out_dev == out_host); otherwise y goes through a device buffer and copies back
    out = host if _SPMV_DIRECT_Y else torch.empty(m, dtype=A.dtype, device=dev)
    _lib.call("trnsparse_csr_spmv_host", m, n, A.nnz, _lib.index_code(lay["row_ptrs"].dtype), _lib.dtype_code(A.dtype),
              _lib.ptr(lay["row_ptrs"]), _lib.ptr(lay["col_indices"]), _lib.ptr(lay["values"]), x.data_ptr(),
              float(alpha), host.data_ptr(), xd.data_ptr(), out.data_ptr(), nch, splits.data_ptr(), need.data_ptr(),
              st.cuda_stream)
    st.synchronize()
    return host


def _spmv_impl(A: CSRMatrix, x: torch.Tensor, alpha: float, y, beta: float) -> torch.Tensor:
    m, n = A.shape
    dev = _dev_of(x)
    if x.dtype != A.dtype:
        raise RuntimeError(f"spmv: dtype mismatch, A is {A.dtype} and x is {x.dtype}")
    lay = A.device_layout(dev)
    if (not x.is_cuda and x.is_pinned() and x.is_contiguous() and (y is None or beta == 0.0)
            and m >= _SPMV_PIPE_MIN_ROWS and n >= _SPMV_PIPE_MIN_ROWS and A.nnz > 0
            and A.dtype in (torch.float32, torch.float64)):
        with torch.cuda.device(dev):
            return _spmv_pipelined(A, lay, x, alpha, dev)
    xd = _on(x, dev)
    use_y = y is not None and beta != 0.0
    yd = _on(y, dev, A.dtype) if use_y else None
    if use_y:
        yd = yd.expand(m).contiguous() if yd.dim() == 0 or yd.shape[0] != m else yd
    out = torch.empty(m, dtype=A.dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.call(
            "trnsparse_csr_spmv", m, n, A.nnz, _lib.index_code(lay["row_ptrs"].dtype), _lib.dtype_code(A.dtype),
            _lib.ptr(lay["row_ptrs"]), _lib.ptr(lay["col_indices"]), _lib.ptr(lay["values"]),
            _lib.ptr(xd), float(alpha), _lib.ptr(yd), float(beta), _lib.ptr(out), _lib.stream_handle(dev),
        )
    return _back(out, x)


def spmm(
    A: CSRMatrix,
    B: torch.Tensor,
    alpha: float = 1.0,
    C: torch.Tensor | None = None,
    beta: float = 0.0,
) -> torch.Tensor:
    """``alpha * A @ B (+ beta * C)`` (reference: trnsparse/ops.py:51-78).
    Differentiable in ``A.values``, ``B`` and ``C``."""
    m, n = A.shape
    assert B.shape[0] == n, f"Dimension mismatch: A is {A.shape}, B is {B.shape}"
    if B.dim() == 1:
        return spmv(A, B, alpha=alpha, y=C, beta=beta)
    if _needs_grad(A.values, B, C):
        use_c = C is not None and beta != 0.0
        return _CsrProductFn.apply(A.values, B, C if use_c else None, A, float(alpha), float(beta))
    return _spmm_impl(A, B, alpha, C, beta)


def _spmm_impl(A: CSRMatrix, B: torch.Tensor, alpha: float, C, beta: float) -> torch.Tensor:
    m, n = A.shape
    dev = _dev_of(B)
    if B.dtype != A.dtype:
        raise RuntimeError(f"spmm: dtype mismatch, A is {A.dtype} and B is {B.dtype}")
    k = B.shape[1]
    lay = A.device_layout(dev)
    Bd = _on(B, dev)
    use_c = C is not None and beta != 0.0
    Cd = None
    if use_c:
        Cd = _on(C, dev, A.dtype)
        if tuple(Cd.shape) != (m, k):
            Cd = Cd.expand(m, k).contiguous()
    out = torch.empty(m, k, dtype=A.dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.call(
            "trnsparse_csr_spmm", m, n, k, A.nnz, _lib.index_code(lay["row_ptrs"].dtype), _lib.dtype_code(A.dtype),
            _lib.ptr(lay["row_ptrs"]), _lib.ptr(lay["col_indices"]), _lib.ptr(lay["values"]),
            _lib.ptr(Bd), k, float(alpha), _lib.ptr(Cd), k, float(beta), _lib.ptr(out), k,
            _lib.stream_handle(dev),
        )
    return _back(out, B)


def _transpose_structure(row_ptrs: torch.Tensor, col_indices: torch.Tensor, m: int, n: int, strict: bool,
                         cache: dict, dev: torch.device) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, int]:
    """Transposed pattern of an m x n CSR structure, built on the device
    (``trnsparse_csr_transpose``): ``(row_ptr_t, col_t, perm, nnz_t)`` with
    ``perm`` the index in A of each entry of A^T (the diagonal left out when
    ``strict``). Index arrays are int32 when the sizes allow. ``cache`` keeps
    one entry per (strict, device), keyed by the structure's fingerprint and
    replaced when the structure changes; values are never cached."""
    from .formats import _fingerprint

    key = ("transpose_structure", strict, str(dev))
    fp = _fingerprint(col_indices, row_ptrs)
    hit = cache.get(key)
    if hit is not None and hit[0] == fp:
        return hit[1]
    idx_t = torch.int32 if row_ptrs.dtype == torch.int32 and col_indices.dtype == torch.int32 else torch.int64
    rp = row_ptrs.to(device=dev, dtype=idx_t).contiguous()
    ci = col_indices.to(device=dev, dtype=idx_t).contiguous()
    nnz = ci.numel()
    rpt = torch.empty(n + 1, dtype=torch.int64, device=dev)
    colt = torch.empty(max(nnz, 1), dtype=torch.int64, device=dev)
    perm = torch.empty(max(nnz, 1), dtype=torch.int64, device=dev)
    ws_bytes = _lib.raw("trnsparse_csr_transpose_workspace_size")(m, n, nnz)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.call("trnsparse_csr_transpose", m, n, nnz, _lib.index_code(idx_t), rp.data_ptr(), ci.data_ptr(),
                  1 if strict else 0, rpt.data_ptr(), colt.data_ptr(), perm.data_ptr(), ws.data_ptr(), ws_bytes,
                  _lib.stream_handle(dev))
    nnz_t = int(rpt[n].item()) if strict else nnz
    colt, perm = colt[:nnz_t], perm[:nnz_t]
    if max(m, nnz_t) < (1 << 31):  # int32 indices halve the index traffic of the transposed products
        rpt, colt = rpt.to(torch.int32), colt.to(torch.int32)
    out = (rpt, colt, perm, nnz_t)
    cache[key] = (fp, out)
    return out


def _gather(src: torch.Tensor, perm: torch.Tensor) -> torch.Tensor:
    """``src[perm]`` on the device with the library's gather kernel."""
    out = torch.empty(perm.numel(), dtype=src.dtype, device=src.device)
    if perm.numel():
        with torch.cuda.device(src.device):
            _lib.call("trnsparse_gather", perm.numel(), src.element_size(), src.data_ptr(), perm.data_ptr(),
                      out.data_ptr(), _lib.stream_handle(src.device))
    return out


def spmv_symmetric(A: CSRMatrix, x: torch.Tensor, alpha: float = 1.0, uplo: str = "upper") -> torch.Tensor:
    """``alpha * (A @ x + strict(A)^T @ x)`` for one stored triangle (ops.py:81-104).

    As in the reference, ``uplo`` does not change the arithmetic: the stored
    entries are A, the off-diagonal ones are mirrored. The transposed strict
    pattern is built once per structure on the device; its values are
    gathered from ``A.values`` on every call (in-place updates of the values
    are always seen). Both products run through the CSR SpMV kernel: the
    first gives ``alpha * A @ x``, the second adds ``alpha * strict(A)^T @ x``
    to it as its ``beta * y`` term.
    """
    m, n = A.shape
    assert m == n, "Matrix must be square for symmetric SpMV"
    dev = _dev_of(x)
    lay = A.device_layout(dev)
    rpt, colt, perm, nnz_t = _transpose_structure(A.row_ptrs, A.col_indices, m, n, True, A._dev, dev)
    ST = CSRMatrix(values=_gather(lay["values"], perm), col_indices=colt, row_ptrs=rpt, shape=(n, m))
    xd = _on(x, dev)
    y = _spmv_impl(A, xd, alpha, None, 0.0)
    return _back(_spmv_impl(ST, xd, alpha, y, 1.0), x)


def sparse_add(A: CSRMatrix, B: CSRMatrix, alpha: float = 1.0, beta: float = 1.0) -> CSRMatrix:
    """Pattern union ``alpha*A + beta*B`` (ops.py:107-133); structural host op."""
    assert A.shape == B.shape, f"Shape mismatch: {A.shape} vs {B.shape}"
    ca, cb = A.to_coo(), B.to_coo()
    idx = torch.stack(
        [torch.cat([ca.row_indices, cb.row_indices]), torch.cat([ca.col_indices.long(), cb.col_indices.long()])]
    )
    vals = torch.cat([alpha * ca.values, beta * cb.values])
    csr = torch.sparse_coo_tensor(idx, vals, size=A.shape).coalesce().to_sparse_csr()
    return CSRMatrix(values=csr.values(), col_indices=csr.col_indices(), row_ptrs=csr.crow_indices(), shape=A.shape)


def sparse_scale(A: CSRMatrix, alpha: float) -> CSRMatrix:
    """``alpha * A`` with copied structure (ops.py:136-143)."""
    return CSRMatrix(
        values=alpha * A.values, col_indices=A.col_indices.clone(), row_ptrs=A.row_ptrs.clone(), shape=A.shape
    )


def sparse_transpose(A: CSRMatrix) -> CSRMatrix:
    """CSR of A^T (ops.py:146-154); structural host op."""
    coo = A.to_coo()
    return COOMatrix(
        values=coo.values, row_indices=coo.col_indices, col_indices=coo.row_indices, shape=(A.shape[1], A.shape[0])
    ).to_csr()


def nnz_per_row(A: CSRMatrix) -> torch.Tensor:
    """Stored entries per row (ops.py:157-159)."""
    return A.row_ptrs[1:] - A.row_ptrs[:-1]


# ---------------------------------------------------------------------------
# BSR
# ---------------------------------------------------------------------------


def _bsr_geometry(A: BSRMatrix, dev: torch.device, dtype: torch.dtype = torch.float32) -> tuple:
    """The seven leading BSR arguments of the C ABI for ``A`` on ``dev``."""
    lay = A.device_layout(dev)
    blocks = lay["blocks"]
    if blocks.dtype != dtype:
        key = ("blocks", dtype)
        if lay.get(key) is None:
            lay[key] = blocks.to(dtype).contiguous()
        blocks = lay[key]
    m, n = A.shape
    return (m, n, A.block_size, A.n_blocks, lay["row_ptr"].data_ptr(), lay["col_idx"].data_ptr(), blocks.data_ptr())


def _sm_count(dev: torch.device) -> int:
    return torch.cuda.get_device_properties(dev).multi_processor_count


def _tc_plan(A: BSRMatrix, lay: dict, dev: torch.device, k: int) -> tuple[torch.Tensor, int, int, int]:
    """Work schedule for the tensor-core kernel, cached per (matrix, N tiling, k tiles).

    Built on the host by the library (trnsparse_bsr_spmm_tc_plan): units of
    (block-row, run of its blocks, N tile), longest first onto the
    least-loaded of one persistent CTA per SM. Returns (plan on the device,
    grid, needs_zero, bn).
    """
    sms = _sm_count(dev)
    bn = 128 if k <= 128 else 256  # wide tiles read each A block once per 256 columns
    key = ("tc_plan", bn, -(-k // bn))
    hit = lay.get(key)
    if hit is not None:
        return hit
    rp = lay["host_row_ptr"].to(torch.int32).contiguous()
    R = rp.numel() - 1
    cap = _lib.raw("trnsparse_bsr_spmm_tc_plan_capacity")(R, A.n_blocks, k, bn, sms)
    if cap < 0:
        raise ValueError("bsr_spmm: cannot plan this shape")
    plan = torch.empty(cap, dtype=torch.int32)
    n_units, grid, zero = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
    _lib.call("trnsparse_bsr_spmm_tc_plan", R, rp.data_ptr(), k, bn, sms, plan.data_ptr(), cap,
              ctypes.byref(n_units), ctypes.byref(grid), ctypes.byref(zero))
    used = ((grid.value + 4) & ~3) + 4 * n_units.value
    lay[key] = (plan[:used].to(dev), grid.value, zero.value, bn)
    return lay[key]


def _tf32_split(lay: dict, dev: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """The 3xTF32 operands of the fp32 blocks: the blocks themselves as the high part (the
    tensor core reads their top 10 mantissa bits) and, cached with the layout, the
    residual it drops as the low part: one extra copy of the blocks."""
    hit = lay.get("tf32_split")
    if hit is None:
        blocks = lay["blocks"]
        if blocks.dtype != torch.float32:
            blocks = blocks.float().contiguous()
        lo = torch.empty_like(blocks)
        with torch.cuda.device(dev):
            _lib.call("trnsparse_bsr_split_tf32", blocks.numel(), blocks.data_ptr(), None, lo.data_ptr(),
                      _lib.stream_handle(dev))
        hit = lay["tf32_split"] = (blocks, lo)
    return hit


def bsr_spmm(A: BSRMatrix, B: torch.Tensor) -> torch.Tensor:
    """``C = A @ B`` for a BSR ``A`` and dense ``B`` (reference: trnsparse/ops.py:162-210).

    The result has A's dtype; rows of empty block-rows are zero. Paths, all
    on the GPU: one right-hand-side column runs the HBM-bound BSR SpMV
    kernel; block size 128 runs the tcgen05 tensor-core kernel (3xTF32 for
    float32, bf16 operands with fp32 accumulation for bfloat16); other block
    sizes run the CUDA-core kernel (float32 FMA). Differentiable in
    ``A.blocks`` and ``B``: dB = A^T dC runs the same kernels on the cached
    transposed matrix, dblocks[k] = dC[rows(k)] B[cols(k)]^T is one batched
    GEMM over the stored blocks.
    """
    if _needs_grad(A.blocks, B):
        return _BsrSpmmFn.apply(A.blocks, B, A)
    return _bsr_spmm_impl(A, B)


def _bsr_spmm_impl(A: BSRMatrix, B: torch.Tensor) -> torch.Tensor:
    m, n = A.shape
    if B.shape[0] != n:
        raise AssertionError(f"Dimension mismatch: A is {A.shape}, B is {tuple(B.shape)}")
    k = B.shape[1]
    dev = _dev_of(B)
    if A.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"bsr_spmm: blocks dtype {A.dtype} not supported (float32, bfloat16)")
    s = _lib.stream_handle(dev)
    lay = A.device_layout(dev)
    with torch.cuda.device(dev):
        if A.block_size == 128 and k > 1 and A.n_blocks > 0:
            bf16 = A.dtype == torch.bfloat16
            Bd = _on(B, dev, torch.bfloat16 if bf16 else torch.float32)
            plan, grid, zero, bn = _tc_plan(A, lay, dev, k)
            # bf16: C straight from the epilogue in bf16 (split block-rows add their partial sums
            # in bf16, as the reference's bf16 block loop accumulates in the blocks' dtype)
            direct = bf16
            kp = -(-k // 8) * 8 if direct else -(-k // 4) * 4  # 16-byte C rows for the TMA stores
            out = torch.empty(m, kp, dtype=torch.bfloat16 if direct else torch.float32, device=dev)
            if bf16:
                (hi, lo), code = (lay["blocks"], None), _lib.BF16
            else:
                (hi, lo), code = _tf32_split(lay, dev), _lib.F32
            ws_bytes = _lib.raw("trnsparse_bsr_spmm_tc_workspace_size")(n, k, code)
            ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
            _lib.call("trnsparse_bsr_spmm_tc", m, n, A.n_blocks, lay["col_idx"].data_ptr(), hi.data_ptr(),
                      _lib.ptr(lo), code, plan.data_ptr(), grid, zero, Bd.data_ptr(), k, k, out.data_ptr(), kp,
                      _lib.BF16 if direct else _lib.F32, bn, ws.data_ptr(), ws_bytes, s)
            if kp != k:
                out = out[:, :k].contiguous()
            return _back(out.to(A.dtype), B)
        Bd = _on(B, dev, torch.float32)
        out = torch.empty(m, k, dtype=torch.float32, device=dev)
        geo = _bsr_geometry(A, dev)
        if k == 1:
            _lib.call("trnsparse_bsr_spmv", *geo, Bd.data_ptr(), 1.0, None, 0.0, out.data_ptr(), s)
        else:
            _lib.call("trnsparse_bsr_spmm_simt", *geo, Bd.data_ptr(), k, k, out.data_ptr(), k, s)
    return _back(out.to(A.dtype), B)


# ---------------------------------------------------------------- autograd of the products
def _needs_grad(*ts) -> bool:
    return torch.is_grad_enabled() and any(isinstance(t, torch.Tensor) and t.requires_grad for t in ts)


def _csr_transpose(A: CSRMatrix, dev: torch.device) -> CSRMatrix:
    """A^T as a CSRMatrix on ``dev``: the transposed structure (built on the
    device once per structure, one cache slot per matrix) and the values
    gathered from A's current values on every call."""
    m, n = A.shape
    rpt, colt, perm, _ = _transpose_structure(A.row_ptrs, A.col_indices, m, n, False, A._dev, dev)
    vals = A.device_layout(dev)["values"]
    return CSRMatrix(values=_gather(vals, perm), col_indices=colt, row_ptrs=rpt, shape=(n, m))


def _csr_values_grad(A: CSRMatrix, dC: torch.Tensor, B: torch.Tensor, alpha: float) -> torch.Tensor:
    """d values[j] = alpha * <dC[row_j], B[col_j]> (the product's adjoint projected
    on A's pattern), one ``trnsparse_csr_sddmm`` launch over the stored entries."""
    dev = dC.device if dC.is_cuda else _dev_of(B)
    lay = A.device_layout(dev)
    G = _on(dC.reshape(dC.shape[0], -1), dev, A.dtype)
    X = _on(B.reshape(B.shape[0], -1), dev, A.dtype)
    k = G.shape[1]
    out = torch.empty(A.nnz, dtype=A.dtype, device=dev)
    with torch.cuda.device(dev):
        _lib.call("trnsparse_csr_sddmm", A.shape[0], A.shape[1], k, A.nnz, _lib.index_code(lay["row_ptrs"].dtype),
                  _lib.dtype_code(A.dtype), lay["row_ptrs"].data_ptr(), lay["col_indices"].data_ptr(), G.data_ptr(),
                  k, X.data_ptr(), k, float(alpha), out.data_ptr(), _lib.stream_handle(dev))
    return out.to(A.values.device)


class _CsrProductFn(torch.autograd.Function):
    """alpha * A @ X (+ beta * Y) with X a vector or matrix: the adjoints are
    dX = alpha * A^T dOut (the same device kernels on the cached transpose),
    dY = beta * dOut, dvalues = alpha * <dOut[row], X[col]>."""

    @staticmethod
    def forward(ctx, values, X, Y, A, alpha, beta):
        ctx.A, ctx.alpha, ctx.beta = A, alpha, beta
        ctx.save_for_backward(X)
        if X.dim() == 1:
            return _spmv_impl(A, X, alpha, Y, beta)
        return _spmm_impl(A, X, alpha, Y, beta)

    @staticmethod
    def backward(ctx, dout):
        A, alpha, beta = ctx.A, ctx.alpha, ctx.beta
        (X,) = ctx.saved_tensors
        dvals = dX = dY = None
        if ctx.needs_input_grad[1]:
            g = dout.to(X.device).contiguous()
            AT = _csr_transpose(A, g.device if g.is_cuda else _dev_of(g))
            dX = _spmv_impl(AT, g, alpha, None, 0.0) if X.dim() == 1 else _spmm_impl(AT, g, alpha, None, 0.0)
        if ctx.needs_input_grad[2]:
            dY = beta * dout
        if ctx.needs_input_grad[0]:
            dvals = _csr_values_grad(A, dout, X, alpha)
        return dvals, dX, dY, None, None, None


def _bsr_transpose(A: BSRMatrix, dev: torch.device) -> BSRMatrix:
    """A^T as a BSRMatrix on ``dev``: the transposed block pattern built on
    the device (``trnsparse_csr_transpose`` over the block pointers) and the
    blocks gathered and transposed by ``trnsparse_bsr_blocks_transpose``. One
    cache slot per matrix, keyed by the fingerprint of A's blocks and indices
    and replaced when they change (so repeated in-place updates of A.blocks
    never accumulate copies)."""
    from .formats import _fingerprint

    key = ("bsr_transpose", str(dev))
    fp = _fingerprint(A.blocks, A.block_col_indices, A.block_row_ptrs)
    hit = A._dev.get(key)
    if hit is not None and hit[0] == fp:
        return hit[1]
    A._dev.pop(key, None)  # free the old transpose before building the new one
    b = A.block_size
    lay = A.device_layout(dev)
    R = lay["row_ptr"].numel() - 1
    Cn = -(-A.shape[1] // b)
    rpt, colt, perm, _ = _transpose_structure(lay["row_ptr"], lay["col_idx"], R, Cn, False, A._dev, dev)
    blocks = lay["blocks"]
    bt = torch.empty_like(blocks)
    if A.n_blocks:
        with torch.cuda.device(dev):
            _lib.call("trnsparse_bsr_blocks_transpose", A.n_blocks, b, blocks.element_size(), blocks.data_ptr(),
                      perm.data_ptr(), bt.data_ptr(), _lib.stream_handle(dev))
    AT = BSRMatrix(blocks=bt, block_col_indices=colt, block_row_ptrs=rpt, shape=(A.shape[1], A.shape[0]),
                   block_size=b)
    A._dev[key] = (fp, AT)
    return AT


def _nt_tc(X: torch.Tensor, Y: torch.Tensor, tiles: torch.Tensor | None, out: torch.Tensor, out_rows: int = 0,
           out_cols: int = 0, mask_kind: int = 0, bounds: torch.Tensor | None = None, ldq: int = 0,
           threshold: float = 0.0) -> None:
    """``trnsparse_nt_tc``: 128 x 128 tiles of X Y^T on the tensor cores (X, Y row-major,
    contraction along the rows; fp32 3xTF32 or bf16)."""
    dev = X.device
    code = _lib.dtype_code(X.dtype)
    mx, K = X.shape
    my = Y.shape[0]
    ws_bytes = _lib.raw("trnsparse_nt_tc_workspace_size")(mx, my, K, code)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    n_tiles = tiles.shape[0] if tiles is not None else 0
    with torch.cuda.device(dev):
        _lib.call("trnsparse_nt_tc", mx, my, K, code, X.data_ptr(), X.stride(0), Y.data_ptr(), Y.stride(0),
                  _lib.ptr(tiles), n_tiles, out.data_ptr(), out.stride(0) if out.dim() == 2 else out.shape[-1],
                  _lib.dtype_code(out.dtype), out_rows, out_cols, mask_kind, _lib.ptr(bounds), ldq, float(threshold),
                  ws.data_ptr(), ws_bytes, _lib.stream_handle(dev))


def _bsr_blocks_grad(A: BSRMatrix, dC: torch.Tensor, B: torch.Tensor) -> torch.Tensor:
    """dblocks[k] = dC[rows of block-row i] @ B[rows of block-column j]^T for
    stored block k = (i, j) (the reference's _BSRSpMMFunction.backward,
    nki/dispatch.py:331-369). Block size 128 with float32 / bfloat16 blocks:
    one tensor-core launch over the stored blocks (``trnsparse_nt_tc``, the
    dC and B tiles read in place); other block sizes: a batched product over
    gathered row blocks."""
    b = A.block_size
    dev = dC.device if dC.is_cuda else _dev_of(B)
    if b == 128 and A.dtype in (torch.float32, torch.bfloat16):
        lay = A.device_layout(dev)
        tiles = lay.get("block_tiles")
        if tiles is None:
            rp, ci = lay["host_row_ptr"], lay["host_col_idx"]
            rows = torch.repeat_interleave(torch.arange(rp.numel() - 1), rp[1:] - rp[:-1])
            tiles = lay["block_tiles"] = torch.stack([rows, ci], 1).to(device=dev, dtype=torch.int32).contiguous()
        X = _on(dC, dev, A.dtype)
        Y = _on(B, dev, A.dtype)
        out = torch.empty(A.n_blocks, b, b, dtype=A.dtype, device=dev)
        if A.n_blocks:
            _nt_tc(X, Y, tiles, out)
        return out.to(A.blocks.device)
    R = A.block_row_ptrs.numel() - 1
    Cn = -(-A.shape[1] // b)
    k = dC.shape[1]
    dCp = torch.zeros(R * b, k, dtype=torch.float32, device=dev)
    dCp[: dC.shape[0]] = dC.float()
    Bp = torch.zeros(Cn * b, k, dtype=torch.float32, device=dev)
    Bp[: B.shape[0]] = B.to(dev).float()
    rp = A.block_row_ptrs.to(device=dev, dtype=torch.long)
    rows = torch.repeat_interleave(torch.arange(R, device=dev), rp[1:] - rp[:-1])
    cols = A.block_col_indices.to(device=dev, dtype=torch.long)
    g = torch.bmm(dCp.view(R, b, k)[rows], Bp.view(Cn, b, k)[cols].transpose(1, 2))
    return g.to(dtype=A.blocks.dtype, device=A.blocks.device)


class _BsrSpmmFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, blocks, B, A):
        ctx.A = A
        ctx.save_for_backward(B)
        return _bsr_spmm_impl(A, B)

    @staticmethod
    def backward(ctx, dC):
        A = ctx.A
        (B,) = ctx.saved_tensors
        dblocks = dB = None
        if ctx.needs_input_grad[1]:
            g = dC.contiguous()
            dB = _bsr_spmm_impl(_bsr_transpose(A, g.device if g.is_cuda else _dev_of(g)), g).to(B.dtype)
            dB = dB.to(B.device)
        if ctx.needs_input_grad[0]:
            dblocks = _bsr_blocks_grad(A, dC, B)
        return dblocks, dB, None


def bsr_spmm_cuda_core(A: BSRMatrix, B: torch.Tensor) -> torch.Tensor:
    """``A @ B`` on the CUDA-core kernel (fp32 FMA): a second, independent
    device implementation used to cross-check the tensor-core path."""
    m, n = A.shape
    dev = _dev_of(B)
    Bd = _on(B, dev, torch.float32)
    out = torch.empty(m, B.shape[1], dtype=torch.float32, device=dev)
    geo = _bsr_geometry(A, dev)
    with torch.cuda.device(dev):
        _lib.call("trnsparse_bsr_spmm_simt", *geo, Bd.data_ptr(), B.shape[1], B.shape[1], out.data_ptr(),
                  B.shape[1], _lib.stream_handle(dev))
    return _back(out, B)


# ---------------------------------------------------------------------------
# Screened SpMM
# ---------------------------------------------------------------------------


def screened_spmm(
    A: torch.Tensor,
    diag_integrals: torch.Tensor,
    B: torch.Tensor,
    threshold: float,
) -> torch.Tensor:
    """``C = (A * mask) @ B`` with the Schwarz mask applied inside the kernel
    (reference: trnsparse/ops.py:213-277).

    1-D ``diag_integrals`` (the reference's signature, square A):
    ``Q = sqrt(|d|)``, ``mask[i,j] = Q[i]*Q[j] > sqrt(threshold)``.
    2-D ``diag_integrals`` (extension): the already-computed pair bounds
    ``Q = schwarz_bounds(G)``; ``mask = screen_quartets(Q, threshold)``,
    i.e. ``Q > sqrt(threshold)`` (trnsparse/screening.py:29-40).
    Comparisons are in float32, like the reference's tensor comparisons.
    Differentiable in ``A`` and ``B`` (the mask is discrete, as in the
    reference's _ScreenedSpMMFunction, nki/dispatch.py:447-484): dB runs the
    same kernel on A^T with the transposed mask; dA = (dC B^T) o mask.
    """
    if _needs_grad(A, B):
        return _ScreenedFn.apply(A, B, diag_integrals, float(threshold))
    return _screened_impl(A, diag_integrals, B, threshold)


class _ScreenedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, A, B, diag_integrals, threshold):
        ctx.threshold = threshold
        ctx.save_for_backward(A, B, diag_integrals)
        return _screened_impl(A, diag_integrals, B, threshold)

    @staticmethod
    def backward(ctx, dC):
        A, B, Q = ctx.saved_tensors
        thr = ctx.threshold
        dA = dB = None
        if ctx.needs_input_grad[1]:
            Qt = Q if Q.dim() == 1 else Q.t().contiguous()  # the 1-D mask is symmetric
            dB = _screened_impl(A.detach().t().contiguous(), Qt, dC.contiguous(), thr).to(B.device)
        if ctx.needs_input_grad[0]:
            # dA = (dC B^T) o mask, one tensor-core launch with the mask in its epilogue
            dev = dC.device if dC.is_cuda else _dev_of(B)
            X = _on(dC, dev, torch.float32)
            Y = _on(B, dev, torch.float32)
            Qd = _on(Q, dev, torch.float32)
            M, K = A.shape
            Kp = -(-K // 4) * 4
            dA = torch.empty(M, Kp, dtype=torch.float32, device=dev)
            _nt_tc(X, Y, None, dA, M, K, 1 if Qd.dim() == 1 else 2, Qd, Qd.stride(0) if Qd.dim() == 2 else 0, thr)
            if Kp != K:
                dA = dA[:, :K].contiguous()
            dA = dA.to(A.device)
        return dA, dB, None, None


def _screened_impl(A: torch.Tensor, diag_integrals: torch.Tensor, B: torch.Tensor, threshold: float) -> torch.Tensor:
    M, K = A.shape
    if diag_integrals.dim() == 1:
        assert diag_integrals.shape[0] == M == K, (
            "screened_spmm requires square A with diag_integrals of matching length; "
            f"got A shape {A.shape}, diag_integrals shape {diag_integrals.shape}"
        )
        kind = 1
    else:
        assert diag_integrals.dim() == 2 and tuple(diag_integrals.shape) == (M, K), (
            f"2-D bounds must match A: got {tuple(diag_integrals.shape)} for A {tuple(A.shape)}"
        )
        kind = 2
    assert B.shape[0] == K, f"Dimension mismatch: A is {tuple(A.shape)}, B is {tuple(B.shape)}"
    if A.dtype != torch.float32:
        raise TypeError(f"screened_spmm: dtype {A.dtype} not supported (float32)")
    N = B.shape[1]
    dev = _dev_of(A, B, diag_integrals)
    Ad = _on(A, dev, torch.float32)
    Qd = _on(diag_integrals, dev, torch.float32)
    Bd = _on(B, dev, torch.float32)
    if K % 4 or Ad.data_ptr() % 16 or Qd.data_ptr() % 16:
        # TMA needs 16-byte row strides and bases: pad K to a multiple of 4 with zero columns
        Kp = -(-K // 4) * 4
        Ap = torch.zeros(M, Kp, device=dev)
        Ap[:, :K] = Ad
        Ad = Ap
        if kind == 2:
            Qp = torch.zeros(M, Kp, device=dev)
            Qp[:, :K] = Qd
            Qd = Qp
    Np = -(-N // 4) * 4  # C rows 16-byte aligned for the kernel's TMA stores
    out = torch.empty(M, Np, dtype=torch.float32, device=dev)
    ws_bytes = _lib.raw("trnsparse_screened_spmm_workspace_size")(K, N)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.call("trnsparse_screened_spmm", M, K, N, Ad.data_ptr(), Ad.shape[1], Qd.data_ptr(), kind,
                  Qd.shape[-1] if kind == 2 else 0, float(threshold), Bd.data_ptr(), N, out.data_ptr(), Np,
                  ws.data_ptr(), ws_bytes, _lib.stream_handle(dev))
    if Np != N:
        out = out[:, :N].contiguous()
    return _back(out, B)


# ---------------------------------------------------------------------------
# Block-sparse attention
# ---------------------------------------------------------------------------


def _attn_tc_ok(dtype, b, seq, hd, heads) -> bool:
    """Shapes the tensor-core attention kernels (forward and backward) take."""
    return dtype == torch.bfloat16 and b == 128 and hd in (64, 128) and seq % 128 == 0 and heads > 0


def _attn_forward(Q, K, V, mask_bsr, scale, cuda_cores: bool = False, want_lse: bool = False):
    """Device forward for (S, D) or (..., S, D) inputs sharing one mask.

    bf16 with block size 128, head_dim 64/128 and seq a multiple of 128 runs
    the tensor-core kernel; everything else (and ``cuda_cores=True``) runs
    the CUDA-core kernel. ``want_lse``: return ``(O, lse)`` with the rows'
    base-2 log-sum-exp from the tensor-core kernel (None otherwise)."""
    seq, hd = Q.shape[-2], Q.shape[-1]
    if Q.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"block_sparse_attention_tiled: dtype {Q.dtype} not supported (float32, bfloat16)")
    dev = _dev_of(Q, K, V)
    lay = mask_bsr.device_layout(dev) if hasattr(mask_bsr, "device_layout") else None
    if lay is not None:
        rp, ci = lay["row_ptr"], lay["col_idx"]
    else:
        rp = mask_bsr.block_row_ptrs.to(device=dev, dtype=torch.int32).contiguous()
        ci = mask_bsr.block_col_indices.to(device=dev, dtype=torch.int32).contiguous()
    b = mask_bsr.block_size
    if rp.shape[0] < seq // b + 1:
        raise AssertionError(f"mask has {rp.shape[0] - 1} block-rows, seq {seq} needs {seq // b}")
    Qd, Kd, Vd = (_on(t, dev, Q.dtype) for t in (Q, K, V))
    heads = Qd.numel() // (seq * hd) if seq * hd else 0
    O = torch.empty_like(Qd)
    code = _lib.F32 if Q.dtype == torch.float32 else _lib.BF16
    tc = not cuda_cores and _attn_tc_ok(Q.dtype, b, seq, hd, heads)
    lse = None
    with torch.cuda.device(dev):
        if tc:
            if want_lse:
                lse = torch.empty(heads * seq, dtype=torch.float32, device=dev)
            _lib.call("trnsparse_bsr_attention_tc_lse", heads, seq, hd, rp.data_ptr(), ci.data_ptr(), Qd.data_ptr(),
                      Kd.data_ptr(), Vd.data_ptr(), O.data_ptr(), lse.data_ptr() if lse is not None else None,
                      float(scale), _lib.stream_handle(dev))
        else:
            _lib.call("trnsparse_bsr_attention", heads, seq, hd, b, rp.data_ptr(), ci.data_ptr(), Qd.data_ptr(),
                      Kd.data_ptr(), Vd.data_ptr(), O.data_ptr(), code, float(scale), _lib.stream_handle(dev))
    return (O, lse) if want_lse else O


def _mask_indices(mask_bsr, dev):
    """Block-row pointers / column indices of the mask and its transposed
    pattern (column pointers / row indices), int32 on ``dev``; cached with the
    mask's device layout when it has one."""
    lay = mask_bsr.device_layout(dev) if hasattr(mask_bsr, "device_layout") else {}
    hit = lay.get("attn_csc")
    if hit is not None:
        return hit
    rp_h = mask_bsr.block_row_ptrs.to(torch.int64).cpu()
    ci_h = mask_bsr.block_col_indices.to(torch.int64).cpu()
    n_rows = rp_h.numel() - 1
    n_cols = -(-mask_bsr.shape[1] // mask_bsr.block_size)
    rows = torch.repeat_interleave(torch.arange(n_rows), rp_h[1:] - rp_h[:-1])
    order = torch.argsort(ci_h * max(n_rows, 1) + rows, stable=True)
    cp_h = torch.zeros(n_cols + 1, dtype=torch.int64)
    cp_h[1:] = torch.cumsum(torch.bincount(ci_h, minlength=n_cols)[:n_cols], 0)
    out = tuple(t.to(device=dev, dtype=torch.int32).contiguous() for t in (rp_h, ci_h, cp_h, rows[order]))
    out = out + (int((cp_h[1:] - cp_h[:-1]).max().item()) if n_cols > 0 else 0,)
    if lay is not None and hasattr(mask_bsr, "device_layout"):
        lay["attn_csc"] = out
    return out


_ATTN_BWD_SPLIT = int(os.environ.get("TRNSPARSE_ATTN_BWD_SPLIT", "16"))


def _attn_bwd_plan(mask_bsr, dev, rp, cp):
    """Host-built unit plan of the tensor-core backward (row units, column
    units, aux entries), cached with the mask's device layout."""
    lay = mask_bsr.device_layout(dev) if hasattr(mask_bsr, "device_layout") else {}
    key = ("attn_bwd_plan", _ATTN_BWD_SPLIT)
    hit = lay.get(key) if lay is not None else None
    if hit is not None:
        return hit
    rp_h = rp.cpu().contiguous()
    cp_h = cp.cpu().contiguous()
    counts = (ctypes.c_int64 * 4)()
    args = (rp_h.numel() - 1, cp_h.numel() - 1, rp_h.data_ptr(), cp_h.data_ptr(), _ATTN_BWD_SPLIT)
    _lib.call("trnsparse_bsr_attention_backward_tc_plan", *args, None, 0, counts)
    n = 4 * (counts[0] + counts[1] + counts[2])
    plan = torch.zeros(max(n, 4), dtype=torch.int32)
    _lib.call("trnsparse_bsr_attention_backward_tc_plan", *args, plan.data_ptr(), plan.numel(), counts)
    out = (plan.to(dev), tuple(int(c) for c in counts))
    if lay is not None and hasattr(mask_bsr, "device_layout"):
        lay[key] = out
    return out


def _attn_backward(Q, K, V, O, dO, mask_bsr, scale, lse=None, cuda_cores: bool = False):
    """Device backward (reference: ops.py:360-473). bf16 shapes the tensor
    cores take run the tcgen05 kernels (dQ row-first, dK/dV column-first,
    with the forward's log-sum-exp ``lse`` when given); everything else (and
    ``cuda_cores=True``) runs the CUDA-core stats, dQ and dK/dV kernels."""
    seq, hd = Q.shape[-2], Q.shape[-1]
    dev = Q.device
    rp, ci, cp, ri, max_col = _mask_indices(mask_bsr, dev)
    b = mask_bsr.block_size
    Qd, Kd, Vd, Od, dOd = (t.to(device=dev, dtype=Q.dtype).contiguous() for t in (Q, K, V, O, dO))
    heads = Qd.numel() // (seq * hd) if seq * hd else 0
    dQ, dK, dV = torch.empty_like(Qd), torch.empty_like(Kd), torch.empty_like(Vd)
    if not cuda_cores and _attn_tc_ok(Q.dtype, b, seq, hd, heads) and rp.numel() - 1 == seq // b and cp.numel() - 1 == seq // b:
        plan, (n_ru, n_cu, n_aux, n_slots) = _attn_bwd_plan(mask_bsr, dev, rp, cp)
        ws_bytes = _lib.raw("trnsparse_bsr_attention_backward_tc_workspace_size")(heads, seq, hd, n_slots)
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            _lib.call("trnsparse_bsr_attention_backward_tc", heads, seq, hd, rp.data_ptr(), ci.data_ptr(),
                      ri.data_ptr(), plan.data_ptr(), n_ru, n_cu, n_aux, n_slots, Qd.data_ptr(), Kd.data_ptr(),
                      Vd.data_ptr(), Od.data_ptr(), dOd.data_ptr(), lse.data_ptr() if lse is not None else None,
                      dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), float(scale), ws.data_ptr(), ws_bytes,
                      _lib.stream_handle(dev))
        return dQ, dK, dV
    code = _lib.F32 if Q.dtype == torch.float32 else _lib.BF16
    ws_bytes = _lib.raw("trnsparse_bsr_attention_backward_workspace_size")(heads, seq, hd, code, max_col)
    ws = torch.empty(max(ws_bytes, 4), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.call("trnsparse_bsr_attention_backward", heads, seq, hd, b, rp.data_ptr(), ci.data_ptr(), cp.data_ptr(),
                  ri.data_ptr(), max_col, Qd.data_ptr(), Kd.data_ptr(), Vd.data_ptr(), Od.data_ptr(), dOd.data_ptr(),
                  dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), code, float(scale), ws.data_ptr(), ws_bytes,
                  _lib.stream_handle(dev))
    return dQ, dK, dV


class _AttnFunction(torch.autograd.Function):
    """Autograd wrapper (reference: ops.py:476-546). Forward and backward
    both run CUDA kernels; the backward follows the reference's Flash-delta
    formulas (ops.py:360-473) over the stored blocks only."""

    @staticmethod
    def forward(ctx, Q, K, V, mask_bsr, scale):
        O, lse = _attn_forward(Q, K, V, mask_bsr, scale, want_lse=True)
        ctx.save_for_backward(Q, K, V, O, lse)
        ctx.mask_bsr, ctx.scale = mask_bsr, scale
        return O

    @staticmethod
    def backward(ctx, dO):
        Q, K, V, O, lse = ctx.saved_tensors
        dQ, dK, dV = _attn_backward(Q, K, V, O, dO, ctx.mask_bsr, ctx.scale, lse=lse)
        return dQ.view_as(Q), dK.view_as(K), dV.view_as(V), None, None


def block_sparse_attention_tiled(
    Q: torch.Tensor,
    K: torch.Tensor,
    V: torch.Tensor,
    mask_bsr: BSRMatrix,
    scale: float | None = None,
) -> torch.Tensor:
    """Block-sparse softmax attention over the stored blocks of ``mask_bsr``
    (reference: trnsparse/ops.py:549-625).

    ``Q, K, V``: ``(seq_len, head_dim)`` as in the reference, or with leading
    batch/head dimensions ``(..., seq_len, head_dim)`` sharing one mask.
    Only the mask's pattern is used. ``scale`` defaults to
    ``head_dim ** -0.5``. float32 or bfloat16 in, same dtype out; softmax in
    float32. Differentiable (backward on the device, see ``_AttnFunction``).
    """
    head_dim = Q.shape[-1]
    if scale is None:
        scale = head_dim**-0.5
    if torch.is_grad_enabled() and (Q.requires_grad or K.requires_grad or V.requires_grad):
        out = _AttnFunction.apply(Q, K, V, mask_bsr, scale)
    else:
        out = _attn_forward(Q, K, V, mask_bsr, scale)
    return out if Q.is_cuda else out.to(Q.device)
