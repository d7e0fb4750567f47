"""CPU oracle: restatement of trnsci/trnsparse v0.6.0's PyTorch CPU path.

Test infrastructure only (see oracle/__init__.py). All functions take and
return CPU torch tensors and raw format arrays, so they do not depend on the
product package.
"""

from __future__ import annotations

import math

import torch

__all__ = [
    "csr_spmm_backward",
    "bsr_spmm_backward",
    "screened_spmm_backward",
    "csr_spmv_symmetric",
    "csr_spmv",
    "csr_spmm",
    "csr_from_dense",
    "bsr_from_dense",
    "bsr_to_dense",
    "bsr_spmm",
    "schwarz_bounds",
    "screen_quartets",
    "screened_spmm",
    "screened_spmm_pair",
    "block_sparse_attention",
    "block_sparse_attention_backward",
    "bsr_diagonal",
    "bsr_matvec",
    "cg_bsr",
    "jacobi_inv_diag",
    "chebyshev_coeffs",
    "chebyshev_bsr",
    "richardson_bsr",
    "power_iteration_bsr",
]


# --------------------------------------------------------------------------- CSR
def csr_spmv(row_ptrs, col_indices, values, shape, x, alpha=1.0, y=None, beta=0.0):
    """trnsparse/ops.py:30-48: alpha * (csr @ x), then + beta*y if y given and beta != 0."""
    A = torch.sparse_csr_tensor(row_ptrs, col_indices, values, size=shape)
    out = alpha * (A @ x)
    if y is not None and beta != 0.0:
        out = out + beta * y
    return out


def csr_spmm(row_ptrs, col_indices, values, shape, B, alpha=1.0, C=None, beta=0.0):
    """trnsparse/ops.py:51-78 (PyTorch branch)."""
    A = torch.sparse_csr_tensor(row_ptrs, col_indices, values, size=shape)
    out = alpha * (A @ B)
    if C is not None and beta != 0.0:
        out = out + beta * C
    return out


def csr_spmv_symmetric(row_ptrs, col_indices, values, shape, x, alpha=1.0):
    """trnsparse/ops.py:81-104: alpha * (A @ x + strict(A)^T @ x), strict(A) = the
    stored entries off the diagonal, summed as a coalesced COO tensor."""
    m, n = shape
    assert m == n, "Matrix must be square for symmetric SpMV"
    rows = torch.repeat_interleave(torch.arange(m), row_ptrs[1:] - row_ptrs[:-1])
    off = rows != col_indices
    A = torch.sparse_csr_tensor(row_ptrs, col_indices, values, size=shape)
    strict = torch.sparse_coo_tensor(torch.stack([rows[off], col_indices[off]]), values[off], size=shape).coalesce()
    return alpha * (A @ x + strict.t() @ x)


def csr_from_dense(A, threshold=0.0):
    """trnsparse/formats.py:269-278 + COO.to_csr (formats.py:104-124).

    Returns (values, col_indices int64, row_ptrs int64)."""
    m, n = A.shape
    keep = torch.abs(A) > threshold
    rows, cols = torch.where(keep)
    vals = A[keep]
    order = torch.argsort(rows * n + cols, stable=True)
    rows, cols, vals = rows[order], cols[order], vals[order]
    row_ptrs = torch.zeros(m + 1, dtype=torch.long)
    for r in rows.tolist():
        row_ptrs[r + 1] += 1
    return vals, cols, torch.cumsum(row_ptrs, 0)


# --------------------------------------------------------------------------- BSR
def bsr_from_dense(A, block_size=128, threshold=0.0):
    """trnsparse/formats.py:184-221. Returns (blocks, block_col_indices, block_row_ptrs)."""
    b = block_size
    m, n = A.shape
    mp, np_ = -(-m // b) * b, -(-n // b) * b
    P = torch.zeros(mp, np_, dtype=A.dtype)
    P[:m, :n] = A
    mb, nbc = mp // b, np_ // b
    blocks, cols, ptrs = [], [], [0]
    for i in range(mb):
        for j in range(nbc):
            blk = P[i * b : (i + 1) * b, j * b : (j + 1) * b]
            if blk.abs().max() > threshold:
                blocks.append(blk.clone())
                cols.append(j)
        ptrs.append(len(cols))
    blocks_t = torch.stack(blocks) if blocks else torch.zeros(0, b, b, dtype=A.dtype)
    return blocks_t, torch.tensor(cols, dtype=torch.long), torch.tensor(ptrs, dtype=torch.long)


def bsr_to_dense(blocks, block_col_indices, block_row_ptrs, shape, block_size):
    """trnsparse/formats.py:233-251."""
    m, n = shape
    b = block_size
    mp, np_ = -(-m // b) * b, -(-n // b) * b
    D = torch.zeros(mp, np_, dtype=blocks.dtype)
    for i in range(mp // b):
        for k in range(int(block_row_ptrs[i]), int(block_row_ptrs[i + 1])):
            j = int(block_col_indices[k])
            D[i * b : (i + 1) * b, j * b : (j + 1) * b] = blocks[k]
    return D[:m, :n].contiguous()


def bsr_spmm(blocks, block_col_indices, block_row_ptrs, shape, block_size, B):
    """trnsparse/ops.py:162-192: out[i] += blocks[idx] @ B[j*b:(j+1)*b] per stored block."""
    m, n = shape
    b = block_size
    k = B.shape[1]
    mp, np_ = -(-m // b) * b, -(-n // b) * b
    if B.shape[0] != n:
        raise AssertionError(f"Dimension mismatch: A is {shape}, B is {tuple(B.shape)}")
    Bp = torch.zeros(np_, k, dtype=B.dtype)
    Bp[:n] = B
    out = torch.zeros(mp, k, dtype=blocks.dtype)
    rp = block_row_ptrs.tolist()
    ci = block_col_indices.tolist()
    for i in range(mp // b):
        for idx in range(rp[i], rp[i + 1]):
            j = ci[idx]
            out[i * b : (i + 1) * b] += blocks[idx] @ Bp[j * b : (j + 1) * b]
    return out[:m]


# --------------------------------------------------------------------------- screening
def schwarz_bounds(diag):
    """trnsparse/screening.py:17-26."""
    return torch.sqrt(torch.abs(diag))


def screen_quartets(Q, threshold=1e-10):
    """trnsparse/screening.py:29-40: threshold**0.5 < Q."""
    return threshold**0.5 < Q


def screened_spmm(A, diag_integrals, B, threshold):
    """trnsparse/ops.py:255-277 (1-D bound vector, PyTorch branch)."""
    assert diag_integrals.dim() == 1
    M, K = A.shape
    assert diag_integrals.shape[0] == M == K
    Q = torch.sqrt(torch.abs(diag_integrals))
    mask = Q.unsqueeze(-1) * Q.unsqueeze(0) > math.sqrt(threshold)
    return (A * mask.to(A.dtype)) @ B


def screened_spmm_pair(A, Q, B, threshold):
    """2-D pair-bound form: (A * screen_quartets(Q, threshold)) @ B (screening.py:29-40)."""
    return (A * screen_quartets(Q, threshold).to(A.dtype)) @ B


# --------------------------------------------------------------------------- product adjoints
def csr_spmm_backward(dense, B, dC):
    """trnsparse/nki/dispatch.py:154-178 (_SpMMFunction.backward): the dense
    gradient dC @ B^T of the materialised A (the stored values' gradient is
    its restriction to A's pattern) and dB = A^T @ dC."""
    return dC @ B.T, dense.T @ dC


def bsr_spmm_backward(blocks, block_col_indices, block_row_ptrs, shape, block_size, B, dC):
    """trnsparse/nki/dispatch.py:331-369 (_BSRSpMMFunction.backward):
    dblocks[k] = dC[row block of k] @ B[col block of k]^T per stored block, and
    dB = A^T @ dC through the materialised dense A."""
    b = block_size
    m, n = shape
    rp = block_row_ptrs.tolist()
    ci = block_col_indices.tolist()
    dblocks = torch.zeros_like(blocks)
    for i in range(len(rp) - 1):
        for k in range(rp[i], rp[i + 1]):
            j = ci[k]
            dblocks[k] = dC[i * b : (i + 1) * b] @ B[j * b : (j + 1) * b].T
    dense = bsr_to_dense(blocks, block_col_indices, block_row_ptrs, shape, b)
    return dblocks, dense.T @ dC


def screened_spmm_backward(A, diag_integrals, B, threshold, dC):
    """trnsparse/nki/dispatch.py:447-484 (_ScreenedSpMMFunction.backward), 1-D
    bounds: mask = sqrt|d_i| sqrt|d_j| > sqrt(threshold);
    dA = (dC @ B^T) * mask, dB = (A * mask)^T @ dC."""
    Q = torch.sqrt(torch.abs(diag_integrals))
    m = ((Q.unsqueeze(-1) * Q.unsqueeze(0)) > math.sqrt(threshold)).to(A.dtype)
    return (dC @ B.T) * m, (A * m).T @ dC


# --------------------------------------------------------------------------- attention
def block_sparse_attention(Q, K, V, block_row_ptrs, block_col_indices, block_size, scale=None):
    """trnsparse/ops.py:280-357: two-pass block-sparse softmax attention.

    Pass 1 keeps per-block row max and stable exp-sum; the host reduction
    combines them into row max / denominator (clamped at 1e-12; empty block
    rows get max 0 and output 0); pass 2 recomputes scores and accumulates
    exp(s - max) / denom @ V. Computes in Q's dtype.
    """
    seq_len, head_dim = Q.shape
    if scale is None:
        scale = head_dim**-0.5
    b = block_size
    mt = seq_len // b
    rp = [int(v) for v in block_row_ptrs.tolist()]
    ci = [int(v) for v in block_col_indices.tolist()]
    nb = len(ci)
    tmax = torch.full((nb, b), float("-inf"), dtype=Q.dtype)
    tsum = torch.zeros((nb, b), dtype=Q.dtype)
    for m in range(mt):
        q = Q[m * b : (m + 1) * b]
        for idx in range(rp[m], rp[m + 1]):
            c = ci[idx]
            s = (q @ K[c * b : (c + 1) * b].T) * scale
            tmax[idx] = s.max(dim=1).values
            tsum[idx] = torch.exp(s - tmax[idx].unsqueeze(1)).sum(dim=1)
    rmax = torch.full((seq_len,), float("-inf"), dtype=Q.dtype)
    rden = torch.zeros(seq_len, dtype=Q.dtype)
    for m in range(mt):
        sl = slice(m * b, (m + 1) * b)
        if rp[m] == rp[m + 1]:
            rmax[sl] = 0.0
            continue
        rmax[sl] = tmax[rp[m] : rp[m + 1]].max(dim=0).values
        for idx in range(rp[m], rp[m + 1]):
            rden[sl] += tsum[idx] * torch.exp(tmax[idx] - rmax[sl])
    rden = rden.clamp(min=1e-12)
    out = torch.zeros(seq_len, head_dim, dtype=Q.dtype)
    for m in range(mt):
        sl = slice(m * b, (m + 1) * b)
        q = Q[sl]
        for idx in range(rp[m], rp[m + 1]):
            c = ci[idx]
            s = (q @ K[c * b : (c + 1) * b].T) * scale
            w = torch.exp(s - rmax[sl].unsqueeze(1)) / rden[sl].unsqueeze(1)
            out[sl] += w @ V[c * b : (c + 1) * b]
    return out


# --------------------------------------------------------------------------- solvers
def block_sparse_attention_backward(Q, K, V, O, dO, block_row_ptrs, block_col_indices, block_size, scale=None):
    """trnsparse/ops.py:360-473 (the recompute path: no saved row statistics).

    D = rowsum(dO o O); row max and denominator recomputed in two passes over
    the stored blocks (empty block rows: max 0), denominator clamped at
    1e-12; then per stored block P = exp(s - max) / denom, dP = dO V^T,
    dS = P (dP - D), dQ += dS K scale, dK += dS^T Q scale, dV += P^T dO.
    Returns (dQ, dK, dV) in Q's dtype.
    """
    seq_len, head_dim = Q.shape
    if scale is None:
        scale = head_dim**-0.5
    b = block_size
    mt = seq_len // b
    rp = [int(v) for v in block_row_ptrs.tolist()]
    ci = [int(v) for v in block_col_indices.tolist()]
    D = (dO * O).sum(dim=-1)
    rmax = torch.full((seq_len,), float("-inf"), dtype=Q.dtype)
    for m in range(mt):
        sl = slice(m * b, (m + 1) * b)
        if rp[m] == rp[m + 1]:
            rmax[sl] = 0.0
            continue
        q = Q[sl]
        rm = rmax[sl]
        for idx in range(rp[m], rp[m + 1]):
            c = ci[idx]
            s = (q @ K[c * b : (c + 1) * b].T) * scale
            rm = torch.maximum(rm, s.max(dim=1).values)
        rmax[sl] = rm
    rden = torch.zeros(seq_len, dtype=Q.dtype)
    for m in range(mt):
        sl = slice(m * b, (m + 1) * b)
        q = Q[sl]
        for idx in range(rp[m], rp[m + 1]):
            c = ci[idx]
            s = (q @ K[c * b : (c + 1) * b].T) * scale
            rden[sl] += torch.exp(s - rmax[sl].unsqueeze(1)).sum(dim=1)
    rden = rden.clamp(min=1e-12)
    dQ, dK, dV = torch.zeros_like(Q), torch.zeros_like(K), torch.zeros_like(V)
    for m in range(mt):
        sl = slice(m * b, (m + 1) * b)
        q, do, d = Q[sl], dO[sl], D[sl]
        for idx in range(rp[m], rp[m + 1]):
            c = ci[idx]
            kb, vb = K[c * b : (c + 1) * b], V[c * b : (c + 1) * b]
            s = (q @ kb.T) * scale
            P = torch.exp(s - rmax[sl].unsqueeze(1)) / rden[sl].unsqueeze(1)
            dP = do @ vb.T
            dS = P * (dP - d.unsqueeze(1))
            dQ[sl] += dS @ kb * scale
            dK[c * b : (c + 1) * b] += dS.T @ q * scale
            dV[c * b : (c + 1) * b] += P.T @ do
    return dQ, dK, dV


def bsr_diagonal(blocks, block_col_indices, block_row_ptrs, shape, block_size):
    """trnsparse/iterative.py:22-41."""
    m = shape[0]
    b = block_size
    mt = -(-m // b)
    out = torch.zeros(mt * b, dtype=blocks.dtype)
    for i in range(mt):
        for k in range(int(block_row_ptrs[i]), int(block_row_ptrs[i + 1])):
            if int(block_col_indices[k]) == i:
                out[i * b : (i + 1) * b] = torch.diagonal(blocks[k])
                break
    return out[:m]


def bsr_matvec(bsr):
    """trnsparse/iterative.py:44-50: matvec = bsr_spmm(A, x[:, None])[:, 0]."""
    blocks, ci, rp, shape, b = bsr

    def mv(x):
        return bsr_spmm(blocks, ci, rp, shape, b, x.unsqueeze(1)).squeeze(1)

    return mv


def jacobi_inv_diag(bsr):
    """trnsparse/iterative.py:129-145 (returns inv_d; raises ValueError like the reference)."""
    d = bsr_diagonal(*bsr)
    if torch.any(d.abs() < 1e-15):
        raise ValueError("Jacobi preconditioner: diagonal has near-zero entries")
    return 1.0 / d


def cg_bsr(bsr, b, x0=None, tol=1e-6, max_iter=1000, inv_d=None, matvec=None, iters_cap=None):
    """trnsparse/iterative.py:53-126 (preconditioner given as Jacobi inv_d or None).

    ``iters_cap`` (oracle-only) stops after that many iterations for timing
    samples; the returned tuple is then a partial run.
    """
    n = b.shape[0]
    mv = matvec or bsr_matvec(bsr)
    x = x0.clone() if x0 is not None else torch.zeros(n, dtype=b.dtype)
    r = b - mv(x)
    b_norm = torch.linalg.norm(b).item()
    if b_norm < 1e-15:
        return x, 0, 0.0
    z = r * inv_d if inv_d is not None else r.clone()
    p = z.clone()
    rz = torch.dot(r, z).item()
    r_norm = float("nan")
    limit = max_iter if iters_cap is None else min(max_iter, iters_cap)
    for k in range(limit):
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
            return x, k + 1, rel
        z = r * inv_d if inv_d is not None else r
        rz_new = torch.dot(r, z).item()
        beta = rz_new / rz
        p = z + beta * p
        rz = rz_new
    return x, max_iter, r_norm / b_norm


def chebyshev_coeffs(lam_min, lam_max, K):
    """trnsparse/iterative.py:148-190 (fp64 recurrence, returned as float32)."""
    c = (lam_max - lam_min) / 2.0
    d = (lam_max + lam_min) / 2.0
    alpha = torch.zeros(K, dtype=torch.float64)
    beta = torch.zeros(K, dtype=torch.float64)
    a_prev = 1.0 / d
    alpha[0] = a_prev
    for k in range(1, K):
        bt = (c * a_prev / 2.0) ** 2
        a_new = 1.0 / (d - bt / a_prev)
        alpha[k] = a_new
        beta[k] = a_new * bt / a_prev
        a_prev = a_new
    return alpha.float(), beta.float()


def chebyshev_bsr(bsr, b, lam_min, lam_max, K=50, x0=None):
    """trnsparse/iterative.py:193-253."""
    n = b.shape[0]
    mv = bsr_matvec(bsr)
    x = x0.clone() if x0 is not None else torch.zeros(n, dtype=b.dtype)
    x_prev = x.clone()
    b_norm = torch.linalg.norm(b).item()
    alpha, beta = chebyshev_coeffs(lam_min, lam_max, K)
    for k in range(K):
        r = b - mv(x)
        x_new = x + alpha[k].item() * r
        if k > 0:
            x_new = x_new + beta[k].item() * (x - x_prev)
        x_prev = x
        x = x_new
    rel = torch.linalg.norm(b - mv(x)).item() / max(b_norm, 1e-15)
    return x, K, rel


def richardson_bsr(bsr, b, omega, K=100, x0=None):
    """trnsparse/iterative.py:256-295."""
    n = b.shape[0]
    mv = bsr_matvec(bsr)
    x = x0.clone() if x0 is not None else torch.zeros(n, dtype=b.dtype)
    b_norm = torch.linalg.norm(b).item()
    for _ in range(K):
        x = x + omega * (b - mv(x))
    rel = torch.linalg.norm(b - mv(x)).item() / max(b_norm, 1e-15)
    return x, K, rel


def power_iteration_bsr(bsr, v0, max_iter=100, tol=1e-9):
    """trnsparse/iterative.py:298-340 (v0 required: the oracle draws no random start)."""
    mv = bsr_matvec(bsr)
    v = v0.clone()
    v = v / torch.linalg.norm(v)
    lam_prev = 0.0
    lam = 0.0
    for k in range(max_iter):
        Av = mv(v)
        lam = torch.dot(v, Av).item()
        norm = torch.linalg.norm(Av).item()
        if norm < 1e-30:
            return 0.0, v, k + 1
        v = Av / norm
        if abs(lam - lam_prev) < tol:
            return lam, v, k + 1
        lam_prev = lam
    return lam, v, max_iter
