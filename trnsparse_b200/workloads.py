"""Seeded synthetic inputs for the five benchmark configurations.

Each builder returns CPU tensors drawn from a ``torch.Generator`` with the
stated seed, so the same inputs are produced on any machine. Shapes, value
distributions and sparsity patterns follow the benchmark definitions:

1. bsr_spmm: 16x16 grid of 128x128 blocks, all diagonal blocks present, each
   off-diagonal block present with p=0.25; block values and B ~ N(0,1);
   B is 2048x256.
2. CSR spmv/spmm: 5-point Poisson Laplacian on a 2048x2048 grid (4 on the
   diagonal, -1 off it), int32 row_ptr/col_idx, x ~ N(0,1); spmm B is n x 32.
3. screened_spmm: n centres uniform in [0,40]^3, G_ij = exp(-|ri-rj|^2/2)
   (float64, stored as float32), Q = sqrt(G), A = Q * N(0,1), B ~ N(0,1),
   threshold 1e-10.
4. block-sparse attention: 16 heads x 16384 x 128 bf16 N(0,1); block (i,j)
   of 128 tokens kept iff j <= i and (i - j < 8 or j < 2).
5. cg_bsr: SPD block-pentadiagonal BSR, 2048 block-rows of 128; diagonal
   blocks 10 I + (M + M^T)/2, off-diagonal blocks at offsets +-1, +-2 with
   A_ji = A_ij^T; all random entries N(0, 0.01), i.e. standard deviation 0.1;
   b ~ N(0,1).
"""

from __future__ import annotations

import numpy as np
import torch

from .formats import BSRMatrix, CSRMatrix


def bsr_random_grid(
    grid: int = 16, b: int = 128, p: float = 0.25, k: int = 256, seed: int = 0, dtype=torch.float32
) -> tuple[BSRMatrix, torch.Tensor]:
    """Config 1 (and scaled-up variants with a larger ``grid``)."""
    g = torch.Generator().manual_seed(seed)
    present = torch.rand(grid, grid, generator=g) < p
    present |= torch.eye(grid, dtype=torch.bool)
    rows, cols = present.nonzero(as_tuple=True)  # row-major order
    nb = rows.numel()
    blocks = torch.randn(nb, b, b, generator=g).to(dtype)
    row_ptrs = torch.zeros(grid + 1, dtype=torch.long)
    row_ptrs[1:] = torch.cumsum(present.sum(1), 0)
    B = torch.randn(grid * b, k, generator=g).to(dtype)
    A = BSRMatrix(blocks=blocks, block_col_indices=cols.clone(), block_row_ptrs=row_ptrs,
                  shape=(grid * b, grid * b), block_size=b)
    return A, B


def poisson2d_csr(n_grid: int = 2048, index_dtype=torch.int32) -> CSRMatrix:
    """5-point Laplacian on an n_grid x n_grid grid, row-major grid numbering."""
    N = n_grid
    n = N * N
    i = np.arange(n, dtype=np.int64)
    gy, gx = i // N, i % N
    # neighbours in ascending column order: up (i-N), left (i-1), self, right (i+1), down (i+N)
    offs = [(-N, gy > 0), (-1, gx > 0), (0, np.ones(n, bool)), (1, gx < N - 1), (N, gy < N - 1)]
    valid = np.stack([v for _, v in offs], axis=1)  # (n, 5)
    cols = np.stack([i + o for o, _ in offs], axis=1)
    vals = np.where(np.array([o for o, _ in offs])[None, :] == 0, 4.0, -1.0).astype(np.float32)
    vals = np.broadcast_to(vals, (n, 5))
    counts = valid.sum(1)
    row_ptrs = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(counts, out=row_ptrs[1:])
    npdt = np.int32 if index_dtype == torch.int32 else np.int64
    return CSRMatrix(
        values=torch.from_numpy(np.ascontiguousarray(vals[valid])),
        col_indices=torch.from_numpy(cols[valid].astype(npdt)),
        row_ptrs=torch.from_numpy(row_ptrs.astype(npdt)),
        shape=(n, n),
    )


def poisson_rhs(n: int, k: int | None = None, seed: int = 1) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, generator=g)
    if k is None:
        return x
    return torch.randn(n, k, generator=g)


def fock_like(n: int = 8192, k: int = 512, seed: int = 2, chunk: int = 1024):
    """Config 3: returns (A, Q, B, diag, threshold); Q is the 2-D pair bound."""
    g = torch.Generator().manual_seed(seed)
    r = torch.rand(n, 3, generator=g, dtype=torch.float64) * 40.0
    Q = torch.empty(n, n, dtype=torch.float32)
    for s in range(0, n, chunk):
        d2 = torch.cdist(r[s : s + chunk], r).pow_(2)
        Q[s : s + chunk] = torch.sqrt(torch.exp(-0.5 * d2).float())
    A = Q * torch.randn(n, n, generator=g)
    B = torch.randn(n, k, generator=g)
    diag = torch.ones(n)  # G_ii = exp(0) = 1: the 1-D bound vector of the reference signature
    return A, Q, B, diag, 1e-10


def sliding_window_mask(seq: int = 16384, b: int = 128, window: int = 8, n_global: int = 2) -> BSRMatrix:
    """Config 4 block mask as a BSRMatrix whose blocks are a zero-stride view (pattern only)."""
    mt = seq // b
    i = torch.arange(mt).unsqueeze(1)
    j = torch.arange(mt).unsqueeze(0)
    keep = (j <= i) & ((i - j < window) | (j < n_global))
    rows, cols = keep.nonzero(as_tuple=True)
    row_ptrs = torch.zeros(mt + 1, dtype=torch.long)
    row_ptrs[1:] = torch.cumsum(keep.sum(1), 0)
    blocks = torch.ones(1, 1, 1).expand(rows.numel(), b, b)
    return BSRMatrix(blocks=blocks, block_col_indices=cols.clone(), block_row_ptrs=row_ptrs,
                     shape=(seq, seq), block_size=b)


def attention_inputs(heads: int = 16, seq: int = 16384, hd: int = 128, seed: int = 3, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return tuple(torch.randn(1, heads, seq, hd, generator=g).to(dtype) for _ in range(3))


def block_pentadiagonal_spd(n_block_rows: int = 2048, b: int = 128, seed: int = 4, std: float = 0.1):
    """Config 5: returns (A, rhs)."""
    g = torch.Generator().manual_seed(seed)
    R = n_block_rows
    diag = torch.randn(R, b, b, generator=g) * std
    diag = 0.5 * (diag + diag.transpose(1, 2)) + 10.0 * torch.eye(b)
    up1 = torch.randn(max(R - 1, 0), b, b, generator=g) * std  # block (i, i+1)
    up2 = torch.randn(max(R - 2, 0), b, b, generator=g) * std  # block (i, i+2)
    cols, blocks, ptrs = [], [], [0]
    for i in range(R):
        for o in (-2, -1, 0, 1, 2):
            j = i + o
            if j < 0 or j >= R:
                continue
            cols.append(j)
            if o == 0:
                blocks.append(diag[i])
            elif o == 1:
                blocks.append(up1[i])
            elif o == 2:
                blocks.append(up2[i])
            elif o == -1:
                blocks.append(up1[j].T)
            else:
                blocks.append(up2[j].T)
        ptrs.append(len(cols))
    A = BSRMatrix(
        blocks=torch.stack(blocks).contiguous(),
        block_col_indices=torch.tensor(cols, dtype=torch.long),
        block_row_ptrs=torch.tensor(ptrs, dtype=torch.long),
        shape=(R * b, R * b),
        block_size=b,
    )
    rhs = torch.randn(R * b, generator=g)
    return A, rhs
