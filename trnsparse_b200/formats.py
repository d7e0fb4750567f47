"""Sparse formats: CSR, COO and BSR containers with a cached device layout.

The containers keep the reference's host-side semantics
(trnsparse/formats.py:21-301): same fields, same constructors, same
structure (block order, index dtypes, padding rules), so code written for
the reference works unchanged. What is new is ``device_layout()``: the first
time an op runs on a matrix, its index arrays and values are copied once to
the GPU in the layout the kernels stream (int32 or int64 indices, contiguous
``(n_blocks, b, b)`` blocks), and the copy is reused until a field is
replaced or modified in place.

Construction from a dense CUDA tensor (``BSRMatrix.from_dense``,
``from_dense``) and ``COOMatrix.to_csr`` of CUDA tensors run on the device
(csrc/formats.cu) and give the same structure and values as the host path
bit for bit; their results stay on the device.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch


def _threshold_in(dtype: torch.dtype, threshold: float) -> float:
    """``threshold`` rounded to ``dtype``: torch compares a tensor with a
    Python scalar in the tensor's dtype (``|v| > 0.1`` is false for the
    float32 0.1)."""
    return float(torch.tensor(float(threshold), dtype=torch.float64).to(dtype).to(torch.float64))


def _dense_args(A: torch.Tensor):
    """(A with unit column stride, its row stride, dtype code) for the C ABI."""
    from . import _lib

    if A.stride(-1) != 1 or (A.shape[0] > 1 and A.stride(0) < A.shape[1]):
        A = A.contiguous()
    lda = A.stride(0) if A.shape[0] > 1 else max(A.shape[1], 1)
    return A, lda, _lib.dtype_code(A.dtype)


_DEVICE_DENSE = (torch.float32, torch.bfloat16)


def _ceil_to(v: int, b: int) -> int:
    return (v + b - 1) // b * b


def _fingerprint(*ts: torch.Tensor) -> tuple:
    return tuple((t.data_ptr(), t._version, tuple(t.shape), t.dtype, t.device) for t in ts)


@dataclass
class CSRMatrix:
    """Compressed Sparse Row matrix (reference: trnsparse/formats.py:21-68).

    values: (nnz,); col_indices: (nnz,); row_ptrs: (m+1,); shape: (m, n).
    Index tensors may be int32 or int64.
    """

    values: torch.Tensor
    col_indices: torch.Tensor
    row_ptrs: torch.Tensor
    shape: tuple[int, int]
    _dev: dict = field(default_factory=dict, init=False, repr=False, compare=False)

    @property
    def nnz(self) -> int:
        return self.values.shape[0]

    @property
    def dtype(self) -> torch.dtype:
        return self.values.dtype

    @property
    def density(self) -> float:
        return self.nnz / (self.shape[0] * self.shape[1])

    def to_dense(self) -> torch.Tensor:
        """Dense (m, n) copy; duplicate entries add up (formats.py:48-51)."""
        return torch.sparse_csr_tensor(
            self.row_ptrs, self.col_indices, self.values, size=self.shape
        ).to_dense()

    def to_coo(self) -> COOMatrix:
        counts = (self.row_ptrs[1:] - self.row_ptrs[:-1]).to(torch.long).cpu()
        rows = torch.repeat_interleave(torch.arange(self.shape[0], dtype=torch.long), counts)
        return COOMatrix(
            values=self.values.clone(),
            row_indices=rows.to(self.values.device),
            col_indices=self.col_indices.clone(),
            shape=self.shape,
        )

    def device_layout(self, device: torch.device) -> dict[str, Any]:
        """Row pointers, column indices and values on ``device`` (cached).

        Both index arrays share one integer type: int32 if both are int32
        (the measured configuration), else int64.
        """
        key = str(device)
        fp = _fingerprint(self.values, self.col_indices, self.row_ptrs)
        hit = self._dev.get(key)
        if hit is not None and hit["fp"] == fp:
            return hit
        idx_t = (
            torch.int32
            if self.row_ptrs.dtype == torch.int32 and self.col_indices.dtype == torch.int32
            else torch.int64
        )
        lay = {
            "fp": fp,
            "row_ptrs": self.row_ptrs.to(device=device, dtype=idx_t).contiguous(),
            "col_indices": self.col_indices.to(device=device, dtype=idx_t).contiguous(),
            "values": self.values.to(device=device).contiguous(),
        }
        self._dev[key] = lay
        return lay

    def __repr__(self) -> str:
        return f"CSRMatrix(shape={self.shape}, nnz={self.nnz}, density={self.density:.4f})"


@dataclass
class COOMatrix:
    """Coordinate (triplet) matrix (reference: trnsparse/formats.py:71-126)."""

    values: torch.Tensor
    row_indices: torch.Tensor
    col_indices: torch.Tensor
    shape: tuple[int, int]

    @property
    def nnz(self) -> int:
        return self.values.shape[0]

    @property
    def dtype(self) -> torch.dtype:
        return self.values.dtype

    @property
    def density(self) -> float:
        return self.nnz / (self.shape[0] * self.shape[1])

    def to_dense(self) -> torch.Tensor:
        m, n = self.shape
        dense = torch.zeros(m, n, dtype=self.dtype, device=self.values.device)
        dense[self.row_indices, self.col_indices] = self.values
        return dense

    def to_csr(self) -> CSRMatrix:
        """Sort entries by (row, col) and compress rows (formats.py:104-124).
        Entries with equal (row, col) keep their order. CUDA tensors are
        converted on the device."""
        m, n = self.shape
        if self.values.is_cuda and self.values.dtype in (torch.float32, torch.float64, torch.bfloat16,
                                                          torch.float16):
            return self._to_csr_device()
        order = torch.argsort(self.row_indices * n + self.col_indices, stable=True)
        rows = self.row_indices[order]
        counts = torch.bincount(rows.to(torch.long).cpu(), minlength=m)[:m]
        row_ptrs = torch.zeros(m + 1, dtype=torch.long)
        row_ptrs[1:] = torch.cumsum(counts, dim=0)
        return CSRMatrix(
            values=self.values[order],
            col_indices=self.col_indices[order],
            row_ptrs=row_ptrs,
            shape=self.shape,
        )

    def _to_csr_device(self) -> CSRMatrix:
        from . import _lib

        m, n = self.shape
        dev = self.values.device
        rows = self.row_indices.to(device=dev, dtype=torch.int64).contiguous()
        cols = self.col_indices.to(device=dev, dtype=torch.int64).contiguous()
        vals = self.values.contiguous()
        nnz = vals.shape[0]
        row_ptrs = torch.empty(m + 1, dtype=torch.int64, device=dev)
        cols_out = torch.empty(nnz, dtype=torch.int64, device=dev)
        vals_out = torch.empty_like(vals)
        ws_bytes = _lib.raw("trnsparse_coo_to_csr_workspace_size")(m, nnz)
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            _lib.call("trnsparse_coo_to_csr", m, n, nnz, rows.data_ptr(), cols.data_ptr(), vals.data_ptr(),
                      _lib.dtype_code(vals.dtype), row_ptrs.data_ptr(), cols_out.data_ptr(), vals_out.data_ptr(),
                      ws.data_ptr(), ws_bytes, _lib.stream_handle(dev))
        return CSRMatrix(values=vals_out, col_indices=cols_out, row_ptrs=row_ptrs, shape=self.shape)

    def __repr__(self) -> str:
        return f"COOMatrix(shape={self.shape}, nnz={self.nnz}, density={self.density:.4f})"


@dataclass
class BSRMatrix:
    """Block-Sparse Row matrix (reference: trnsparse/formats.py:130-263).

    blocks: (nb, b, b); block_col_indices: (nb,); block_row_ptrs: (ceil(M/b)+1,);
    shape: (M, N) element shape (padding to whole blocks is implicit);
    block_size: b (default 128, the tile both the reference's Tensor Engine and
    the B200 tcgen05 path use).

    ``device_layout(device)`` returns (and caches) the GPU image the kernels
    stream: contiguous blocks, int32 ``block_row_ptr``/``block_col_idx``, and
    the derived per-kernel data (3xTF32 hi/lo split, work schedules) that the
    ops add under their own keys.
    """

    blocks: torch.Tensor
    block_col_indices: torch.Tensor
    block_row_ptrs: torch.Tensor
    shape: tuple[int, int]
    block_size: int = 128
    _dev: dict = field(default_factory=dict, init=False, repr=False, compare=False)

    @property
    def n_blocks(self) -> int:
        return self.blocks.shape[0]

    @property
    def nnz(self) -> int:
        return self.n_blocks * self.block_size * self.block_size

    @property
    def dtype(self) -> torch.dtype:
        return self.blocks.dtype

    @property
    def density(self) -> float:
        m, n = self.shape
        total = (m // self.block_size) * (n // self.block_size)
        return self.n_blocks / total if total else 0.0

    @classmethod
    def from_dense(cls, A: torch.Tensor, block_size: int = 128, threshold: float = 0.0) -> BSRMatrix:
        """Keep block (i, j) iff some |A| entry in it exceeds ``threshold``.

        Blocks are ordered row-major over the block grid, so column indices
        ascend within each block-row (formats.py:184-221). A float32 or
        bfloat16 CUDA tensor is screened and packed on the device.
        """
        b = block_size
        m, n = A.shape
        if A.is_cuda and A.dtype in _DEVICE_DENSE:
            return cls._from_dense_device(A, b, threshold)
        mp, np_ = _ceil_to(m, b), _ceil_to(n, b)
        if (mp, np_) != (m, n):
            Ap = A.new_zeros(mp, np_)
            Ap[:m, :n] = A
            A = Ap
        mb, nbc = mp // b, np_ // b
        grid = A.reshape(mb, b, nbc, b).transpose(1, 2)  # (mb, nbc, b, b) view
        keep = grid.abs().amax(dim=(-2, -1)) > threshold
        row_ptrs = torch.zeros(mb + 1, dtype=torch.long)
        row_ptrs[1:] = torch.cumsum(keep.sum(dim=1).cpu(), dim=0)
        where = keep.nonzero(as_tuple=False)
        return cls(
            blocks=grid[keep].contiguous(),
            block_col_indices=where[:, 1].to(torch.long),
            block_row_ptrs=row_ptrs,
            shape=(m, n),
            block_size=b,
        )

    @classmethod
    def _from_dense_device(cls, A: torch.Tensor, b: int, threshold: float) -> BSRMatrix:
        from . import _lib

        m, n = A.shape
        dev = A.device
        A, lda, code = _dense_args(A)
        mb, nbc = _ceil_to(m, b) // b, _ceil_to(n, b) // b
        row_ptrs = torch.empty(mb + 1, dtype=torch.int64, device=dev)
        ws_bytes = _lib.raw("trnsparse_bsr_from_dense_workspace_size")(m, n, b)
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
        thr = _threshold_in(A.dtype, threshold)
        with torch.cuda.device(dev):
            st = _lib.stream_handle(dev)
            _lib.call("trnsparse_bsr_from_dense_count", m, n, A.data_ptr(), lda, code, b, thr, row_ptrs.data_ptr(),
                      ws.data_ptr(), ws_bytes, st)
            nb = int(row_ptrs[-1].item()) if mb > 0 else 0
            blocks = torch.empty(nb, b, b, dtype=A.dtype, device=dev)
            cols = torch.empty(nb, dtype=torch.int64, device=dev)
            if nb > 0:
                _lib.call("trnsparse_bsr_from_dense_fill", m, n, A.data_ptr(), lda, code, b, blocks.data_ptr(),
                          cols.data_ptr(), ws.data_ptr(), st)
        return cls(blocks=blocks, block_col_indices=cols, block_row_ptrs=row_ptrs, shape=(m, n), block_size=b)

    @classmethod
    def from_csr(cls, csr: CSRMatrix, block_size: int = 128, threshold: float = 0.0) -> BSRMatrix:
        return cls.from_dense(csr.to_dense(), block_size=block_size, threshold=threshold)

    def block_rows(self) -> torch.Tensor:
        """Block-row index of every stored block (host, int64)."""
        counts = (self.block_row_ptrs[1:] - self.block_row_ptrs[:-1]).to(torch.long).cpu()
        return torch.repeat_interleave(torch.arange(counts.shape[0], dtype=torch.long), counts)

    def to_dense(self) -> torch.Tensor:
        m, n = self.shape
        b = self.block_size
        mb, nbc = _ceil_to(m, b) // b, _ceil_to(n, b) // b
        grid = torch.zeros(mb, nbc, b, b, dtype=self.dtype)
        if self.n_blocks:
            grid[self.block_rows(), self.block_col_indices.to(torch.long).cpu()] = self.blocks.cpu()
        return grid.transpose(1, 2).reshape(mb * b, nbc * b)[:m, :n].contiguous()

    def to_csr(self) -> CSRMatrix:
        return from_dense(self.to_dense(), threshold=0.0)

    def device_layout(self, device: torch.device) -> dict[str, Any]:
        """Blocks and int32 block indices on ``device`` (cached; see class doc)."""
        key = str(device)
        fp = _fingerprint(self.blocks, self.block_col_indices, self.block_row_ptrs)
        hit = self._dev.get(key)
        if hit is not None and hit["fp"] == fp:
            return hit
        nbr = _ceil_to(self.shape[0], self.block_size) // self.block_size
        if self.block_row_ptrs.shape[0] != nbr + 1:
            raise AssertionError(
                f"block_row_ptrs has {self.block_row_ptrs.shape[0]} entries, expected {nbr + 1}"
            )
        lay = {
            "fp": fp,
            "blocks": self.blocks.to(device=device).contiguous(),
            "row_ptr": self.block_row_ptrs.to(device=device, dtype=torch.int32).contiguous(),
            "col_idx": self.block_col_indices.to(device=device, dtype=torch.int32).contiguous(),
            "host_row_ptr": self.block_row_ptrs.to(torch.long).cpu(),
            "host_col_idx": self.block_col_indices.to(torch.long).cpu(),
        }
        self._dev[key] = lay
        return lay

    def __repr__(self) -> str:
        return (
            f"BSRMatrix(shape={self.shape}, block_size={self.block_size}, "
            f"n_blocks={self.n_blocks}, block_density={self.density:.4f})"
        )


def from_dense(A: torch.Tensor, threshold: float = 0.0) -> CSRMatrix:
    """Dense -> CSR keeping entries with |v| > threshold (formats.py:269-278).
    A float32 or bfloat16 CUDA tensor is converted on the device."""
    m, n = A.shape
    if A.is_cuda and A.dtype in _DEVICE_DENSE:
        return _csr_from_dense_device(A, threshold)
    keep = A.abs() > threshold
    rows, cols = torch.where(keep)
    coo = COOMatrix(values=A[keep], row_indices=rows, col_indices=cols, shape=(m, n))
    return coo.to_csr()


def _csr_from_dense_device(A: torch.Tensor, threshold: float) -> CSRMatrix:
    from . import _lib

    m, n = A.shape
    dev = A.device
    A, lda, code = _dense_args(A)
    thr = _threshold_in(A.dtype, threshold)
    row_ptrs = torch.empty(m + 1, dtype=torch.int64, device=dev)
    ws_bytes = _lib.raw("trnsparse_csr_from_dense_workspace_size")(m)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    # the count pass also writes a bit mask of the kept entries (1/32 of A's elements), so
    # a sparse result is gathered through it instead of reading A a second time
    mask = torch.empty(max(_lib.raw("trnsparse_csr_from_dense_mask_bytes")(m, n) // 4, 1), dtype=torch.int32,
                       device=dev)
    with torch.cuda.device(dev):
        st = _lib.stream_handle(dev)
        _lib.call("trnsparse_csr_from_dense_count_mask", m, n, A.data_ptr(), lda, code, thr, row_ptrs.data_ptr(),
                  mask.data_ptr(), ws.data_ptr(), ws_bytes, st)
        nnz = int(row_ptrs[-1].item())
        vals = torch.empty(nnz, dtype=A.dtype, device=dev)
        cols = torch.empty(nnz, dtype=torch.int64, device=dev)
        if nnz > 0:
            # a gathered entry costs a 32-byte sector; a re-read costs the row's element bytes
            if nnz * 64 < m * n * A.element_size():
                _lib.call("trnsparse_csr_from_dense_fill_masked", m, n, A.data_ptr(), lda, code, row_ptrs.data_ptr(),
                          mask.data_ptr(), vals.data_ptr(), cols.data_ptr(), st)
            else:
                _lib.call("trnsparse_csr_from_dense_fill", m, n, A.data_ptr(), lda, code, thr, row_ptrs.data_ptr(),
                          vals.data_ptr(), cols.data_ptr(), st)
    return CSRMatrix(values=vals, col_indices=cols, row_ptrs=row_ptrs, shape=(m, n))


def from_scipy(sp_matrix) -> CSRMatrix:
    """scipy.sparse -> CSR with float32 values and int64 indices (formats.py:281-291)."""
    import scipy.sparse as sp

    csr = sp.csr_matrix(sp_matrix)
    return CSRMatrix(
        values=torch.tensor(csr.data, dtype=torch.float32),
        col_indices=torch.tensor(csr.indices, dtype=torch.long),
        row_ptrs=torch.tensor(csr.indptr, dtype=torch.long),
        shape=csr.shape,
    )


def eye_sparse(n: int, dtype: torch.dtype = torch.float32) -> CSRMatrix:
    return CSRMatrix(
        values=torch.ones(n, dtype=dtype),
        col_indices=torch.arange(n, dtype=torch.long),
        row_ptrs=torch.arange(n + 1, dtype=torch.long),
        shape=(n, n),
    )
