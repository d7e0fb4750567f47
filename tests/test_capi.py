"""The C-ABI library loads and exports every entry point declared in include/*.h."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

from trnsparse_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols() -> set[str]:
    syms = set()
    for h in (ROOT / "include").glob("*.h"):
        syms |= set(re.findall(r"TRNSPARSE_API\s+[\w\s\*]+?\b(trnsparse_\w+)\s*\(", h.read_text()))
    return syms


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert {"trnsparse_last_error", "trnsparse_csr_spmv", "trnsparse_csr_spmm"} <= syms


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [s for s in sorted(declared_symbols()) if not hasattr(lib, s)]
    assert not missing, f"not exported: {missing}"


def test_binding_table_matches_header():
    assert set(_lib.SIGNATURES) == declared_symbols()


def test_error_reporting_without_gpu():
    lib = _lib.load()
    # argument validation happens before any CUDA call
    rc = lib.trnsparse_csr_spmv(-1, 1, 0, 0, 0, None, None, None, None, 1.0, None, 0.0, None, None)
    assert rc == _lib.ERR_ARG
    assert b"negative" in lib.trnsparse_last_error()
    assert lib.trnsparse_version() >= 100
    assert isinstance(lib, ctypes.CDLL)


def _plan(row_ptr, k, bn, ctas):
    import torch

    rp = torch.tensor(row_ptr, dtype=torch.int32)
    R = len(row_ptr) - 1
    cap = _lib.raw("trnsparse_bsr_spmm_tc_plan_capacity")(R, row_ptr[-1], k, bn, ctas)
    plan = torch.zeros(cap, dtype=torch.int32)
    nu, grid, zero = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _lib.call("trnsparse_bsr_spmm_tc_plan", R, rp.data_ptr(), k, bn, ctas, plan.data_ptr(), cap,
              ctypes.byref(nu), ctypes.byref(grid), ctypes.byref(zero))
    g = grid.value
    head = (g + 4) & ~3
    offs = plan[: g + 1].tolist()
    units = plan[head: head + 4 * nu.value].view(-1, 4).tolist()
    return offs, units, g, zero.value


def test_spmm_tc_plan_covers_every_block_once_per_tile():
    """Host scheduler of the tensor-core bsr_spmm (no GPU): every stored block is in
    exactly one unit per N tile, units stay inside their block-row, empty block-rows
    get a zero-storing unit, reduce-add only where a block-row is split, and the CTA
    offsets partition the unit list."""
    import random

    rng = random.Random(5)
    for R, ctas, k, bn in [(16, 148, 256, 256), (128, 148, 512, 256), (7, 4, 100, 128), (300, 148, 64, 128),
                           (3, 148, 1000, 256)]:
        lens = [0 if rng.random() < 0.15 else rng.randint(1, 40) for _ in range(R)]
        rp = [0]
        for L in lens:
            rp.append(rp[-1] + L)
        offs, units, g, zero = _plan(rp, k, bn, ctas)
        tiles = -(-k // bn)
        assert 1 <= g <= ctas and offs[0] == 0 and offs[-1] == len(units)
        assert all(a <= b for a, b in zip(offs, offs[1:]))
        seen = {}
        split_rows = set()
        for row, b0, b1, w in units:
            tile, reduce = w & ~(1 << 30), bool(w & (1 << 30))
            assert 0 <= tile < tiles and rp[row] <= b0 <= b1 <= rp[row + 1]
            if reduce:
                split_rows.add(row)
            if lens[row] == 0:
                assert b0 == b1 and not reduce
            for b in range(b0, b1):
                seen[(b, tile)] = seen.get((b, tile), 0) + 1
        assert seen == {(b, t): 1 for b in range(rp[-1]) for t in range(tiles)}
        for row in range(R):
            n_units = sum(1 for u in units if u[0] == row)
            assert n_units >= tiles
            assert (row in split_rows) == (n_units > tiles)
        assert zero == (1 if split_rows else 0)


def test_spmm_tc_plan_rejects_small_buffer():
    import torch

    rp = torch.tensor([0, 3, 5], dtype=torch.int32)
    plan = torch.zeros(4, dtype=torch.int32)
    nu, grid, zero = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    rc = _lib.load().trnsparse_bsr_spmm_tc_plan(2, ctypes.c_void_p(rp.data_ptr()), 256, 256, 148,
                                               ctypes.c_void_p(plan.data_ptr()), 4, ctypes.byref(nu),
                                               ctypes.byref(grid), ctypes.byref(zero))
    assert rc == _lib.ERR_ARG


def test_attention_backward_tc_plan():
    """Host plan of the tensor-core attention backward (no GPU): per mode every
    stored (fixed, partner) pair is in exactly one unit, units hold at most
    `split` partners and come longest first, a fixed block with more partners
    than `split` gets one workspace slot shared by its units (and an aux
    entry), and blocks with no partner get a zero-fill aux entry."""
    import random

    import torch

    rng = random.Random(11)
    for n, split in [(20, 16), (20, 3), (7, 1), (33, 5)]:
        keep = [[j <= i and (i - j < 3 or j < 2) and rng.random() > 0.1 for j in range(n)] for i in range(n)]
        keep[n // 2] = [False] * n
        rp = [0]
        for i in range(n):
            rp.append(rp[-1] + sum(keep[i]))
        cp = [0]
        for j in range(n):
            cp.append(cp[-1] + sum(keep[i][j] for i in range(n)))
        rp_t, cp_t = torch.tensor(rp, dtype=torch.int32), torch.tensor(cp, dtype=torch.int32)
        counts = (ctypes.c_int64 * 4)()
        args = (n, n, ctypes.c_void_p(rp_t.data_ptr()), ctypes.c_void_p(cp_t.data_ptr()), split)
        assert _lib.load().trnsparse_bsr_attention_backward_tc_plan(*args, None, 0, counts) == _lib.OK
        total = 4 * (counts[0] + counts[1] + counts[2])
        plan = torch.zeros(total, dtype=torch.int32)
        assert _lib.load().trnsparse_bsr_attention_backward_tc_plan(
            *args, ctypes.c_void_p(plan.data_ptr()), total, counts) == _lib.OK
        units = plan.view(-1, 4).tolist()
        ru, cu, aux = units[:counts[0]], units[counts[0]:counts[0] + counts[1]], units[counts[0] + counts[1]:]
        slots_used = set()
        for mode, ptr, us in ((0, rp, ru), (1, cp, cu)):
            covered = {}
            lengths = [u[2] - u[1] for u in us]
            assert lengths == sorted(lengths, reverse=True)
            for f, b0, b1, slot in us:
                assert ptr[f] <= b0 < b1 <= ptr[f + 1] and b1 - b0 <= split
                long = ptr[f + 1] - ptr[f] > split
                assert (slot >= 0) == long
                if long:
                    assert [mode, f, slot, 0] in aux
                    slots_used.add(slot)
                for e in range(b0, b1):
                    covered[e] = covered.get(e, 0) + 1
            assert covered == {e: 1 for e in range(ptr[-1])}
            for f in range(n):
                if ptr[f + 1] == ptr[f]:
                    assert [mode, f, -1, 0] in aux
        assert slots_used == set(range(counts[3]))


def test_new_entry_points_validate_before_cuda():
    """Argument checks of the host-buffer spmv, the format builders and the
    attention-backward entries run before any CUDA call (no GPU here)."""
    import torch

    lib = _lib.load()
    splits = torch.tensor([0, 10], dtype=torch.int64)
    need = torch.tensor([5], dtype=torch.int64)
    p = ctypes.c_void_p(1)
    # n_chunks out of range
    rc = lib.trnsparse_csr_spmv_host(10, 10, 1, 0, 0, p, p, p, p, 1.0, p, p, p, 0, ctypes.c_void_p(splits.data_ptr()),
                                     ctypes.c_void_p(need.data_ptr()), None)
    assert rc == _lib.ERR_ARG and b"n_chunks" in lib.trnsparse_last_error()
    # row splits that do not span the rows
    bad = torch.tensor([0, 9], dtype=torch.int64)
    rc = lib.trnsparse_csr_spmv_host(10, 10, 1, 0, 0, p, p, p, p, 1.0, p, p, p, 1, ctypes.c_void_p(bad.data_ptr()),
                                     ctypes.c_void_p(need.data_ptr()), None)
    assert rc == _lib.ERR_ARG and b"row_splits" in lib.trnsparse_last_error()
    # x_need past n
    far = torch.tensor([11], dtype=torch.int64)
    rc = lib.trnsparse_csr_spmv_host(10, 10, 1, 0, 0, p, p, p, p, 1.0, p, p, p, 1, ctypes.c_void_p(splits.data_ptr()),
                                     ctypes.c_void_p(far.data_ptr()), None)
    assert rc == _lib.ERR_ARG
    # format builders: dtype and workspace checks
    assert lib.trnsparse_bsr_from_dense_count(4, 4, p, 4, _lib.F64, 2, 0.0, p, p, 1 << 20, None) == _lib.ERR_ARG
    assert lib.trnsparse_bsr_from_dense_count(4, 4, p, 4, _lib.F32, 2, 0.0, p, p, 1, None) == _lib.ERR_ARG
    assert b"workspace" in lib.trnsparse_last_error()
    assert lib.trnsparse_csr_from_dense_count(4, 4, p, 2, _lib.F32, 0.0, p, p, 1 << 20, None) == _lib.ERR_ARG
    assert lib.trnsparse_coo_to_csr(4, 4, 1 << 33, p, p, p, _lib.F32, p, p, p, p, 1 << 40, None) == _lib.ERR_ARG
    assert _lib.raw("trnsparse_coo_to_csr_workspace_size")(4, 10) >= 8 * 20
    # attention backward on the tensor cores: shape checks
    assert lib.trnsparse_bsr_attention_backward_tc(1, 100, 128, p, p, p, p, 0, 0, 0, 0, p, p, p, p, p, None, p, p,
                                                   p, 1.0, p, 1 << 30, None) == _lib.ERR_ARG
    assert b"seq" in lib.trnsparse_last_error()
    assert lib.trnsparse_bsr_attention_backward_tc(1, 128, 96, p, p, p, p, 0, 0, 0, 0, p, p, p, p, p, None, p, p,
                                                   p, 1.0, p, 1 << 30, None) == _lib.ERR_ARG
    assert _lib.raw("trnsparse_bsr_attention_backward_tc_workspace_size")(2, 256, 128, 3) == 4 * (2 * 512 + 3 * 2 * 2 * 128 * 128)


def test_csr_from_dense_mask_bytes():
    """Size of the kept-entry bit mask of CSR from_dense (host function, no GPU): one
    uint32 word per 32 columns of every row, zero for negative sizes."""
    f = _lib.raw("trnsparse_csr_from_dense_mask_bytes")
    for m, n in [(0, 0), (1, 1), (3, 31), (3, 32), (3, 33), (8192, 8192), (7, 100000)]:
        assert f(m, n) == 4 * m * ((n + 31) // 32)
    assert f(-1, 5) == 0 and f(5, -1) == 0
