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
