"""ctypes binding of ``libtrnsparse_b200.so`` (the C ABI in ``include/trnsparse_b200.h``).

This module is the only place Python touches the native library. There is no
fallback: if the library or a CUDA device is missing, every op raises.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import torch

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("TRNSPARSE_B200_LIB", _PKG / "libtrnsparse_b200.so"))

# enums mirrored from include/trnsparse_b200.h
OK, ERR_ARG, ERR_DTYPE, ERR_ALIGN, ERR_CUDA, ERR_TIMEOUT, ERR_UNSUPPORTED, ERR_VALUE = range(8)
F32, F64, BF16, F16 = 0, 1, 2, 3
I32, I64 = 0, 1

_DTYPE = {torch.float32: F32, torch.float64: F64, torch.bfloat16: BF16, torch.float16: F16}
_INDEX = {torch.int32: I32, torch.int64: I64}

_i64, _i32, _f64, _p = C.c_int64, C.c_int, C.c_double, C.c_void_p

# name -> argtypes; restype is int (trnsparse_status) unless listed in _RESTYPE
SIGNATURES: dict[str, list] = {
    "trnsparse_last_error": [],
    "trnsparse_version": [],
    "trnsparse_csr_spmv": [_i64, _i64, _i64, _i32, _i32, _p, _p, _p, _p, _f64, _p, _f64, _p, _p],
    "trnsparse_csr_spmv_host": [_i64, _i64, _i64, _i32, _i32, _p, _p, _p, _p, _f64, _p, _p, _p, _i32, _p, _p, _p],
    "trnsparse_csr_spmm": [_i64, _i64, _i64, _i64, _i32, _i32, _p, _p, _p, _p, _i64, _f64, _p, _i64, _f64, _p, _i64, _p],
}
_BSR = [_i64, _i64, _i32, _i64, _p, _p, _p]  # m, n, b, n_blocks, row_ptr, col_idx, blocks
_sz = C.c_size_t
SIGNATURES.update({
    "trnsparse_device_error": [C.POINTER(C.c_int), _i32],
    "trnsparse_bsr_spmv": _BSR + [_p, _f64, _p, _f64, _p, _p],
    "trnsparse_bsr_cg_workspace_size": [_i64, _i32],
    "trnsparse_bsr_cg_start": _BSR + [_p, _p, _i32, _p, _i32, _p, _sz, _p],
    "trnsparse_bsr_cg_iterate": _BSR + [_p, _p, _f64, _i32, _i32, _i32, _p, _p],
    "trnsparse_bsr_chebyshev": _BSR + [_p, _p, _p, _i32, _p, _p, _p, _p],
    "trnsparse_bsr_richardson": _BSR + [_p, _f64, _i32, _p, _p, _p, _p],
    "trnsparse_dot": [_i64, _p, _p, _p, _p],
    "trnsparse_bsr_power_workspace_size": [_i64, _i32],
    "trnsparse_bsr_power_iterate": _BSR + [_p, _p, _f64, _i32, _i32, _i32, _p, _sz, _p],
    "trnsparse_bsr_power_finish": [_i64, _p, _i32, _p, _p],
    "trnsparse_bsr_spmm_simt": _BSR + [_p, _i64, _i64, _p, _i64, _p],
    "trnsparse_bsr_spmm_tc_workspace_size": [_i64, _i64, _i32],
    "trnsparse_bsr_spmm_tc_plan_capacity": [_i64, _i64, _i64, _i32, _i32],
    "trnsparse_bsr_spmm_tc_plan": [_i64, _p, _i64, _i32, _i32, _p, _i64, _p, _p, _p],
    "trnsparse_bsr_spmm_tc": [_i64, _i64, _i64, _p, _p, _p, _i32, _p, _i32, _i32, _p, _i64, _i64, _p, _i64, _i32,
                              _i32, _p, _sz, _p],
    "trnsparse_bsr_split_tf32": [_i64, _p, _p, _p, _p],
    "trnsparse_screened_spmm_workspace_size": [_i64, _i64],
    "trnsparse_screened_spmm": [_i64, _i64, _i64, _p, _i64, _p, _i32, _i64, _f64, _p, _i64, _p, _i64, _p, _sz, _p],
    "trnsparse_bsr_attention": [_i64, _i64, _i64, _i32, _p, _p, _p, _p, _p, _p, _i32, _f64, _p],
    "trnsparse_bsr_attention_tc": [_i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _f64, _p],
    "trnsparse_bsr_attention_tc_lse": [_i64, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _f64, _p],
    "trnsparse_bsr_attention_backward_tc_plan": [_i64, _i64, _p, _p, _i32, _p, _i64, _p],
    "trnsparse_bsr_attention_backward_tc_workspace_size": [_i64, _i64, _i64, _i64],
    "trnsparse_bsr_from_dense_workspace_size": [_i64, _i64, _i32],
    "trnsparse_bsr_from_dense_count": [_i64, _i64, _p, _i64, _i32, _i32, C.c_float, _p, _p, _sz, _p],
    "trnsparse_bsr_from_dense_fill": [_i64, _i64, _p, _i64, _i32, _i32, _p, _p, _p, _p],
    "trnsparse_csr_from_dense_workspace_size": [_i64],
    "trnsparse_csr_from_dense_count": [_i64, _i64, _p, _i64, _i32, C.c_float, _p, _p, _sz, _p],
    "trnsparse_csr_from_dense_fill": [_i64, _i64, _p, _i64, _i32, C.c_float, _p, _p, _p, _p],
    "trnsparse_csr_from_dense_mask_bytes": [_i64, _i64],
    "trnsparse_csr_from_dense_count_mask": [_i64, _i64, _p, _i64, _i32, C.c_float, _p, _p, _p, _sz, _p],
    "trnsparse_csr_from_dense_fill_masked": [_i64, _i64, _p, _i64, _i32, _p, _p, _p, _p, _p],
    "trnsparse_coo_to_csr_workspace_size": [_i64, _i64],
    "trnsparse_coo_to_csr": [_i64, _i64, _i64, _p, _p, _p, _i32, _p, _p, _p, _p, _sz, _p],
    "trnsparse_bsr_attention_backward_tc": [_i64, _i64, _i64, _p, _p, _p, _p, _i32, _i32, _i32, _i32, _p, _p, _p, _p,
                                            _p, _p, _p, _p, _p, _f64, _p, _sz, _p],
    "trnsparse_bsr_cg_layout": [_i64, _i32, C.POINTER(C.c_size_t)],
    "trnsparse_bsr_cg_dist_start": [_i64, _i64, _p, _p, _i32, _p, _sz, _p],
    "trnsparse_bsr_cg_dist_phase": _BSR + [_p, _p, _f64, _i32, _i32, _i32, _p, _p],
    "trnsparse_peer_comm_bytes": [_i32],
    "trnsparse_peer_alloc": [_sz, C.POINTER(C.c_void_p), _p],
    "trnsparse_peer_open": [_p, C.POINTER(C.c_void_p)],
    "trnsparse_peer_close": [_p],
    "trnsparse_peer_free": [_p],
    "trnsparse_peer_bump_epoch": [_p, _sz, _i32, _p],
    "trnsparse_peer_reduce_push": [_p, _i32, _i32, _sz, _p, _p, _i32, C.c_longlong, C.c_longlong, _p, _p, _i32,
                                   _i32, _p],
    "trnsparse_bsr_cg_fused_start": [_i64, _i64, _i32, _p, _p, _i32, _p, _sz, _p, _i32, _i32, _sz, _p, _i32, _p],
    "trnsparse_bsr_cg_fused_phase": _BSR + [_p, _p, _f64, _i32, _i32, _i32, _p, _p, _i32, _i32, _sz, _p, _i32, _p],
    "trnsparse_bsr_attention_backward_workspace_size": [_i64, _i64, _i64, _i32, _i32],
    "trnsparse_bsr_attention_backward": [_i64, _i64, _i64, _i32, _p, _p, _p, _p, _i32, _p, _p, _p, _p, _p, _p, _p, _p,
                                         _i32, _f64, _p, _sz, _p],
    "trnsparse_bsr_chebyshev_step": _BSR + [_p, _p, _p, _p, _f64, _f64, _i32, _p],
    "trnsparse_bsr_residual_sq": _BSR + [_p, _p, _p, _p],
    "trnsparse_bsr_power_step": _BSR + [_p, _p, _p, _p],
    "trnsparse_vec_div_norm": [_i64, _p, _p, _p, _p],
    "trnsparse_bsr_cgcg_workspace_size": [_i64, _i32],
    "trnsparse_bsr_cgcg_layout": [_i64, _i32, _p],
    "trnsparse_bsr_cgcg_solve": _BSR + [_p, _p, _p, _f64, _i32, _i64, _p, _sz, _sz, _p, _i32, _i32, _sz, _p, _i32,
                                        _p],
    "trnsparse_bsr_cg_coop_run": _BSR + [_p, _p, _f64, _i32, _i32, _i32, _p, _p, _i32, _i32, _sz, _p, _i32, _p],
    "trnsparse_bsr_cg_noalloc": _BSR + [_p, _p, _i32, _p, _f64, _i32, _p, _p],
    "trnsparse_csr_transpose_workspace_size": [_i64, _i64, _i64],
    "trnsparse_csr_transpose": [_i64, _i64, _i64, _i32, _p, _p, _i32, _p, _p, _p, _p, _sz, _p],
    "trnsparse_csr_sddmm": [_i64, _i64, _i64, _i64, _i32, _i32, _p, _p, _p, _i64, _p, _i64, _f64, _p, _p],
    "trnsparse_nt_tc_workspace_size": [_i64, _i64, _i64, _i32],
    "trnsparse_nt_tc": [_i64, _i64, _i64, _i32, _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i32, _i64, _i64, _i32, _p,
                        _i64, _f64, _p, _sz, _p],
    "trnsparse_gather": [_i64, _i32, _p, _p, _p, _p],
    "trnsparse_bsr_blocks_transpose": [_i64, _i32, _i32, _p, _p, _p, _p],
})
_RESTYPE = {
    "trnsparse_last_error": C.c_char_p,
    "trnsparse_bsr_cg_workspace_size": C.c_size_t,
    "trnsparse_bsr_power_workspace_size": C.c_size_t,
    "trnsparse_bsr_spmm_tc_workspace_size": C.c_size_t,
    "trnsparse_bsr_cgcg_workspace_size": C.c_size_t,
    "trnsparse_bsr_attention_backward_workspace_size": C.c_size_t,
    "trnsparse_bsr_attention_backward_tc_workspace_size": C.c_size_t,
    "trnsparse_bsr_from_dense_workspace_size": C.c_size_t,
    "trnsparse_csr_from_dense_workspace_size": C.c_size_t,
    "trnsparse_csr_from_dense_mask_bytes": C.c_size_t,
    "trnsparse_coo_to_csr_workspace_size": C.c_size_t,
    "trnsparse_csr_transpose_workspace_size": C.c_size_t,
    "trnsparse_nt_tc_workspace_size": C.c_size_t,
    "trnsparse_bsr_spmm_tc_plan_capacity": C.c_int64,
    "trnsparse_screened_spmm_workspace_size": C.c_size_t,
    "trnsparse_peer_comm_bytes": C.c_size_t,
}

_lib = None


class TrnsparseError(RuntimeError):
    """A C-ABI call returned a non-zero trnsparse_status."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def load(path: Path | str | None = None) -> C.CDLL:
    """Load (once) and return the native library; raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise RuntimeError(
            f"trnsparse_b200 native library not found at {p}; build it with "
            "`python -m trnsparse_b200.build` (there is no CPU fallback)"
        )
    lib = C.CDLL(str(p))
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _RESTYPE.get(name, C.c_int)
    if path is None:
        _lib = lib
    return lib


def raw(name: str):
    """The ctypes function object (for entry points that return a value, not a status)."""
    return getattr(load(), name)


def device_error(clear: bool = True) -> int:
    """Device-side error word of the current device (0 = no bounded wait gave up)."""
    v = C.c_int(0)
    call("trnsparse_device_error", C.byref(v), 1 if clear else 0)
    return v.value


def call(name: str, *args) -> None:
    """Invoke a status-returning entry point and raise on failure."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != OK:
        msg = lib.trnsparse_last_error().decode(errors="replace")
        if rc == ERR_ARG:
            raise AssertionError(msg)
        if rc == ERR_VALUE:
            raise ValueError(msg)
        raise TrnsparseError(rc, f"{name} failed (status {rc}): {msg}")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE[dt]
    except KeyError:
        raise TypeError(f"trnsparse_b200: unsupported dtype {dt}") from None


def index_code(dt: torch.dtype) -> int:
    try:
        return _INDEX[dt]
    except KeyError:
        raise TypeError(f"trnsparse_b200: unsupported index dtype {dt}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda() -> torch.device:
    """The CUDA device ops run on (the current device); raises without one."""
    if not torch.cuda.is_available():
        raise RuntimeError("trnsparse_b200 requires a CUDA device (B200, sm_100a); none is available")
    load()
    return torch.device("cuda", torch.cuda.current_device())
