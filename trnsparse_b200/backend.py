"""Backend selection kept for API compatibility (reference: trnsparse/nki/dispatch.py:36-85).

The reference switches between a PyTorch CPU path and Trainium NKI kernels.
This package has exactly one backend, the CUDA one: ``get_backend()``
returns ``"cuda"``, and ``set_backend`` accepts ``"cuda"`` or ``"auto"``
(both mean the CUDA kernels) and rejects anything else, including
``"pytorch"`` and ``"nki"``, rather than silently running another path.
"""

from __future__ import annotations

HAS_NKI = False

_backend = "cuda"


def set_backend(backend: str) -> None:
    global _backend
    if backend not in ("cuda", "auto"):
        raise ValueError(
            f"trnsparse_b200 has a single CUDA backend; backend={backend!r} is not available"
        )
    _backend = "cuda"


def get_backend() -> str:
    return _backend
