"""Test infrastructure: CPU restatement of the reference's sparse compute path.

NOT part of the product. Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import this package, and only as the
checker / the timed CPU baseline, never as a code path of ``trnsparse_b200``.

Each function restates the algorithm of the reference trnsci/trnsparse
v0.6.0 CPU path (cited as file:line) in our own code, on CPU torch tensors.
Where the reference's arithmetic lives in a third-party library — the CSR
products are ``torch.sparse_csr_tensor @ dense`` (PyTorch ATen, the image's
torch 2.11.0) and the dense products are ``torch.matmul`` (ATen/MKL) — the
oracle calls the same library routine, and parity is pinned on the
reference's own known-answer tests plus golden vectors produced by running
the reference itself (``tests/golden/make_golden.py``).
"""

from .ref import *  # noqa: F401,F403
from .ref import __all__  # noqa: F401
