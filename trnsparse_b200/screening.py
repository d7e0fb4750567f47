"""Schwarz / density screening (reference: trnsparse/screening.py:1-87).

These are elementwise mask definitions. ``screened_spmm`` applies the same
comparisons inside its CUDA kernel; the functions here build the masks as
tensors for callers that want them, on whatever device the input lives.
"""

from __future__ import annotations

import torch


def schwarz_bounds(diagonal_integrals: torch.Tensor) -> torch.Tensor:
    """Q = sqrt(|(mu nu|mu nu)|) (screening.py:17-26)."""
    return torch.sqrt(torch.abs(diagonal_integrals))


def screen_quartets(Q: torch.Tensor, threshold: float = 1e-10) -> torch.Tensor:
    """Boolean mask ``threshold**0.5 < Q`` of significant pairs (screening.py:29-40).

    The Python-float square root is compared against Q in Q's dtype, exactly as
    the reference's tensor comparison does.
    """
    return threshold**0.5 < Q


def density_screen(Q: torch.Tensor, P: torch.Tensor, threshold: float = 1e-10) -> torch.Tensor:
    """Pairs with ``Q * max(|P| * Q) > threshold`` (screening.py:43-64)."""
    return Q * (torch.abs(P) * Q).max() > threshold


def sparsity_stats(Q: torch.Tensor, threshold: float = 1e-10) -> dict:
    """Pair / quartet counts for a set of bounds (screening.py:67-87)."""
    n = Q.shape[0]
    sig = int(screen_quartets(Q, threshold).sum().item())
    pairs = n * n
    quartets = pairs * pairs
    return {
        "n_shells": n,
        "total_pairs": pairs,
        "significant_pairs": sig,
        "pair_sparsity": 1.0 - sig / pairs,
        "total_quartets": quartets,
        "significant_quartets_upper": sig * sig,
        "quartet_sparsity_lower": 1.0 - (sig * sig) / quartets,
    }
