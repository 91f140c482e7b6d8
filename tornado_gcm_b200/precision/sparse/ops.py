"""Structural-sparsity helpers for spectral coefficients — reference
``precision/sparse/ops.py:15-100``.

The modal layout of this framework (and of the reference's transforms) is
``(2M-1, L)`` with zonal rows ordered ``[0, +1, -1, +2, -2, …]``; row ``r``
carries ``|m| = (r + 1) // 2`` and entry ``(r, l)`` is a valid spherical
harmonic iff ``|m| ≤ l``.  (The reference's ``triangular_mask`` assumes a
``[0, 1, …, M-1, -(M-1), …, -1]`` row order instead, which does not match its
own transforms; this module uses the layout the transforms produce.)
"""

from __future__ import annotations

import torch


def abs_order(M2: int, device=None) -> torch.Tensor:
    return (torch.arange(M2, device=device) + 1) // 2


def triangular_mask(M: int, L: int, device: torch.device | str = "cpu") -> torch.Tensor:
    """Boolean (M, L) mask of valid (|m| ≤ l) coefficients."""
    return abs_order(M, device)[:, None] <= torch.arange(L, device=device)[None, :]


def adaptive_threshold_mask(x: torch.Tensor, threshold: float = 1e-6) -> torch.Tensor:
    return x.abs() >= threshold


def count_structural_zeros(M: int, L: int) -> tuple[int, int]:
    """(number of valid entries, number of entries)."""
    return int(triangular_mask(M, L).sum()), M * L


def memory_savings_ratio(M: int, L: int, mode: str = "structural", high_order_cutoff: float = 0.5) -> float:
    """Fraction of dense-FP32 memory saved by a storage mode."""
    n_valid, n_total = count_structural_zeros(M, L)
    cut = int(high_order_cutoff * L)
    if mode == "structural":
        return 1.0 - n_valid / n_total
    if mode == "mixed":
        return 1.0 - (M * cut * 4 + M * (L - cut) * 2) / (n_total * 4)
    if mode == "structural+mixed":
        mask = triangular_mask(M, L)
        low = int(mask[:, :cut].sum())
        high = int(mask[:, cut:].sum())
        return 1.0 - (low * 4 + high * 2) / (n_total * 4)
    raise ValueError(f"unknown sparse mode {mode!r}")
