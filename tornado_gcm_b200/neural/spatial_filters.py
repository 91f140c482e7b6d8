"""Spectral filters as modules — reference ``neural/spatial_filters.py:19-99``.

The per-``l`` coefficients are buffers; applying a filter is one broadcast
multiply over the modal ``(…, 2M-1, L)`` field.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn


class _ModalScale(nn.Module):
    def _set(self, coeffs: np.ndarray) -> None:
        self.register_buffer("_coeffs", torch.as_tensor(coeffs, dtype=torch.float32), persistent=False)

    @property
    def coefficients(self) -> torch.Tensor:
        return self._coeffs

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x * self._coeffs.to(x.device, x.dtype)


class ExponentialModalFilter(_ModalScale):
    """``s_l = exp(-a · ((l/L - c)/(1 - c))^(2·order))`` for ``l/L > c``, else 1."""

    def __init__(self, grid, attenuation: float = 16.0, order: int = 18, cutoff: float = 0.0):
        super().__init__()
        self.grid, self.attenuation, self.order, self.cutoff = grid, attenuation, order, cutoff
        L = grid.total_wavenumbers
        k = np.arange(L, dtype=np.float64) / L
        x = np.clip((k - cutoff) / (1.0 - cutoff), 0.0, None)
        self._set(np.where(k > cutoff, np.exp(-attenuation * x ** (2 * order)), 1.0))


class HorizontalDiffusionFilter(_ModalScale):
    """``s_l = exp(-τ · (l(l+1)/a²)^n)``."""

    def __init__(self, grid, tau: float = 0.01, n_diff: int = 1):
        super().__init__()
        self.grid, self.tau, self.n_diff = grid, tau, n_diff
        l = np.arange(grid.total_wavenumbers, dtype=np.float64)
        self._set(np.exp(-tau * (l * (l + 1) / grid.radius ** 2) ** n_diff))


class ComposedFilter(nn.Module):
    def __init__(self, *filters: nn.Module):
        super().__init__()
        self.filters = nn.ModuleList(filters)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for f in self.filters:
            x = f(x)
        return x
