"""Spectral filters as per-total-wavenumber scalings (reference ``core/filtering.py``).

Each builder returns a callable ``x -> x * s[l]``; the callable also exposes
``.scaling`` (FP64 numpy vector over l) so that the fused GPU step can fold
several filters into one multiply.
"""

from __future__ import annotations

from typing import Callable

import numpy as np
import torch


class SpectralScaling:
    """Multiply the last (total wavenumber) axis by a fixed vector."""

    def __init__(self, scaling: np.ndarray):
        self.scaling = np.asarray(scaling, dtype=np.float64)
        self._cache: dict = {}

    def tensor(self, device, dtype) -> torch.Tensor:
        key = (str(device), dtype)
        t = self._cache.get(key)
        if t is None:
            t = torch.as_tensor(self.scaling, dtype=dtype, device=device)
            self._cache[key] = t
        return t

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return x * self.tensor(x.device, x.dtype)

    def compose(self, other: "SpectralScaling") -> "SpectralScaling":
        return SpectralScaling(self.scaling * other.scaling)


def exponential_scaling(total_wavenumbers: int, attenuation: float, order: int, cutoff: float) -> np.ndarray:
    k = np.arange(total_wavenumbers, dtype=np.float64)
    k_max = k[-1]
    if k_max == 0:
        return np.ones_like(k)
    frac = k / k_max
    arg = np.zeros_like(frac)
    sel = frac > cutoff
    arg[sel] = ((frac[sel] - cutoff) / (1.0 - cutoff)) ** (2 * order)
    return np.exp(-attenuation * arg)


def exponential_filter(grid, attenuation: float = 16.0, order: int = 18, cutoff: float = 0.0) -> SpectralScaling:
    return SpectralScaling(exponential_scaling(grid.modal_shape[-1], attenuation, order, cutoff))


def horizontal_diffusion_filter(grid, scale: float, order: int = 1) -> SpectralScaling:
    eig = np.asarray(grid.laplacian_eigenvalues, dtype=np.float64)
    return SpectralScaling(np.exp(scale * (-eig) ** order))


def identity_filter() -> Callable[[torch.Tensor], torch.Tensor]:
    return lambda x: x
