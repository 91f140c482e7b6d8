"""Vertical-coordinate containers for neural modules — reference ``neural/coordinates.py:22-101``."""

from __future__ import annotations

import dataclasses

import numpy as np
import torch

from tornado_gcm_b200.core import hybrid_coordinates as hybrid_mod
from tornado_gcm_b200.core import sigma_coordinates as sigma_mod

ERA5_37_HPA = (1, 2, 3, 5, 7, 10, 20, 30, 50, 70, 100, 125, 150, 175, 200, 225, 250, 300, 350, 400, 450, 500,
               550, 600, 650, 700, 750, 775, 800, 825, 850, 875, 900, 925, 950, 975, 1000)


@dataclasses.dataclass(frozen=True)
class TimeDelta:
    """Non-dimensional time step."""

    value: float

    def __float__(self) -> float:
        return float(self.value)


@dataclasses.dataclass(frozen=True)
class SigmaLevels:
    sigma: sigma_mod.SigmaCoordinates

    @property
    def centers(self) -> np.ndarray:
        return self.sigma.centers

    @property
    def boundaries(self) -> np.ndarray:
        return self.sigma.boundaries

    @property
    def layers(self) -> int:
        return self.sigma.layers

    @property
    def layer_thickness(self) -> np.ndarray:
        return self.sigma.layer_thickness

    @classmethod
    def equidistant(cls, n_layers: int) -> "SigmaLevels":
        return cls(sigma_mod.SigmaCoordinates.equidistant(n_layers))


@dataclasses.dataclass(frozen=True)
class HybridLevels:
    hybrid: hybrid_mod.HybridCoordinates

    @property
    def layers(self) -> int:
        return self.hybrid.layers

    @property
    def a_boundaries(self) -> np.ndarray:
        return self.hybrid.a_boundaries

    @property
    def b_boundaries(self) -> np.ndarray:
        return self.hybrid.b_boundaries

    def pressure_at_level(self, surface_pressure: torch.Tensor) -> torch.Tensor:
        return self.hybrid.pressure_centers(surface_pressure)

    @classmethod
    def from_sigma(cls, sigma: sigma_mod.SigmaCoordinates) -> "HybridLevels":
        return cls(hybrid_mod.HybridCoordinates.from_sigma_levels(sigma))


@dataclasses.dataclass(frozen=True)
class PressureLevels:
    """Fixed pressure levels (units as given, hPa for the ERA5 set)."""

    levels: np.ndarray

    @property
    def n_levels(self) -> int:
        return len(self.levels)

    @classmethod
    def era5_37(cls) -> "PressureLevels":
        return cls(np.asarray(ERA5_37_HPA, dtype=np.float64))

    @classmethod
    def from_list(cls, levels) -> "PressureLevels":
        return cls(np.asarray(levels, dtype=np.float64))
