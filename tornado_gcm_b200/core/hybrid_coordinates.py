"""Hybrid sigma-pressure coordinate P = a + b·Ps (reference ``core/hybrid_coordinates.py``)."""

from __future__ import annotations

import dataclasses
import os

import numpy as np
import torch

from tornado_gcm_b200.core import sigma_coordinates

_DATA_DIR = os.path.join(os.path.dirname(os.path.dirname(__file__)), "data")


def _col(t: torch.Tensor, like: torch.Tensor, nd: int) -> torch.Tensor:
    t = t.to(dtype=like.dtype, device=like.device)
    return t.reshape((-1,) + (1,) * nd)


@dataclasses.dataclass(frozen=True)
class HybridCoordinates:
    a_boundaries: np.ndarray
    b_boundaries: np.ndarray

    def __post_init__(self):
        a = np.asarray(self.a_boundaries, dtype=np.float64)
        b = np.asarray(self.b_boundaries, dtype=np.float64)
        if len(a) != len(b):
            raise ValueError("a_boundaries and b_boundaries must have the same length; "
                             f"got {len(a)} and {len(b)}.")
        object.__setattr__(self, "a_boundaries", a)
        object.__setattr__(self, "b_boundaries", b)

    @classmethod
    def from_coefficients(cls, a_coeffs, b_coeffs, p0: float = 1000.0) -> "HybridCoordinates":
        return cls(np.asarray(a_coeffs, dtype=np.float64) * p0, np.asarray(b_coeffs, dtype=np.float64))

    @classmethod
    def analytic_levels(cls, n_levels: int, p_top: float = 0.0, p0: float = 1000.0, sigma_exponent: float = 3.0,
                        stretch_exponent: float = 2.0) -> "HybridCoordinates":
        eta = np.linspace(0.0, 1.0, n_levels + 1) ** stretch_exponent
        p = p_top + eta * (p0 - p_top)
        b = eta ** sigma_exponent
        a = p / p0 - b
        a[0], b[0] = p_top / p0, 0.0
        a[-1], b[-1] = 0.0, 1.0
        return cls.from_coefficients(a, b, p0)

    @classmethod
    def from_sigma_levels(cls, sigma_levels) -> "HybridCoordinates":
        b = np.asarray(sigma_levels.boundaries, dtype=np.float64)
        return cls(np.zeros_like(b), b)

    @classmethod
    def from_csv(cls, name: str = "ecmwf137") -> "HybridCoordinates":
        """Load one of the bundled a/b tables (``ecmwf137`` or ``ufs127``)."""
        path = os.path.join(_DATA_DIR, f"{name}_hybrid_levels.csv")
        a, b = [], []
        with open(path) as fh:
            header = fh.readline().replace(",", "\t").split("\t")
            ia = next(i for i, h in enumerate(header) if h.strip().startswith("a"))
            ib = next(i for i, h in enumerate(header) if h.strip() == "b")
            for line in fh:
                parts = line.replace(",", "\t").split("\t")
                if len(parts) > max(ia, ib):
                    a.append(float(parts[ia]))
                    b.append(float(parts[ib]))
        # table a is in Pa; this class keeps a in hPa like the reference's p0 = 1000 convention
        return cls(np.asarray(a) / 100.0, np.asarray(b))

    @property
    def layers(self) -> int:
        return len(self.a_boundaries) - 1

    @property
    def pressure_thickness(self) -> np.ndarray:
        return np.diff(self.a_boundaries)

    @property
    def sigma_thickness(self) -> np.ndarray:
        return np.diff(self.b_boundaries)

    @property
    def a_centers(self) -> np.ndarray:
        return 0.5 * (self.a_boundaries[1:] + self.a_boundaries[:-1])

    @property
    def b_centers(self) -> np.ndarray:
        return 0.5 * (self.b_boundaries[1:] + self.b_boundaries[:-1])

    @property
    def center_to_center(self) -> np.ndarray:
        return np.diff(self.b_centers)

    def get_eta(self, p_surface: float) -> np.ndarray:
        return self.a_centers / p_surface + self.b_centers

    def pressure_boundaries(self, surface_pressure: torch.Tensor) -> torch.Tensor:
        nd = surface_pressure.dim()
        a = _col(torch.as_tensor(self.a_boundaries), surface_pressure, nd)
        b = _col(torch.as_tensor(self.b_boundaries), surface_pressure, nd)
        return a + b * surface_pressure.unsqueeze(0)

    def pressure_centers(self, surface_pressure: torch.Tensor) -> torch.Tensor:
        pb = self.pressure_boundaries(surface_pressure)
        return 0.5 * (pb[1:] + pb[:-1])

    def layer_thickness(self, surface_pressure: torch.Tensor) -> torch.Tensor:
        nd = surface_pressure.dim()
        da = _col(torch.as_tensor(self.pressure_thickness), surface_pressure, nd)
        db = _col(torch.as_tensor(self.sigma_thickness), surface_pressure, nd)
        return da + db * surface_pressure.unsqueeze(0)

    def get_sigma_boundaries(self, surface_pressure: float) -> np.ndarray:
        return self.a_boundaries / surface_pressure + self.b_boundaries

    def get_sigma_centers(self, surface_pressure: float) -> np.ndarray:
        sb = self.get_sigma_boundaries(surface_pressure)
        return 0.5 * (sb[1:] + sb[:-1])

    def to_sigma(self, surface_pressure: float = 1000.0) -> sigma_coordinates.SigmaCoordinates:
        sb = self.get_sigma_boundaries(surface_pressure)
        sb = (sb - sb[0]) / (sb[-1] - sb[0])
        return sigma_coordinates.SigmaCoordinates(sb)

    def __hash__(self):
        return hash((tuple(self.a_boundaries.tolist()), tuple(self.b_boundaries.tolist())))

    def __eq__(self, other):
        return (isinstance(other, HybridCoordinates) and np.array_equal(self.a_boundaries, other.a_boundaries)
                and np.array_equal(self.b_boundaries, other.b_boundaries))


def _dp(coordinates: HybridCoordinates, x: torch.Tensor, surface_pressure, axis: int) -> torch.Tensor:
    pos = axis % x.ndim
    shape = [1] * x.ndim
    shape[pos] = -1
    da = torch.as_tensor(coordinates.pressure_thickness, dtype=x.dtype, device=x.device).reshape(shape)
    db = torch.as_tensor(coordinates.sigma_thickness, dtype=x.dtype, device=x.device).reshape(shape)
    return da + db * surface_pressure


def cumulative_integral_over_pressure(x, surface_pressure, coordinates: HybridCoordinates, axis: int = -3,
                                      downward: bool = True) -> torch.Tensor:
    xdp = x * _dp(coordinates, x, surface_pressure, axis)
    if downward:
        return torch.cumsum(xdp, dim=axis)
    return torch.flip(torch.cumsum(torch.flip(xdp, [axis]), dim=axis), [axis])


def integral_over_pressure(x, surface_pressure, coordinates: HybridCoordinates, axis: int = -3,
                           keepdims: bool = True) -> torch.Tensor:
    pos = axis % x.ndim
    shape = [1] * x.ndim
    shape[pos] = -1
    da = torch.as_tensor(coordinates.pressure_thickness, dtype=x.dtype, device=x.device).reshape(shape)
    db = torch.as_tensor(coordinates.sigma_thickness, dtype=x.dtype, device=x.device).reshape(shape)
    return (x * da).sum(dim=axis, keepdim=keepdims) + surface_pressure * (x * db).sum(dim=axis, keepdim=keepdims)


def centered_difference(x: torch.Tensor, coordinates: HybridCoordinates, axis: int = -3) -> torch.Tensor:
    pos = axis % x.ndim
    shape = [1] * x.ndim
    shape[pos] = -1
    inv = torch.as_tensor(1.0 / coordinates.center_to_center, dtype=x.dtype, device=x.device).reshape(shape)
    return torch.diff(x, dim=axis) * inv


def centered_vertical_advection(w: torch.Tensor, x: torch.Tensor, coordinates: HybridCoordinates,
                                axis: int = -3) -> torch.Tensor:
    pos = axis % x.ndim
    dx = centered_difference(x, coordinates, pos)
    zw = torch.zeros_like(w.narrow(pos, 0, 1))
    zx = torch.zeros_like(dx.narrow(pos, 0, 1))
    p = torch.cat([zw, w, zw], dim=pos) * torch.cat([zx, dx, zx], dim=pos)
    n1 = p.shape[pos]
    return -0.5 * (p.narrow(pos, 1, n1 - 1) + p.narrow(pos, 0, n1 - 1))
