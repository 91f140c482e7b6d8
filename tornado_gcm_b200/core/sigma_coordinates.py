"""Sigma (normalised pressure) vertical coordinate and vertical calculus.

Behaviour follows reference ``core/sigma_coordinates.py:42-346``.  The
cumulative integral is computed as an FP64 prefix sum (the reference uses an
upper-triangular FP64 matmul, which is the same prefix sum evaluated in
float64); results are cast back to the input dtype.
"""

from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np
import torch


@dataclasses.dataclass(frozen=True)
class SigmaCoordinates:
    """Layer boundaries σ_{k±1/2}, increasing from 0 (top) to 1 (surface)."""

    boundaries: np.ndarray

    def __init__(self, boundaries):
        b = np.asarray(boundaries, dtype=np.float64)
        if not (np.isclose(b[0], 0) and np.isclose(b[-1], 1)):
            raise ValueError(f"Expected boundaries[0]=0, boundaries[-1]=1, got boundaries={b}")
        if not np.all(np.diff(b) > 0):
            raise ValueError(f"Expected boundaries to be monotonically increasing, got {b}")
        object.__setattr__(self, "boundaries", b)

    @property
    def internal_boundaries(self) -> np.ndarray:
        return self.boundaries[1:-1]

    @property
    def centers(self) -> np.ndarray:
        return 0.5 * (self.boundaries[1:] + self.boundaries[:-1])

    @property
    def layer_thickness(self) -> np.ndarray:
        return np.diff(self.boundaries)

    @property
    def center_to_center(self) -> np.ndarray:
        return np.diff(self.centers)

    @property
    def layers(self) -> int:
        return len(self.boundaries) - 1

    @classmethod
    def equidistant(cls, layers: int, dtype=np.float32) -> "SigmaCoordinates":
        return cls(np.linspace(0, 1, layers + 1, dtype=dtype))

    @classmethod
    def from_centers(cls, centers) -> "SigmaCoordinates":
        c = np.asarray(centers, dtype=np.float64)
        n = len(c)
        # boundaries b_1..b_n satisfy (b_{k} + b_{k+1})/2 = c_k with b_0 = 0
        b = np.zeros(n + 1)
        for k in range(n):
            b[k + 1] = 2.0 * c[k] - b[k]
        return cls(b)

    def asdict(self):
        return {"boundaries": self.boundaries.tolist()}

    def __hash__(self):
        return hash(tuple(self.centers.tolist()))

    def __eq__(self, other):
        return isinstance(other, SigmaCoordinates) and np.array_equal(self.centers, other.centers)


def _axis_vector(values: np.ndarray, x: torch.Tensor, axis: int) -> torch.Tensor:
    shape = [1] * x.ndim
    shape[axis] = -1
    return torch.as_tensor(values, dtype=x.dtype, device=x.device).reshape(shape)


def centered_difference(x: torch.Tensor, coordinates: SigmaCoordinates, axis: int = -3) -> torch.Tensor:
    """∂x/∂σ at the internal boundaries (n-1 values)."""
    if coordinates.layers != x.shape[axis]:
        raise ValueError(
            f"x.shape[axis] must equal coordinates.layers; got {x.shape[axis]} and {coordinates.layers}."
        )
    pos = axis % x.ndim
    n = x.shape[pos]
    dx = x.narrow(pos, 1, n - 1) - x.narrow(pos, 0, n - 1)
    return dx * _axis_vector(1.0 / coordinates.center_to_center, x, pos)


def _prefix_sum_f64(xds: torch.Tensor, pos: int, reverse: bool = False) -> torch.Tensor:
    x64 = xds.to(torch.float64)
    if reverse:
        out = torch.flip(torch.cumsum(torch.flip(x64, dims=[pos]), dim=pos), dims=[pos])
    else:
        out = torch.cumsum(x64, dim=pos)
    return out.to(xds.dtype)


def cumulative_sigma_integral(x: torch.Tensor, coordinates: SigmaCoordinates, axis: int = -3,
                              downward: bool = True) -> torch.Tensor:
    if coordinates.layers != x.shape[axis]:
        raise ValueError(
            f"x.shape[axis] must equal coordinates.layers; got {x.shape[axis]} and {coordinates.layers}."
        )
    pos = axis % x.ndim
    xds = x * _axis_vector(coordinates.layer_thickness, x, pos)
    return _prefix_sum_f64(xds, pos, reverse=not downward)


CUMULATIVE_SIGMA_INTEGRAL_BACKEND = "prefix_sum_f64acc"


def sigma_integral(x: torch.Tensor, coordinates: SigmaCoordinates, axis: int = -3,
                   keepdims: bool = True) -> torch.Tensor:
    if coordinates.layers != x.shape[axis]:
        raise ValueError(
            f"x.shape[axis] must equal coordinates.layers; got {x.shape[axis]} and {coordinates.layers}."
        )
    pos = axis % x.ndim
    xds = x * _axis_vector(coordinates.layer_thickness, x, pos)
    return xds.sum(dim=pos, keepdim=keepdims)


def cumulative_log_sigma_integral(x: torch.Tensor, coordinates: SigmaCoordinates, axis: int = -3,
                                  downward: bool = True) -> torch.Tensor:
    """Trapezoid-rule cumulative integral in log σ."""
    if coordinates.layers != x.shape[axis]:
        raise ValueError("x.shape[axis] must equal coordinates.layers")
    pos = axis % x.ndim
    n = x.shape[pos]
    mid = 0.5 * (x.narrow(pos, 1, n - 1) + x.narrow(pos, 0, n - 1))
    integrand = torch.cat([mid, x.narrow(pos, n - 1, 1)], dim=pos)
    dlog = np.diff(np.log(coordinates.centers), append=0)
    xds = integrand * _axis_vector(dlog, x, pos)
    if downward:
        return torch.cumsum(xds, dim=pos)
    return torch.flip(torch.cumsum(torch.flip(xds, dims=[pos]), dim=pos), dims=[pos])


def centered_vertical_advection(w: torch.Tensor, x: torch.Tensor, coordinates: SigmaCoordinates,
                                axis: int = -3,
                                w_boundary_values: Optional[tuple[torch.Tensor, torch.Tensor]] = None,
                                dx_dsigma_boundary_values: Optional[tuple[torch.Tensor, torch.Tensor]] = None,
                                ) -> torch.Tensor:
    """−(w ∂x/∂σ) at layer centres from boundary values of w (n-1 internal)."""
    pos = axis % x.ndim
    dx = centered_difference(x, coordinates, pos)
    if w_boundary_values is None:
        zshape = list(w.shape)
        zshape[pos] = 1
        z = torch.zeros(zshape, dtype=w.dtype, device=w.device)
        w_boundary_values = (z, z)
    if dx_dsigma_boundary_values is None:
        zshape = list(dx.shape)
        zshape[pos] = 1
        z = torch.zeros(zshape, dtype=dx.dtype, device=dx.device)
        dx_dsigma_boundary_values = (z, z)
    w_full = torch.cat([w_boundary_values[0], w, w_boundary_values[1]], dim=pos)
    dx_full = torch.cat([dx_dsigma_boundary_values[0], dx, dx_dsigma_boundary_values[1]], dim=pos)
    prod = w_full * dx_full
    n1 = prod.shape[pos]
    return -0.5 * (prod.narrow(pos, 1, n1 - 1) + prod.narrow(pos, 0, n1 - 1))


def upwind_vertical_advection(w: torch.Tensor, x: torch.Tensor, coordinates: SigmaCoordinates,
                              axis: int = -3) -> torch.Tensor:
    pos = axis % x.ndim
    dx = centered_difference(x, coordinates, pos)
    zw_shape = list(w.shape)
    zw_shape[pos] = 1
    zw = torch.zeros(zw_shape, dtype=w.dtype, device=w.device)
    zx_shape = list(dx.shape)
    zx_shape[pos] = 1
    zx = torch.zeros(zx_shape, dtype=dx.dtype, device=dx.device)
    w_up = torch.cat([zw, w], dim=pos)
    w_dn = torch.cat([w, zw], dim=pos)
    dx_up = torch.cat([zx, dx], dim=pos)
    dx_dn = torch.cat([dx, zx], dim=pos)
    return -(torch.clamp(w_up, min=0) * dx_up + torch.clamp(w_dn, max=0) * dx_dn)
