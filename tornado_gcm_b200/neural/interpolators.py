"""Vertical interpolation between level types — reference ``neural/interpolators.py:28-284``.

Columns are interpolated all at once: the pressure of every source and
target level is formed per column (σ·ps, a + b·ps, or fixed), the columns
are flattened to ``(n_columns, n_levels)`` and a batched ``searchsorted``
locates each target level.  (The reference loops over every (lon, lat)
column in Python.)  Conservative regridding uses the exact per-column layer
bounds (the reference approximates them with the global-mean surface
pressure).
"""

from __future__ import annotations

from typing import Dict, Optional, Union

import numpy as np
import torch

from tornado_gcm_b200.core import vertical_interpolation as vi
from tornado_gcm_b200.neural.coordinates import HybridLevels, PressureLevels, SigmaLevels

Levels = Union[SigmaLevels, HybridLevels, PressureLevels]


def _n_levels(levels: Levels) -> int:
    return levels.n_levels if isinstance(levels, PressureLevels) else levels.layers


def _level_pressures(levels: Levels, surface_pressure: Optional[torch.Tensor], like: torch.Tensor) -> torch.Tensor:
    """Pressure at level centres, ``(…, n, lon, lat)`` or ``(n,)`` for fixed levels."""
    dev = like.device
    dt = like.dtype if surface_pressure is None else surface_pressure.dtype
    if isinstance(levels, PressureLevels):
        return torch.as_tensor(levels.levels, dtype=dt, device=dev)
    if surface_pressure is None:
        raise ValueError(f"{type(levels).__name__} needs the surface pressure")
    ps = surface_pressure if surface_pressure.dim() >= 3 else surface_pressure.unsqueeze(-3)
    if isinstance(levels, SigmaLevels):
        return torch.as_tensor(levels.centers, dtype=dt, device=dev).reshape(-1, 1, 1) * ps
    if isinstance(levels, HybridLevels):
        a, b = np.asarray(levels.a_boundaries), np.asarray(levels.b_boundaries)
        ac = torch.as_tensor(0.5 * (a[1:] + a[:-1]), dtype=dt, device=dev).reshape(-1, 1, 1)
        bc = torch.as_tensor(0.5 * (b[1:] + b[:-1]), dtype=dt, device=dev).reshape(-1, 1, 1)
        return ac + bc * ps
    raise TypeError(f"Unsupported level type: {type(levels)}")


def _columns(p: torch.Tensor, like: torch.Tensor, n: int) -> torch.Tensor:
    """Broadcast level pressures to ``like``'s columns: ``(cols, n)``."""
    if p.dim() == 1:
        shape = tuple(like.shape[:-3]) + (n,) + tuple(like.shape[-2:])
        p = p.reshape(-1, 1, 1).expand(shape)
    else:
        p = p.expand(tuple(like.shape[:-3]) + (n,) + tuple(like.shape[-2:]))
    return p.movedim(-3, -1).reshape(-1, n)


class LinearOnPressure:
    """Column-wise linear interpolation in pressure (linear or constant extrapolation)."""

    def __init__(self, target_levels: Levels, extrapolation: str = "linear"):
        if extrapolation not in ("linear", "constant"):
            raise ValueError("extrapolation must be 'linear' or 'constant'")
        self.target_levels = target_levels
        self.extrapolation = extrapolation

    def interpolate_field(self, field: torch.Tensor, source_levels: Levels,
                          surface_pressure: Optional[torch.Tensor] = None) -> torch.Tensor:
        ns, nt = field.shape[-3], _n_levels(self.target_levels)
        src = _columns(_level_pressures(source_levels, surface_pressure, field), field, ns).to(field.dtype)
        tgt = _columns(_level_pressures(self.target_levels, surface_pressure, field), field[..., :1, :, :]
                       .expand(tuple(field.shape[:-3]) + (nt,) + tuple(field.shape[-2:])), nt).to(field.dtype)
        vals = field.movedim(-3, -1).reshape(-1, ns)
        out = vi._column_interp(tgt.contiguous(), src.contiguous(), vals.contiguous(), self.extrapolation)
        lead = tuple(field.shape[:-3])
        return out.reshape(lead + tuple(field.shape[-2:]) + (nt,)).movedim(-1, -3)

    def __call__(self, inputs: Dict[str, torch.Tensor], source_levels: Levels) -> Dict[str, torch.Tensor]:
        ps = inputs.get("surface_pressure")
        return {k: self.interpolate_field(v, source_levels, ps) if v.ndim >= 3 else v
                for k, v in inputs.items() if k != "surface_pressure"}


def _pressure_bounds(levels: Levels, surface_pressure: Optional[torch.Tensor], like: torch.Tensor) -> torch.Tensor:
    dev, dt = like.device, like.dtype
    if isinstance(levels, PressureLevels):
        p = np.asarray(levels.levels, dtype=np.float64)
        b = np.empty(len(p) + 1)
        b[1:-1] = 0.5 * (p[1:] + p[:-1])
        b[0] = max(0.0, p[0] - 0.5 * (p[1] - p[0]))
        b[-1] = p[-1] + 0.5 * (p[-1] - p[-2])
        return torch.as_tensor(b, dtype=dt, device=dev)
    if isinstance(levels, SigmaLevels):
        sb = torch.as_tensor(levels.boundaries, dtype=dt, device=dev)
        if surface_pressure is None:
            return sb
        ps = surface_pressure if surface_pressure.dim() >= 3 else surface_pressure.unsqueeze(-3)
        return sb.reshape(-1, 1, 1) * ps
    raise TypeError(f"Unsupported level type: {type(levels)}")


class ConservativeOnPressure:
    """Overlap-weighted regridding between layer bounds, per column."""

    def __init__(self, target_levels: SigmaLevels):
        self.target_levels = target_levels

    def regrid_field(self, field: torch.Tensor, source_levels: Levels,
                     surface_pressure: Optional[torch.Tensor] = None) -> torch.Tensor:
        ns, nt = field.shape[-3], self.target_levels.layers
        sb = _pressure_bounds(source_levels, surface_pressure, field)
        tb = _pressure_bounds(self.target_levels, surface_pressure, field)
        if sb.dim() == 1 and tb.dim() == 1:
            return vi.regrid_conservative(field, vi.conservative_regrid_weights(sb, tb))
        like = field[..., :1, :, :]
        sbc = _columns(sb, like.expand(tuple(field.shape[:-3]) + (ns + 1,) + tuple(field.shape[-2:])), ns + 1)
        tbc = _columns(tb, like.expand(tuple(field.shape[:-3]) + (nt + 1,) + tuple(field.shape[-2:])), nt + 1)
        upper = torch.minimum(tbc[:, 1:, None], sbc[:, None, 1:])
        lower = torch.maximum(tbc[:, :-1, None], sbc[:, None, :-1])
        ov = torch.clamp(upper - lower, min=0)                        # (cols, nt, ns)
        rs = ov.sum(-1, keepdim=True)
        w = ov / torch.where(rs == 0, torch.ones_like(rs), rs)
        vals = field.movedim(-3, -1).reshape(-1, ns, 1)
        out = torch.bmm(w, vals).squeeze(-1)
        return out.reshape(tuple(field.shape[:-3]) + tuple(field.shape[-2:]) + (nt,)).movedim(-1, -3)

    def __call__(self, inputs: Dict[str, torch.Tensor], source_levels: Levels) -> Dict[str, torch.Tensor]:
        ps = inputs.get("surface_pressure")
        return {k: self.regrid_field(v, source_levels, ps) if v.ndim >= 3 else v
                for k, v in inputs.items() if k != "surface_pressure"}


def get_surface_pressure(geopotential: torch.Tensor, geopotential_at_surface: torch.Tensor,
                         pressure_levels: PressureLevels, gravity_acceleration: float = 1.0) -> torch.Tensor:
    """Pressure where ``Φ = Φ_s`` by linear interpolation / extrapolation in each column.

    ``geopotential_at_surface`` is a geopotential (``g·z_s``), so the default
    ``gravity_acceleration`` of 1 leaves it as is.
    """
    return vi.get_surface_pressure(vi.PressureCoordinates(np.asarray(pressure_levels.levels)), geopotential,
                                   geopotential_at_surface / gravity_acceleration, gravity_acceleration)
