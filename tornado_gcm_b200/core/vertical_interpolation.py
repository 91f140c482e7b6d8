"""Vertical interpolation between pressure and sigma levels
(reference ``core/vertical_interpolation.py:25-312``), batch-aware and
vectorised over columns."""

from __future__ import annotations

import dataclasses
from typing import Any, Dict

import numpy as np
import torch

from tornado_gcm_b200.core import sigma_coordinates


class PressureCoordinates:
    def __init__(self, centers):
        c = np.asarray(centers, dtype=np.float64)
        if not np.all(np.diff(c) > 0):
            raise ValueError(f"centers must be monotonically increasing, got {c}")
        self.centers = c

    @property
    def layers(self) -> int:
        return len(self.centers)

    def asdict(self) -> Dict[str, Any]:
        return {"centers": self.centers.tolist()}

    def __hash__(self):
        return hash(tuple(self.centers.tolist()))

    def __eq__(self, other):
        return isinstance(other, PressureCoordinates) and np.array_equal(self.centers, other.centers)


def interp_1d(x: torch.Tensor, xp: torch.Tensor, fp: torch.Tensor) -> torch.Tensor:
    """np.interp semantics: linear inside, constant outside."""
    idx = torch.searchsorted(xp.contiguous(), x.contiguous()).clamp(1, len(xp) - 1)
    x0, x1 = xp[idx - 1], xp[idx]
    w = (x - x0) / (x1 - x0)
    out = fp[idx - 1] + w * (fp[idx] - fp[idx - 1])
    out = torch.where(x <= xp[0], fp[0], out)
    return torch.where(x >= xp[-1], fp[-1], out)


def linear_interp_with_linear_extrap(x: torch.Tensor, xp: torch.Tensor, fp: torch.Tensor) -> torch.Tensor:
    idx = torch.searchsorted(xp.contiguous(), x.contiguous()).clamp(1, len(xp) - 1)
    x0, x1 = xp[idx - 1], xp[idx]
    return fp[idx - 1] + (x - x0) / (x1 - x0) * (fp[idx] - fp[idx - 1])


def _column_interp(target: torch.Tensor, source: torch.Tensor, values: torch.Tensor, extrapolate: str) -> torch.Tensor:
    """Per-column interpolation; all args (..., n_cols, n_levels); source ascending per column."""
    n_src = source.shape[-1]
    idx = torch.searchsorted(source.contiguous(), target.contiguous()).clamp(1, n_src - 1)
    x0, x1 = source.gather(-1, idx - 1), source.gather(-1, idx)
    f0, f1 = values.gather(-1, idx - 1), values.gather(-1, idx)
    den = x1 - x0
    safe = torch.where(den == 0, torch.ones_like(den), den)
    out = torch.where(den == 0, f0, f0 + (target - x0) / safe * (f1 - f0))
    if extrapolate == "constant":
        out = torch.where(target <= source[..., :1], values[..., :1].expand_as(out), out)
        out = torch.where(target >= source[..., -1:], values[..., -1:].expand_as(out), out)
    return out


def _to_cols(x: torch.Tensor) -> tuple[torch.Tensor, tuple]:
    lead, n, i, j = x.shape[:-3], x.shape[-3], x.shape[-2], x.shape[-1]
    return x.reshape(*lead, n, i * j).transpose(-1, -2), (lead, i, j)


def _from_cols(c: torch.Tensor, meta) -> torch.Tensor:
    lead, i, j = meta
    return c.transpose(-1, -2).reshape(*lead, c.shape[-1], i, j)


def interp_pressure_to_sigma(fields: dict, pressure_coords: PressureCoordinates,
                             sigma_coords: sigma_coordinates.SigmaCoordinates, surface_pressure: torch.Tensor) -> dict:
    """Fields (..., n_pressure, lon, lat) → (..., n_sigma, lon, lat) at σ·ps."""
    sp = surface_pressure
    src = torch.as_tensor(pressure_coords.centers, dtype=sp.dtype, device=sp.device)
    sig = torch.as_tensor(sigma_coords.centers, dtype=sp.dtype, device=sp.device)

    def regrid(x):
        if not torch.is_tensor(x) or x.ndim < 3 or x.shape[-3] != pressure_coords.layers:
            return x
        vals, meta = _to_cols(x)
        tgt_full = sig.reshape(-1, 1, 1) * (sp if sp.dim() >= 3 else sp.unsqueeze(-3))
        tgt, _ = _to_cols(tgt_full.expand(*x.shape[:-3], len(sig), *x.shape[-2:]))
        srcb = src.expand(*vals.shape[:-1], len(src))
        return _from_cols(_column_interp(tgt, srcb, vals, "constant"), meta)

    return {k: regrid(v) for k, v in fields.items()}


def interp_sigma_to_pressure(fields: dict, pressure_coords: PressureCoordinates,
                             sigma_coords: sigma_coordinates.SigmaCoordinates, surface_pressure: torch.Tensor) -> dict:
    sp = surface_pressure
    sig = torch.as_tensor(sigma_coords.centers, dtype=sp.dtype, device=sp.device)
    tgt_levels = torch.as_tensor(pressure_coords.centers, dtype=sp.dtype, device=sp.device)

    def regrid(x):
        if not torch.is_tensor(x) or x.ndim < 3 or x.shape[-3] != len(sig):
            return x
        vals, meta = _to_cols(x)
        src_full = sig.reshape(-1, 1, 1) * (sp if sp.dim() >= 3 else sp.unsqueeze(-3))
        src, _ = _to_cols(src_full.expand(*x.shape[:-3], len(sig), *x.shape[-2:]))
        tgt = tgt_levels.expand(*vals.shape[:-1], len(tgt_levels))
        return _from_cols(_column_interp(tgt.contiguous(), src, vals, "constant"), meta)

    return {k: regrid(v) for k, v in fields.items()}


def conservative_regrid_weights(source_bounds: torch.Tensor, target_bounds: torch.Tensor) -> torch.Tensor:
    """(n_target, n_source) overlap weights, rows normalised to 1."""
    upper = torch.minimum(target_bounds[1:, None], source_bounds[None, 1:])
    lower = torch.maximum(target_bounds[:-1, None], source_bounds[None, :-1])
    ov = torch.clamp(upper - lower, min=0)
    rs = ov.sum(dim=1, keepdim=True)
    return ov / torch.where(rs == 0, torch.ones_like(rs), rs)


def regrid_conservative(x: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    return torch.einsum("ts,...sij->...tij", weights.to(x.dtype), x)


def get_surface_pressure(pressure_levels: PressureCoordinates, geopotential: torch.Tensor, orography: torch.Tensor,
                         gravity_acceleration: float) -> torch.Tensor:
    """Pressure where the geopotential equals g·orography (linear extrapolation)."""
    levels = torch.as_tensor(pressure_levels.centers, dtype=geopotential.dtype, device=geopotential.device)
    rel = orography * gravity_acceleration - geopotential  # increases with pressure
    vals, meta = _to_cols(rel)
    lv = levels.expand(*vals.shape[:-1], len(levels))
    zero = torch.zeros(*vals.shape[:-1], 1, dtype=vals.dtype, device=vals.device)
    # interpolate pressure as a function of rel at rel = 0
    out = _column_interp(zero, vals.contiguous(), lv.contiguous(), "linear")
    return _from_cols(out, meta)
