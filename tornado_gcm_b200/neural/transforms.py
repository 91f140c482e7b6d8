"""Dict → dict feature transforms — reference ``neural/transforms.py:29-477``.

Normalisation (``ShiftAndNormalize`` and its inverse), unit scaling
(``NondimensionalizeTransform``), nodal (u, v) → modal (δ, ζ)
(``ToModalWithDivCurl``), tendency level scaling and clipping, soft / hard
clips, per-level inverse scales, spectral derivative features
(``ToModalDiffOperators``), modal↔nodal and wavenumber clipping.

Transforms that convert several fields between nodal and modal space stack
the fields along the leading axis and make ONE transform call
(:func:`batched_to_nodal` / :func:`batched_to_modal`): on the GPU that is one
pair of tcgen05 GEMM launches for all fields instead of a pair per field.
"""

from __future__ import annotations

import math
from typing import Dict, Optional, Sequence

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F


def _lift(v: torch.Tensor, trailing: int = 2) -> tuple[torch.Tensor, tuple]:
    """View ``v`` as ``(rows, a, b)`` and remember its leading shape."""
    lead = tuple(v.shape[:-trailing])
    return v.reshape((-1,) + tuple(v.shape[-trailing:])), lead


def _batched(fn, tensors: Dict, out_shape_fn) -> Dict:
    if not tensors:
        return {}
    keys = list(tensors)
    groups: dict = {}
    for k in keys:  # stack tensors that share dtype/device
        t = tensors[k]
        groups.setdefault((t.dtype, t.device), []).append(k)
    out = {}
    for ks in groups.values():
        lifted = [_lift(tensors[k]) for k in ks]
        rows = [x.shape[0] for x, _ in lifted]
        res = fn(torch.cat([x for x, _ in lifted], 0))
        for k, (x, lead), part in zip(ks, lifted, torch.split(res, rows, 0)):
            out[k] = part.reshape(lead + tuple(part.shape[-2:]))
    return {k: out[k] for k in keys}


def batched_to_nodal(grid, tensors: Dict) -> Dict:
    """``grid.to_nodal`` of every value with one transform call per dtype."""
    return _batched(grid.to_nodal, tensors, None)


def batched_to_modal(grid, tensors: Dict) -> Dict:
    """``grid.to_modal`` of every value with one transform call per dtype."""
    return _batched(grid.to_modal, tensors, None)


def _as(v, like: torch.Tensor):
    return v.to(like.device, like.dtype) if isinstance(v, torch.Tensor) else v


class ShiftAndNormalize(nn.Module):
    """``(x - shift) / scale`` for keys present in both tables."""

    def __init__(self, shifts: Dict, scales: Dict, global_scale: Optional[float] = None):
        super().__init__()
        self.shifts = dict(shifts)
        g = 1.0 if global_scale is None else global_scale
        self.scales = {k: v * g for k, v in scales.items()}

    def forward(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        return {k: (v - _as(self.shifts[k], v)) / _as(self.scales[k], v)
                if k in self.shifts and k in self.scales else v for k, v in inputs.items()}


class InverseShiftAndNormalize(ShiftAndNormalize):
    """``x * scale + shift``."""

    def forward(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        return {k: v * _as(self.scales[k], v) + _as(self.shifts[k], v)
                if k in self.shifts and k in self.scales else v for k, v in inputs.items()}


class NondimensionalizeTransform(nn.Module):
    """Multiply each field by the non-dimensional value of one of its units."""

    def __init__(self, inputs_to_units_mapping: Dict[str, str], physics_specs):
        super().__init__()
        from tornado_gcm_b200.utils.units import parse_units

        self.mapping = dict(inputs_to_units_mapping)
        self.physics_specs = physics_specs
        self._scale_factors = {k: float(physics_specs.nondimensionalize(1.0 * parse_units(u)))
                               for k, u in self.mapping.items()}

    def forward(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        return {k: v * self._scale_factors[k] if k in self._scale_factors else v for k, v in inputs.items()}


class ToModalWithDivCurl(nn.Module):
    """Nodal ``(u, v, …)`` → modal ``(divergence, vorticity, …)``.

    ``u·secφ`` and ``v·secφ`` are transformed (in the same batched call as
    every other field) and turned into δ, ζ with the cos-lat divergence and
    curl operators, the inverse of
    :func:`~tornado_gcm_b200.core.spherical_harmonic.vor_div_to_uv_nodal`.
    (The reference scales by ``sec²φ`` here, ``neural/transforms.py:180-185``,
    which does not invert its own ``u, v`` construction.)
    """

    def __init__(self, grid, u_key: str = "u_component_of_wind", v_key: str = "v_component_of_wind"):
        super().__init__()
        self.grid = grid
        self.u_key = u_key
        self.v_key = v_key

    def forward(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        rest = dict(inputs)
        u = rest.pop(self.u_key, None)
        v = rest.pop(self.v_key, None)
        nodal = {k: t for k, t in rest.items()
                 if isinstance(t, torch.Tensor) and tuple(t.shape[-2:]) == tuple(self.grid.nodal_shape)}
        other = {k: t for k, t in rest.items() if k not in nodal}
        if u is not None and v is not None:
            sec = torch.as_tensor(1.0 / self.grid.cos_lat, dtype=u.dtype, device=u.device)
            nodal["__u"], nodal["__v"] = u * sec, v * sec
        modal = batched_to_modal(self.grid, nodal)
        if u is not None and v is not None:
            um, vm = modal.pop("__u"), modal.pop("__v")
            modal["divergence"] = self.grid.div_cos_lat((um, vm))
            modal["vorticity"] = self.grid.curl_cos_lat((um, vm))
        modal.update(other)
        return modal


class TendencyTransform(nn.Module):
    """Per-level scaling (axis -3) then optional clipping."""

    def __init__(self, level_scales: Optional[Dict] = None, clip_min: Optional[Dict] = None,
                 clip_max: Optional[Dict] = None):
        super().__init__()
        self.level_scales = level_scales or {}
        self.clip_min = clip_min or {}
        self.clip_max = clip_max or {}

    def forward(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        out = {}
        for k, v in inputs.items():
            if k in self.level_scales:
                s = self.level_scales[k]
                if isinstance(s, torch.Tensor):
                    shape = [1] * v.ndim
                    shape[-3] = -1
                    s = s.to(v.device, v.dtype).reshape(shape)
                v = v * s
            if k in self.clip_min or k in self.clip_max:
                v = torch.clamp(v, min=self.clip_min.get(k), max=self.clip_max.get(k))
            out[k] = v
        return out


class SoftClip(nn.Module):
    """Smooth clip of ``(-inf, inf)`` into ``(-max_value, max_value)``.

    ``f(x) = high - range · s(range - s(x - low)) / s(range)`` with
    ``s(t) = h · softplus(t / h)``: the identity well inside the range,
    saturating over a width of about ``h · log 2`` at each edge.
    """

    def __init__(self, max_value: float = 16.0, hinge_softness: float = 1.0):
        super().__init__()
        if max_value < 0 or hinge_softness < 0:
            raise ValueError(f"max_value and hinge_softness must be positive, got {max_value}, {hinge_softness}")
        self.max_value = float(max_value)
        self.hinge_softness = float(hinge_softness)
        self._low, self._high = -self.max_value, self.max_value
        self._range = self._high - self._low
        h = self.hinge_softness
        self._sp_range = h * math.log1p(math.exp(self._range / h)) if self._range / h < 30 else self._range

    def _s(self, x: torch.Tensor) -> torch.Tensor:
        return self.hinge_softness * F.softplus(x / self.hinge_softness)

    def clip(self, x: torch.Tensor) -> torch.Tensor:
        return self._high - self._range * self._s(self._range - self._s(x - self._low)) / self._sp_range

    _clip_fn = clip

    def forward(self, inputs):
        if isinstance(inputs, torch.Tensor):
            return self.clip(inputs)
        return {k: self.clip(v) for k, v in inputs.items()}


class HardClip(nn.Module):
    def __init__(self, min_val: Optional[float] = None, max_val: Optional[float] = None):
        super().__init__()
        self.min_val = min_val
        self.max_val = max_val

    def forward(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        return {k: torch.clamp(v, min=self.min_val, max=self.max_val) for k, v in inputs.items()}


class InverseLevelScale(nn.Module):
    """Divide selected keys by a per-level scale (leading axis = levels)."""

    def __init__(self, keys_to_scale: Sequence[str], scales: Sequence[float]):
        super().__init__()
        self.keys_to_scale = set(keys_to_scale)
        self.register_buffer("_inv_scales", 1.0 / torch.as_tensor(np.asarray(scales), dtype=torch.float32),
                             persistent=False)

    def forward(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        out = {}
        for k, v in inputs.items():
            if k in self.keys_to_scale:
                inv = self._inv_scales.to(v.device, v.dtype).reshape((-1,) + (1,) * (v.ndim - 1))
                v = v * inv
            out[k] = v
        return out


class SequentialTransform(nn.Module):
    def __init__(self, transforms: Sequence[nn.Module]):
        super().__init__()
        self.transforms = nn.ModuleList(transforms)

    def forward(self, inputs):
        for t in self.transforms:
            inputs = t(inputs)
        return inputs


class IdentityTransform(nn.Module):
    def __init__(self, grid=None, **kwargs):
        super().__init__()

    def forward(self, inputs):
        return inputs


class EmptyTransform(nn.Module):
    def __init__(self, grid=None, **kwargs):
        super().__init__()

    def forward(self, inputs):
        return {}


class ToModalDiffOperators(nn.Module):
    """Spectral derivative features of ``{(name, cos_lat_order): modal}``.

    For each input: ``name_dlon`` = cosφ ∂f/∂λ and ``name_dlat`` = cosφ ∂f/∂φ
    (order + 1), and ``name_del2`` = ∇²f (same order).
    """

    def __init__(self, grid):
        super().__init__()
        self.grid = grid

    def forward(self, inputs: Dict[tuple, torch.Tensor]) -> Dict[tuple, torch.Tensor]:
        if not inputs:
            return {}
        keys = list(inputs)
        lifted = [_lift(inputs[k]) for k in keys]
        rows = [x.shape[0] for x, _ in lifted]
        stacked = torch.cat([x for x, _ in lifted], 0)
        dlon, dlat = self.grid.cos_lat_grad(stacked, clip=False)
        lap = self.grid.laplacian(stacked)
        out = {}
        for key, (x, lead), a, b, c in zip(keys, lifted, torch.split(dlon, rows), torch.split(dlat, rows),
                                          torch.split(lap, rows)):
            name, order = key_parts(key)
            out[make_key(key, name + "_dlon", order + 1)] = a.reshape(lead + a.shape[-2:])
            out[make_key(key, name + "_dlat", order + 1)] = b.reshape(lead + b.shape[-2:])
            out[make_key(key, name + "_del2", order)] = c.reshape(lead + c.shape[-2:])
        return out


def key_parts(key) -> tuple[str, int]:
    """``(name, cos_lat_order)`` of a :class:`KeyWithCosLatFactor` or a plain pair."""
    if hasattr(key, "factor_order"):
        return key.name, int(key.factor_order)
    name, order = key
    return name, int(order)


def make_key(like, name: str, order: int):
    """A key of the same kind as ``like``."""
    if hasattr(like, "factor_order"):
        return type(like)(name, order)
    return (name, order)


class ModalToNodalTransform(nn.Module):
    def __init__(self, grid):
        super().__init__()
        self.grid = grid

    def forward(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        return batched_to_nodal(self.grid, inputs)


class NodalToModalTransform(nn.Module):
    def __init__(self, grid):
        super().__init__()
        self.grid = grid

    def forward(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        return batched_to_modal(self.grid, inputs)


class ClipTransform(nn.Module):
    """Zero the highest ``wavenumbers_to_clip`` total wavenumbers."""

    def __init__(self, grid, wavenumbers_to_clip: int = 1):
        super().__init__()
        self.grid = grid
        self.wavenumbers_to_clip = wavenumbers_to_clip

    def forward(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        return {k: self.grid.clip_wavenumbers(v, n=self.wavenumbers_to_clip) for k, v in inputs.items()}
