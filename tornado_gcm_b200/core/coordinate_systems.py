"""Horizontal × vertical coordinate system (reference ``core/coordinate_systems.py``)."""

from __future__ import annotations

import dataclasses
from typing import Any, Callable, Sequence

import torch

from tornado_gcm_b200.core import spherical_harmonic


def _map_tensors(fn, x):
    if isinstance(x, torch.Tensor):
        return fn(x)
    if isinstance(x, dict):
        return {k: _map_tensors(fn, v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return type(x)(_map_tensors(fn, v) for v in x)
    return x


@dataclasses.dataclass(frozen=True)
class CoordinateSystem:
    horizontal: spherical_harmonic.Grid
    vertical: Any

    @property
    def nodal_shape(self):
        return (self.vertical.layers,) + tuple(self.horizontal.nodal_shape)

    @property
    def modal_shape(self):
        return (self.vertical.layers,) + tuple(self.horizontal.modal_shape)

    @property
    def surface_nodal_shape(self):
        return (1,) + tuple(self.horizontal.nodal_shape)

    @property
    def surface_modal_shape(self):
        return (1,) + tuple(self.horizontal.modal_shape)

    def with_horizontal(self, grid) -> "CoordinateSystem":
        return dataclasses.replace(self, horizontal=grid)


def get_spectral_downsample_fn(coords, save_coords, expect_same_vertical: bool = True) -> Callable:
    if expect_same_vertical and coords.vertical != save_coords.vertical:
        raise ValueError("Downsampling vertical resolution is not supported.")
    m_end, l_end = save_coords.horizontal.modal_shape
    return lambda state: _map_tensors(lambda x: x[..., :m_end, :l_end], state)


def get_spectral_upsample_fn(coords, save_coords, expect_same_vertical: bool = True) -> Callable:
    if expect_same_vertical and coords.vertical != save_coords.vertical:
        raise ValueError("Upsampling vertical resolution is not supported.")
    sm, sl = save_coords.horizontal.modal_shape
    cm, cl = coords.horizontal.modal_shape
    if sm < cm or sl < cl:
        raise ValueError("save_coords resolution smaller than coords.")
    return lambda state: _map_tensors(lambda x: torch.nn.functional.pad(x, (0, sl - cl, 0, sm - cm)), state)


def get_spectral_interpolate_fn(source_coords, target_coords, expect_same_vertical: bool = True) -> Callable:
    if source_coords.horizontal.total_wavenumbers < target_coords.horizontal.total_wavenumbers:
        return get_spectral_upsample_fn(source_coords, target_coords, expect_same_vertical)
    return get_spectral_downsample_fn(source_coords, target_coords, expect_same_vertical)


def maybe_to_nodal(fields: Any, coords: CoordinateSystem) -> Any:
    shape = tuple(coords.horizontal.nodal_shape)
    return _map_tensors(lambda x: x if tuple(x.shape[-2:]) == shape else coords.horizontal.to_nodal(x), fields)


def maybe_to_modal(fields: Any, coords: CoordinateSystem) -> Any:
    shape = tuple(coords.horizontal.modal_shape)
    return _map_tensors(lambda x: x if tuple(x.shape[-2:]) == shape else coords.horizontal.to_modal(x), fields)


def scale_levels_for_matching_keys(inputs: dict, scales: torch.Tensor, keys_to_scale: Sequence[str] = ()) -> dict:
    if scales.ndim != 1:
        raise ValueError(f"scales must be 1d, got shape {scales.shape}")
    s = scales[:, None, None]

    def rec(d):
        return {k: (rec(v) if isinstance(v, dict) else (v * s if k in keys_to_scale and isinstance(v, torch.Tensor) else v))
                for k, v in d.items()}
    return rec(inputs)
