"""Axis helpers for level-structured fields — reference ``neural/field_utils.py:17-119``."""

from __future__ import annotations

import torch


def _axis(x: torch.Tensor, axis: int) -> int:
    return axis if axis >= 0 else x.ndim + axis


def _along(ref: torch.Tensor, like: torch.Tensor, axis: int) -> torch.Tensor:
    shape = [1] * like.ndim
    shape[_axis(like, axis)] = -1
    return torch.as_tensor(ref).to(like.device, like.dtype).reshape(shape)


def reconstruct_1d_field_from_ref_values(field: torch.Tensor, ref_values, axis: int = -3) -> torch.Tensor:
    """``field + ref`` with the 1-D profile broadcast along ``axis`` (e.g. T = T' + T_ref)."""
    return field + _along(ref_values, field, axis)


def extract_1d_field_perturbation(field: torch.Tensor, ref_values, axis: int = -3) -> torch.Tensor:
    """``field - ref`` with the 1-D profile broadcast along ``axis``."""
    return field - _along(ref_values, field, axis)


def slice_along_axis(x: torch.Tensor, start: int, length: int, axis: int = -3) -> torch.Tensor:
    return x.narrow(_axis(x, axis), start, length)


def pad_along_axis(x: torch.Tensor, pad_before: int, pad_after: int, axis: int = -3, value: float = 0.0):
    pos = _axis(x, axis)
    pads = [0, 0] * (x.ndim - 1 - pos) + [pad_before, pad_after]
    return torch.nn.functional.pad(x, pads, value=value)


def weighted_vertical_mean(x: torch.Tensor, weights, axis: int = -3, keepdim: bool = True) -> torch.Tensor:
    w = _along(weights, x, axis)
    return (x * w).sum(dim=_axis(x, axis), keepdim=keepdim) / w.sum()


def repeat_surface_to_volume(surface: torch.Tensor, n_layers: int, axis: int = -3) -> torch.Tensor:
    """Insert a level axis of length ``n_layers`` (a broadcast view, no copy)."""
    pos = axis if axis >= 0 else surface.ndim + 1 + axis
    x = surface.unsqueeze(pos)
    shape = list(x.shape)
    shape[pos] = n_layers
    return x.expand(shape)


def vertical_flip(x: torch.Tensor, axis: int = -3) -> torch.Tensor:
    return torch.flip(x, dims=[_axis(x, axis)])
