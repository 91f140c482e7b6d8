"""Reanalysis preprocessing — reference ``training/data_pipeline.py:32-512``.

Time conversion (``datetime64`` ↔ non-dimensional ``sim_time``), xarray →
array dicts in ``(time, [level], lon, lat)`` order, forcing providers
(nearest-time lookup, persistence, day-of-year climatology, anomaly
persistence), selective temporal shifts, bilinear regridding and
nearest-neighbour NaN filling on the sphere.

:class:`BilinearRegridder` precomputes its two 1-D stencils once and applies
them as gathers on any device (numpy arrays in, numpy out; torch tensors
stay on their device), so a whole ``(time, level, lon, lat)`` block regrids in
two vectorised passes.  :class:`NearestNaNFiller` uses a k-d tree on unit
vectors (chord distance is monotone in great-circle distance), instead of a
brute-force haversine search.  xarray is optional: the xarray entry points
import it when called.
"""

from __future__ import annotations

import logging
from typing import Optional, Sequence

import numpy as np
import torch

logger = logging.getLogger(__name__)


# ───────────────────────── time ─────────────────────────


def datetime64_to_sim_time(times, reference_datetime, time_scale_hours: float = 1.0) -> np.ndarray:
    """``(t - t_ref) / time_scale`` with the scale in hours."""
    d = (np.asarray(times) - np.datetime64(reference_datetime)).astype("timedelta64[s]").astype(np.float64)
    return d / (time_scale_hours * 3600.0)


def sim_time_to_datetime64(sim_time, reference_datetime, time_scale_hours: float = 1.0) -> np.ndarray:
    s = np.round(np.asarray(sim_time, dtype=np.float64) * time_scale_hours * 3600.0).astype(np.int64)
    return np.datetime64(reference_datetime) + s.astype("timedelta64[s]")


def with_sim_time(data: dict, times, reference_datetime=None, time_scale_hours: float = 1.0) -> dict:
    """Add a ``sim_time`` entry shaped ``(T, 1, …)`` to broadcast against the fields."""
    if "sim_time" in data:
        return data
    times = np.asarray(times)
    st = datetime64_to_sim_time(times, times[0] if reference_datetime is None else reference_datetime,
                                time_scale_hours)
    out = dict(data)
    sample = next((v for k, v in data.items() if k != "sim_time"), None)
    if sample is not None and np.ndim(sample) > 1:
        st = st.reshape((len(st),) + (1,) * (np.ndim(sample) - 1))
    out["sim_time"] = st
    return out


# ───────────────────────── xarray ─────────────────────────

_DIM_ALIASES = {"time": ("time",), "level": ("level", "lev", "pressure_level"),
                "longitude": ("longitude", "lon"), "latitude": ("latitude", "lat")}


def inputs_from_xarray(dataset, input_variables: Optional[Sequence[str]] = None, reference_datetime=None,
                       time_scale_hours: float = 1.0) -> dict:
    """``{name: (time, [level→1], lon, lat)}`` plus ``sim_time``; warns about missing vars / NaNs."""
    if input_variables is not None:
        missing = set(input_variables) - set(dataset.data_vars)
        if missing:
            logger.warning("missing variables %s", sorted(missing))
        dataset = dataset[[v for v in input_variables if v in dataset.data_vars]]
    out = {}
    for name in dataset.data_vars:
        var = dataset[name]
        order = [next(a for a in _DIM_ALIASES[d] if a in var.dims) for d in _DIM_ALIASES
                 if any(a in var.dims for a in _DIM_ALIASES[d])]
        arr = np.asarray(var.transpose(*order).values)
        if not any(a in var.dims for a in _DIM_ALIASES["level"]) and arr.ndim >= 2:
            arr = np.expand_dims(arr, -3)
        n_nan = int(np.isnan(arr).sum()) if np.issubdtype(arr.dtype, np.floating) else 0
        if n_nan:
            logger.warning("variable %s has %d NaNs (%.2f%%)", name, n_nan, 100.0 * n_nan / arr.size)
        out[name] = arr
    if "time" in dataset.dims:
        out = with_sim_time(out, dataset["time"].values, reference_datetime, time_scale_hours)
    return out


def forcings_from_xarray(dataset, forcing_variables: Optional[Sequence[str]] = None, reference_datetime=None,
                         time_scale_hours: float = 1.0) -> dict:
    return inputs_from_xarray(dataset, forcing_variables, reference_datetime, time_scale_hours)


# ───────────────────────── forcing providers ─────────────────────────


class DynamicDataForcing:
    """Nearest-time forcing lookup; NaN fields when the nearest time is farther than ``dt_tolerance``."""

    def __init__(self, times, data: dict, dt_tolerance: float = 1.0):
        self.times = np.asarray(times, dtype=np.float64).ravel()
        self.data = data
        self.dt_tolerance = float(dt_tolerance)

    def __call__(self, sim_time: float) -> dict:
        i = int(np.argmin(np.abs(self.times - float(sim_time))))
        far = abs(self.times[i] - float(sim_time)) > self.dt_tolerance
        out = {}
        for k, a in self.data.items():
            v = torch.as_tensor(np.asarray(a[i]), dtype=torch.float32)
            out[k] = torch.full_like(v, float("nan")) if far else v
        return out


class PersistenceDataForcing:
    """Always the first time slice."""

    def __init__(self, data: dict):
        self._forcing = {k: torch.as_tensor(np.asarray(a[0]), dtype=torch.float32) for k, a in data.items()}

    def __call__(self, sim_time: float) -> dict:
        return dict(self._forcing)


class Climatology:
    """Day-of-year climatology (nearest tabulated day)."""

    def __init__(self, climatology: dict, times_dayofyear: Optional[np.ndarray] = None):
        self.climatology = climatology
        n = next(iter(climatology.values())).shape[0]
        self.times_dayofyear = np.arange(1, n + 1) if times_dayofyear is None else np.asarray(times_dayofyear)

    def __call__(self, dayofyear: int) -> dict:
        i = int(np.argmin(np.abs(self.times_dayofyear - dayofyear)))
        return {k: torch.as_tensor(np.asarray(a[i]), dtype=torch.float32) for k, a in self.climatology.items()}


class AnomalyPersistence:
    """``climatology(t) + (x(t0) - climatology(t0))``, with fractions clipped to [0, 1]."""

    def __init__(self, initial_data: dict, climatology: Climatology, initial_dayofyear: int,
                 clip_variables: Sequence[str] = ("sea_ice_cover",)):
        c0 = climatology(initial_dayofyear)
        self.anomaly = {k: torch.as_tensor(np.asarray(v), dtype=torch.float32) - c0[k]
                        for k, v in initial_data.items() if k in c0}
        self.climatology = climatology
        self.clip_variables = set(clip_variables)

    def __call__(self, dayofyear: int) -> dict:
        out = {}
        for k, c in self.climatology(dayofyear).items():
            v = c + self.anomaly[k] if k in self.anomaly else c
            out[k] = v.clamp(0.0, 1.0) if k in self.clip_variables else v
        return out


def selective_temporal_shift(data: dict, variables: Sequence[str], shift: int) -> dict:
    """Selected variables lag the others by ``shift`` steps (negative: lead); time cut to the overlap."""
    if shift == 0:
        return data
    T = next(iter(data.values())).shape[0]
    s = abs(shift)
    sel, rest = (slice(0, T - s), slice(s, T)) if shift > 0 else (slice(s, T), slice(0, T - s))
    return {k: a[sel] if k in variables else a[rest] for k, a in data.items()}


# ───────────────────────── regridding ─────────────────────────


class BilinearRegridder:
    """Bilinear ``(…, lon, lat)`` regridding; longitude periodic, latitude clamped."""

    def __init__(self, source_lon, source_lat, target_lon, target_lat, degrees: bool = True):
        conv = np.deg2rad if degrees else (lambda x: np.asarray(x, dtype=np.float64))
        self._lon_idx, self._lon_w = self._interp_weights(conv(source_lon), conv(target_lon), True)
        self._lat_idx, self._lat_w = self._interp_weights(conv(source_lat), conv(target_lat), False)

    @staticmethod
    def _interp_weights(src: np.ndarray, tgt: np.ndarray, periodic: bool):
        src, tgt = np.asarray(src, dtype=np.float64), np.asarray(tgt, dtype=np.float64)
        n = len(src)
        if periodic:
            two_pi = 2 * np.pi
            s = np.mod(src, two_pi)
            order = np.argsort(s)
            s_sorted = s[order]
            t = np.mod(tgt, two_pi)
            j = (np.searchsorted(s_sorted, t, side="right") - 1) % n
            j1 = (j + 1) % n
            span = np.mod(s_sorted[j1] - s_sorted[j], two_pi)
            span = np.where(span == 0, two_pi, span)
            frac = np.mod(t - s_sorted[j], two_pi)
            return np.stack([order[j], order[j1]], -1), frac / span
        ascending = src[-1] >= src[0]
        s = src if ascending else src[::-1]
        j = np.clip(np.searchsorted(s, tgt) - 1, 0, n - 2)
        w = np.clip((tgt - s[j]) / np.where(s[j + 1] > s[j], s[j + 1] - s[j], 1.0), 0.0, 1.0)
        idx = np.stack([j, j + 1], -1)
        if not ascending:
            idx = n - 1 - idx
        return idx, w

    def __call__(self, field):
        is_t = torch.is_tensor(field)
        f = field if is_t else torch.as_tensor(np.asarray(field))
        dev, dt = f.device, (f.dtype if f.is_floating_point() else torch.float64)
        f = f.to(dt)
        li = torch.as_tensor(self._lat_idx, device=dev)
        lw = torch.as_tensor(self._lat_w, device=dev, dtype=dt)
        g = f[..., li[:, 0]] * (1 - lw) + f[..., li[:, 1]] * lw
        oi = torch.as_tensor(self._lon_idx, device=dev)
        ow = torch.as_tensor(self._lon_w, device=dev, dtype=dt)[:, None]
        out = g[..., oi[:, 0], :] * (1 - ow) + g[..., oi[:, 1], :] * ow
        return out if is_t else out.cpu().numpy()


class NearestNaNFiller:
    """Replace NaNs with the value of the nearest valid point on the sphere."""

    def __init__(self, lon, lat):
        lon_r, lat_r = np.deg2rad(np.asarray(lon, dtype=np.float64)), np.deg2rad(np.asarray(lat, dtype=np.float64))
        LON, LAT = np.meshgrid(lon_r, lat_r, indexing="ij")
        self._xyz = np.stack([np.cos(LAT) * np.cos(LON), np.cos(LAT) * np.sin(LON), np.sin(LAT)], -1).reshape(-1, 3)
        self.shape = LON.shape

    def fill(self, field: np.ndarray) -> np.ndarray:
        from scipy.spatial import cKDTree

        a = np.array(field, dtype=np.float64, copy=True)
        flat = a.reshape((-1,) + (int(np.prod(self.shape)),))
        for row in flat:
            bad = np.isnan(row)
            if not bad.any() or bad.all():
                continue
            tree = cKDTree(self._xyz[~bad])
            _, nn = tree.query(self._xyz[bad])
            row[bad] = row[~bad][nn]
        return flat.reshape(a.shape).astype(np.asarray(field).dtype, copy=False)

    __call__ = fill
