"""Physics feature modules — reference ``neural/features.py:76-950``.

Every module maps ``(inputs, memory, diagnostics, randomness, forcing)`` to a
dict of nodal features of shape ``(channels, lon, lat)`` (leading batch axes
allowed).  Feature keys follow the reference so that packed channel orders
(sorted keys, :func:`pack_features`) match checkpoints trained with it.

The reference converts each modal field to nodal space with its own
transform call (and recomputes u, v once per module).  Here a module gathers
all the modal fields it needs, including derivative features, and converts
them in ONE batched transform (:func:`~tornado_gcm_b200.neural.transforms.batched_to_nodal`),
then applies the ``sec(lat)^order`` factors; on the GPU that is one pair of
tcgen05 GEMM launches per module instead of one pair per field.
"""

from __future__ import annotations

import math
from typing import Dict, Optional, Sequence

import numpy as np
import torch
import torch.nn as nn

from tornado_gcm_b200.core import spherical_harmonic
from tornado_gcm_b200.neural.transforms import batched_to_modal, batched_to_nodal, key_parts
from tornado_gcm_b200.utils.typing import KeyWithCosLatFactor

OROGRAPHY_KEY = "orography"
REFERENCE_DATETIME_KEY = "reference_datetime"
_SKIP = ("sim_time", "u_component_of_wind", "v_component_of_wind")


def _device_of(inputs: Dict) -> torch.device:
    for v in inputs.values():
        if isinstance(v, torch.Tensor):
            return v.device
        if isinstance(v, dict):
            for t in v.values():
                if isinstance(t, torch.Tensor):
                    return t.device
    return torch.device("cpu")


def _surface(v: torch.Tensor) -> torch.Tensor:
    return v.unsqueeze(0) if v.ndim == 2 else v


def _sec_factors(grid, device, dtype) -> dict:
    sec = torch.as_tensor(1.0 / grid.cos_lat, dtype=dtype, device=device)
    return {0: None, 1: sec, 2: sec * sec}


def modal_features_to_nodal(grid, modal: Dict) -> Dict[str, torch.Tensor]:
    """``{KeyWithCosLatFactor: modal}`` → ``{name: nodal · sec^order}`` in one batched transform."""
    if not modal:
        return {}
    keys = list(modal)
    nodal = batched_to_nodal(grid, {i: modal[k] for i, k in enumerate(keys)})
    ref = nodal[0]
    sec = _sec_factors(grid, ref.device, ref.dtype)
    out = {}
    for i, k in enumerate(keys):
        name, order = key_parts(k)
        s = sec.get(order)
        if s is None and order > 2:
            s = sec[1] ** order
        out[name] = nodal[i] if s is None else nodal[i] * s
    return out


class FeatureModule(nn.Module):
    """Base class: ``forward(inputs, memory, diagnostics, randomness, forcing) -> dict``."""

    def forward(self, inputs: Dict, memory=None, diagnostics=None, randomness=None, forcing=None) -> Dict:
        raise NotImplementedError


class RadiationFeatures(FeatureModule):
    """Clear-sky incoming solar flux proxy: ``max(cos θ_z, 0)``.

    ``cos θ_z = cosφ cosδ cos h + sinφ sinδ`` with declination
    ``δ = 23.45° sin(orbital phase - spring equinox phase)`` and hour angle
    ``h = synodic phase + λ - π``.  ``sim_time`` (in units of
    ``time_scale_hours``) drives both phases; without it the time-mean
    ``cosφ`` is returned.
    """

    EARTH_AXIS_INCLINATION = math.radians(23.45)
    SPRING_EQUINOX_PHASE = 2 * math.pi * 79.0 / 365.25
    TSI = 1361.0

    def __init__(self, grid, reference_datetime_ordinal: float = 0.0, time_scale_hours: float = 1.0):
        super().__init__()
        self.grid = grid
        self.reference_datetime_ordinal = reference_datetime_ordinal
        self.time_scale_hours = time_scale_hours

    def _orbital_phase(self, sim_time: float) -> float:
        days = sim_time * self.time_scale_hours / 24.0 + self.reference_datetime_ordinal
        return 2 * math.pi * days / 365.25

    def _synodic_phase(self, sim_time: float) -> float:
        return 2 * math.pi * ((sim_time * self.time_scale_hours) % 24.0) / 24.0

    def cos_zenith(self, sim_time: float, device=None) -> torch.Tensor:
        lon, sin_lat = self.grid.nodal_axes
        lon = torch.as_tensor(lon, dtype=torch.float32, device=device)
        sl = torch.as_tensor(sin_lat, dtype=torch.float32, device=device)
        cl = torch.sqrt(1.0 - sl * sl)
        dec = self.EARTH_AXIS_INCLINATION * math.sin(self._orbital_phase(sim_time) - self.SPRING_EQUINOX_PHASE)
        h = self._synodic_phase(sim_time) + lon - math.pi
        return cl[None, :] * math.cos(dec) * torch.cos(h)[:, None] + sl[None, :] * math.sin(dec)

    def forward(self, inputs, memory=None, diagnostics=None, randomness=None, forcing=None):
        device = _device_of(inputs)
        t = inputs.get("sim_time")
        if t is not None:
            return {"radiation": torch.clamp(self.cos_zenith(float(torch.as_tensor(t).float().mean()), device),
                                             min=0.0)[None]}
        _, sin_lat = self.grid.nodal_axes
        cl = torch.sqrt(1.0 - torch.as_tensor(sin_lat, dtype=torch.float32, device=device) ** 2)
        return {"radiation": cl.expand(self.grid.nodal_shape[0], -1)[None]}


class ForcingFeatures(FeatureModule):
    def __init__(self, forcing_to_include: Sequence[str] = ()):
        super().__init__()
        self.forcing_to_include = list(forcing_to_include)

    def forward(self, inputs, memory=None, diagnostics=None, randomness=None, forcing=None):
        if forcing is None:
            return {}
        return {k: _surface(forcing[k]) for k in self.forcing_to_include if k in forcing}


class PressureFeatures(FeatureModule):
    """``p_k = σ_k · exp(lnps)`` on every level."""

    def __init__(self, grid, sigma_centers):
        super().__init__()
        self.grid = grid
        self.register_buffer("_sigma_centers", torch.as_tensor(np.asarray(sigma_centers), dtype=torch.float32),
                             persistent=False)

    def forward(self, inputs, memory=None, diagnostics=None, randomness=None, forcing=None):
        lnps = inputs.get("log_surface_pressure")
        if lnps is None:
            return {}
        ps = torch.exp(self.grid.to_nodal(lnps))
        sig = self._sigma_centers.to(ps.device, ps.dtype).reshape(-1, 1, 1)
        return {"pressure": sig * ps}


class OrographyFeatures(FeatureModule):
    def __init__(self, nodal_orography: torch.Tensor):
        super().__init__()
        self.register_buffer("_orography", _surface(torch.as_tensor(nodal_orography)), persistent=False)

    def forward(self, inputs, memory=None, diagnostics=None, randomness=None, forcing=None):
        return {OROGRAPHY_KEY: self._orography.to(_device_of(inputs))}


class LatitudeFeatures(FeatureModule):
    def __init__(self, grid):
        super().__init__()
        self.grid = grid

    def forward(self, inputs, memory=None, diagnostics=None, randomness=None, forcing=None):
        _, sin_lat = self.grid.nodal_axes
        sl = torch.as_tensor(sin_lat, dtype=torch.float32, device=_device_of(inputs))
        n_lon = self.grid.nodal_shape[0]
        return {"sin_latitude": sl.expand(n_lon, -1)[None],
                "cos_latitude": torch.sqrt(1.0 - sl * sl).expand(n_lon, -1)[None]}


class RandomnessFeatures(FeatureModule):
    def forward(self, inputs, memory=None, diagnostics=None, randomness=None, forcing=None):
        if randomness is None:
            return {}
        if hasattr(randomness, "nodal_value"):
            v = randomness.nodal_value
            return {} if v is None else {"randomness": _surface(v)}
        return {k: _surface(v) for k, v in randomness.items()}


class VelocityAndPrognostics(FeatureModule):
    """u, v (from ζ, δ) and the prognostic fields as nodal features, plus optional
    derivative features from ``compute_gradients_fn`` (e.g.
    :class:`~tornado_gcm_b200.neural.transforms.ToModalDiffOperators`)."""

    def __init__(self, grid, fields_to_include: Optional[Sequence[str]] = None,
                 compute_gradients_fn: Optional[nn.Module] = None,
                 features_transform_fn: Optional[nn.Module] = None):
        super().__init__()
        self.grid = grid
        self.fields_to_include = None if fields_to_include is None else list(fields_to_include)
        self.compute_gradients_fn = compute_gradients_fn
        self.features_transform_fn = features_transform_fn

    def _wanted(self, key: str) -> bool:
        return self.fields_to_include is None or key in self.fields_to_include

    def modal_features(self, inputs: Dict, prefix: str = "") -> Dict:
        feats: Dict = {}
        if "vorticity" in inputs and "divergence" in inputs:
            cu, cv = spherical_harmonic.get_cos_lat_vector(inputs["vorticity"], inputs["divergence"], self.grid,
                                                           clip=False)
            feats[KeyWithCosLatFactor(prefix + "u", 1)] = cu
            feats[KeyWithCosLatFactor(prefix + "v", 1)] = cv
        for key, val in inputs.items():
            if key in _SKIP:
                continue
            if key in ("vorticity", "divergence"):
                if self.fields_to_include is not None and key in self.fields_to_include:
                    feats[KeyWithCosLatFactor(prefix + key, 0)] = val
                continue
            if key == "tracers" and isinstance(val, dict):
                for tk, tv in val.items():
                    if self._wanted(tk):
                        feats[KeyWithCosLatFactor(prefix + tk, 0)] = tv
                continue
            if isinstance(val, torch.Tensor) and self._wanted(key):
                feats[KeyWithCosLatFactor(prefix + key, 0)] = val
        if self.compute_gradients_fn is not None:
            feats.update(self.compute_gradients_fn(feats))
        return feats

    def _extract_features(self, inputs: Dict, prefix: str = "") -> Dict[str, torch.Tensor]:
        out = modal_features_to_nodal(self.grid, self.modal_features(inputs, prefix))
        return self.features_transform_fn(out) if self.features_transform_fn is not None else out

    def forward(self, inputs, memory=None, diagnostics=None, randomness=None, forcing=None):
        return self._extract_features(inputs)


class MemoryVelocityAndValues(VelocityAndPrognostics):
    """Same features of the memory state, keys prefixed ``memory_``."""

    def forward(self, inputs, memory=None, diagnostics=None, randomness=None, forcing=None):
        if memory is None:
            return {}
        return self._extract_features(memory, prefix="memory_")


class CombinedFeatures(FeatureModule):
    """Union of several modules' features; duplicate keys are an error."""

    def __init__(self, feature_modules: Sequence[nn.Module], features_to_exclude: Sequence[str] = ()):
        super().__init__()
        self.feature_modules = nn.ModuleList(feature_modules)
        self.features_to_exclude = set(features_to_exclude)

    def forward(self, inputs, memory=None, diagnostics=None, randomness=None, forcing=None):
        out: Dict[str, torch.Tensor] = {}
        for mod in self.feature_modules:
            for k, v in mod(inputs, memory=memory, diagnostics=diagnostics, randomness=randomness,
                            forcing=forcing).items():
                if k in self.features_to_exclude:
                    continue
                if k in out:
                    raise ValueError(f"Duplicate feature key: {k}")
                out[k] = v
        return out


class FloatDataFeatures(FeatureModule):
    """Static nodal covariates (e.g. land-sea mask, surface geopotential), with
    optional derivative features computed spectrally (one batched analysis,
    one batched synthesis)."""

    def __init__(self, grid, covariates: Dict[str, torch.Tensor], compute_gradients_fn: Optional[nn.Module] = None):
        super().__init__()
        self.grid = grid
        self.compute_gradients_fn = compute_gradients_fn
        self._cov_keys = list(covariates)
        for k, v in covariates.items():
            self.register_buffer(f"_cov_{k}", _surface(torch.as_tensor(v)), persistent=False)

    def forward(self, inputs, memory=None, diagnostics=None, randomness=None, forcing=None):
        device = _device_of(inputs)
        feats = {k: getattr(self, f"_cov_{k}").to(device) for k in self._cov_keys}
        if self.compute_gradients_fn is not None and feats:
            modal = batched_to_modal(self.grid, feats)
            grads = self.compute_gradients_fn({KeyWithCosLatFactor(k, 0): v for k, v in modal.items()})
            feats.update(modal_features_to_nodal(self.grid, grads))
        return feats


class LearnedPositionalFeatures(FeatureModule):
    """A learned ``(latent, lon, lat)`` field returned as is."""

    def __init__(self, positional_param: nn.Parameter):
        super().__init__()
        self.positional_param = positional_param

    def forward(self, inputs, memory=None, diagnostics=None, randomness=None, forcing=None):
        return {"learned_positional_features": self.positional_param}


_VOLUME_FIELDS = ("divergence", "vorticity", "u", "v", "temperature_variation", "specific_humidity",
                  "specific_cloud_liquid_water_content", "specific_cloud_ice_water_content")


def _velocity_and_fields(grid, inputs: Dict, fields: Sequence[str], level_slice=None) -> Dict[str, torch.Tensor]:
    """Nodal u, v (physical, sec-scaled) and the listed state fields in one batched transform."""
    modal: Dict = {}
    if "vorticity" in inputs and "divergence" in inputs and ("u" in fields or "v" in fields):
        cu, cv = spherical_harmonic.get_cos_lat_vector(inputs["vorticity"], inputs["divergence"], grid, clip=False)
        if "u" in fields:
            modal[KeyWithCosLatFactor("u", 1)] = cu
        if "v" in fields:
            modal[KeyWithCosLatFactor("v", 1)] = cv
    for key, val in inputs.items():
        if key == "tracers" and isinstance(val, dict):
            for tk, tv in val.items():
                if tk in fields:
                    modal[KeyWithCosLatFactor(tk, 0)] = tv
        elif key in fields and key not in _SKIP and isinstance(val, torch.Tensor):
            modal[KeyWithCosLatFactor(key, 0)] = val
    if level_slice is not None:
        modal = {k: v[..., level_slice, :, :] for k, v in modal.items()}
    return modal_features_to_nodal(grid, modal)


class EmbeddingVolumeFeatures(FeatureModule):
    """Volume fields + pressure stacked as ``(channels, levels, lon, lat)`` in sorted-key
    order, passed through a vertical conv tower, split into ``{feature_name}_{i}``."""

    def __init__(self, grid, conv_tower: nn.Module, sigma_centers, n_output: int = 32, feature_name: str = "CNN1D",
                 volume_fields: Sequence[str] = _VOLUME_FIELDS, embedding_scales: Optional[Dict] = None,
                 embedding_shifts: Optional[Dict] = None):
        super().__init__()
        self.grid = grid
        self.conv_tower = conv_tower
        self.n_output = n_output
        self.feature_name = feature_name
        self.volume_fields = list(volume_fields)
        self.register_buffer("_sigma_centers", torch.as_tensor(np.asarray(sigma_centers), dtype=torch.float32),
                             persistent=False)
        self.embedding_scales = embedding_scales
        self.embedding_shifts = embedding_shifts

    def _extract_volume_features(self, inputs: Dict) -> Dict[str, torch.Tensor]:
        feats = _velocity_and_fields(self.grid, inputs, self.volume_fields)
        lnps = inputs.get("log_surface_pressure")
        if lnps is not None:
            ps = torch.exp(self.grid.to_nodal(lnps))
            feats["pressure"] = self._sigma_centers.to(ps.device, ps.dtype).reshape(-1, 1, 1) * ps
        tmpl = next((feats[k] for k in ("specific_humidity", "temperature_variation", "u", "vorticity",
                                        "divergence") if k in feats), None)
        if tmpl is None and feats:
            tmpl = next(iter(feats.values()))
        if tmpl is not None:  # absent tracers enter as zeros so the channel count is fixed
            for name in self.volume_fields:
                feats.setdefault(name, torch.zeros_like(tmpl))
        return feats

    def forward(self, inputs, memory=None, diagnostics=None, randomness=None, forcing=None):
        feats = self._extract_volume_features(inputs)
        if self.embedding_scales is not None and self.embedding_shifts is not None:
            feats = {k: (v - self.embedding_shifts[k]) / self.embedding_scales[k]
                     if k in self.embedding_scales and k in self.embedding_shifts else v for k, v in feats.items()}
        stacked = torch.stack([feats[k] for k in sorted(feats)], dim=0)
        out = self.conv_tower(stacked)
        return {f"{self.feature_name}_{i}": out[i] for i in range(self.n_output)}


class EmbeddingSurfaceFeatures(FeatureModule):
    """Land / sea / sea-ice surface embedding (NeuralGCM ``NodalLandSeaIceEmbedding``).

    Bottom-level (u, v, T', q) feed the land and sea-ice towers, SST the sea
    tower; the outputs are blended with weights ``land``,
    ``(1-land)(1-ice)`` and ``(1-land)·ice``.
    """

    def __init__(self, grid, land_epd: nn.Module, sea_epd: nn.Module, sea_ice_epd: nn.Module,
                 land_sea_mask: torch.Tensor, land_norm: tuple, sea_norm: tuple, sea_ice_norm: tuple,
                 output_size: int = 8):
        super().__init__()
        self.grid = grid
        self.land_epd, self.sea_epd, self.sea_ice_epd = land_epd, sea_epd, sea_ice_epd
        self.output_size = output_size
        self.register_buffer("_land_mask", _surface(torch.as_tensor(land_sea_mask)), persistent=False)
        self.land_scales, self.land_shifts = land_norm
        self.sea_scales, self.sea_shifts = sea_norm
        self.sea_ice_scales, self.sea_ice_shifts = sea_ice_norm

    def _extract_bottom_level_features(self, inputs: Dict,
                                       fields: Sequence[str] = ("u", "v", "temperature_variation",
                                                                "specific_humidity")) -> Dict[str, torch.Tensor]:
        return _velocity_and_fields(self.grid, inputs, fields, level_slice=slice(-1, None))

    @staticmethod
    def _normalize(feats: Dict, scales: Dict, shifts: Dict) -> Dict:
        return {k: (v - shifts[k]) / scales[k] if k in scales and k in shifts else v for k, v in feats.items()}

    @staticmethod
    def _pack_sorted(feats: Dict) -> torch.Tensor:
        return torch.cat([feats[k] for k in sorted(feats)], dim=0)

    def forward(self, inputs, memory=None, diagnostics=None, randomness=None, forcing=None):
        device = _device_of(inputs)
        bottom = self._extract_bottom_level_features(inputs)
        land_out = self.land_epd(self._pack_sorted(self._normalize(bottom, self.land_scales, self.land_shifts)))
        forcing = forcing or {}
        if "sea_surface_temperature" in forcing:
            sea_in = self._normalize({"sea_surface_temperature": _surface(forcing["sea_surface_temperature"]).to(
                device)}, self.sea_scales, self.sea_shifts)
            sea_out = self.sea_epd(self._pack_sorted(sea_in))
        else:
            sea_out = self.sea_epd(land_out.new_zeros((1,) + tuple(land_out.shape[1:])))
        ice = dict(bottom)
        sic = forcing.get("sea_ice_cover")
        ice["sea_ice_cover"] = _surface(sic).to(device) if sic is not None else torch.zeros_like(
            next(iter(bottom.values())))
        ice_out = self.sea_ice_epd(self._pack_sorted(self._normalize(ice, self.sea_ice_scales, self.sea_ice_shifts)))
        land = self._land_mask.to(device, land_out.dtype)
        sea = 1.0 - land
        ice_frac = _surface(sic).to(device, land_out.dtype) if sic is not None else torch.zeros_like(land)
        emb = land * land_out + (1.0 - ice_frac) * sea * sea_out + ice_frac * sea * ice_out
        return {"surface_embedding": emb}


def pack_features(features: Dict[str, torch.Tensor]) -> torch.Tensor:
    """Concatenate features along the channel axis in sorted-key order."""
    return torch.cat([_surface(features[k]) for k in sorted(features)], dim=0)
