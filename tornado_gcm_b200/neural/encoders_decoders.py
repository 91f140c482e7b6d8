"""Pressure-level data ↔ model state — reference ``neural/encoders_decoders.py:32-495``.

* :class:`WeatherbenchToPrimitiveEncoder`: surface pressure from geopotential
  and surface geopotential, linear interpolation of (u, v, T, q) from
  pressure levels to σ·ps, (u, v) → (ζ, δ), ``T' = T - T_ref``, ln ps; all
  fields go to modal space in one batched transform.
* :class:`LearnedWeatherbenchToPrimitiveEncoder`: the same plus a network
  correction (nodal or modal) for selected fields.
* :class:`PrimitiveToWeatherbenchDecoder`: u, v, T, geopotential (with
  virtual-temperature correction when humidity is present) and tracers on σ
  levels, interpolated to the output pressure levels; the nodal fields come
  from one batched synthesis.
* :class:`LearnedPrimitiveToWeatherbenchDecoder`: optional randomness and
  state perturbation, decoder diagnostics, model-space and data-space features
  (``model_`` / ``data_`` prefixes), masked additive corrections and an
  output transform.

Velocities are recovered as ``(cosφ·u)·secφ`` (the reference decoder scales by
``sec²φ``, ``neural/encoders_decoders.py:300-302``, which is not the inverse of
its encoder).
"""

from __future__ import annotations

from typing import Dict, Optional

import numpy as np
import torch
import torch.nn as nn

from tornado_gcm_b200.core import primitive_equations as pe
from tornado_gcm_b200.core import spherical_harmonic
from tornado_gcm_b200.core import vertical_interpolation as vi
from tornado_gcm_b200.neural.transforms import batched_to_modal
from tornado_gcm_b200.utils.typing import KeyWithCosLatFactor


def _state_dict(state: pe.State) -> Dict[str, torch.Tensor]:
    d = {"vorticity": state.vorticity, "divergence": state.divergence,
         "temperature_variation": state.temperature_variation, "log_surface_pressure": state.log_surface_pressure}
    d.update(state.tracers)
    return d


class WeatherbenchToPrimitiveEncoder(nn.Module):
    def __init__(self, coords, physics_specs, reference_temperatures, input_pressure_levels,
                 orography: Optional[torch.Tensor] = None):
        super().__init__()
        self.coords = coords
        self.physics_specs = physics_specs
        self.ref_temps = np.asarray(reference_temperatures, dtype=np.float64)
        self.input_pressure = vi.PressureCoordinates(np.asarray(input_pressure_levels))
        if orography is not None:
            self.register_buffer("_orography", torch.as_tensor(orography), persistent=False)
        else:
            self._orography = None

    def weatherbench_to_primitive(self, wb_dict: Dict[str, torch.Tensor]) -> pe.State:
        """``wb_dict``: ``u_component_of_wind``, ``v_component_of_wind``, ``temperature``,
        ``geopotential`` (``(n_pressure, lon, lat)``), optional ``specific_humidity``
        and other tracers on the same levels, optional ``geopotential_at_surface``."""
        grid, vertical = self.coords.horizontal, self.coords.vertical
        g = self.physics_specs.g
        t = wb_dict["temperature"]
        geo = wb_dict["geopotential"]
        if "geopotential_at_surface" in wb_dict:
            zs = wb_dict["geopotential_at_surface"] / g
        elif self._orography is not None:
            zs = self._orography.to(t.device, t.dtype)
        else:
            zs = torch.zeros_like(geo[..., -1:, :, :])
        ps = vi.get_surface_pressure(self.input_pressure, geo, zs, g)             # (…, 1, lon, lat)
        names = {"u": wb_dict["u_component_of_wind"], "v": wb_dict["v_component_of_wind"], "t": t}
        tracer_keys = [k for k, v in wb_dict.items() if k.startswith("specific_") and torch.is_tensor(v)
                       and v.shape[-3:] == t.shape[-3:]]
        for k in tracer_keys:
            names[k] = wb_dict[k]
        on_sigma = vi.interp_pressure_to_sigma(names, self.input_pressure, vertical, ps)
        cos = torch.as_tensor(grid.cos_lat, dtype=t.dtype, device=t.device)
        t_ref = torch.as_tensor(self.ref_temps, dtype=t.dtype, device=t.device).reshape(-1, 1, 1)
        modal = batched_to_modal(grid, {"u": on_sigma["u"] / cos, "v": on_sigma["v"] / cos,
                                        "t": on_sigma["t"] - t_ref, "lnps": torch.log(ps),
                                        **{k: on_sigma[k] for k in tracer_keys}})
        vor = grid.curl_cos_lat((modal["u"], modal["v"]))
        div = grid.div_cos_lat((modal["u"], modal["v"]))
        return pe.State(vor, div, modal["t"], modal["lnps"], {k: modal[k] for k in tracer_keys})

    def forward(self, wb_dict: Dict[str, torch.Tensor]) -> pe.State:
        return self.weatherbench_to_primitive(wb_dict)


class LearnedWeatherbenchToPrimitiveEncoder(WeatherbenchToPrimitiveEncoder):
    """Physics encoding plus ``correction_net(features_fn(state))`` on the fields that
    ``prediction_mask`` does not switch off.  Nodal corrections are transformed
    in one batched analysis."""

    def __init__(self, coords, physics_specs, reference_temperatures, input_pressure_levels, features_fn: nn.Module,
                 correction_net: nn.Module, correction_transform: Optional[nn.Module] = None,
                 prediction_mask: Optional[Dict[str, bool]] = None, orography: Optional[torch.Tensor] = None):
        super().__init__(coords, physics_specs, reference_temperatures, input_pressure_levels, orography)
        self.features_fn = features_fn
        self.correction_net = correction_net
        self.correction_transform = correction_transform
        self.prediction_mask = prediction_mask or {}

    def forward(self, wb_dict: Dict[str, torch.Tensor], forcing: Optional[Dict[str, torch.Tensor]] = None) -> pe.State:
        st = self.weatherbench_to_primitive(wb_dict)
        corr = self.correction_net(self.features_fn(_state_dict(st), forcing=forcing))
        if self.correction_transform is not None:
            corr = self.correction_transform(corr)
        fields = _state_dict(st)
        use = {k: c for k, c in corr.items() if k in fields and self.prediction_mask.get(k, True) and c is not None}
        nodal = {k: c for k, c in use.items() if c.shape != fields[k].shape}
        modal = batched_to_modal(self.coords.horizontal, nodal)
        for k, c in use.items():
            fields[k] = fields[k] + (modal[k] if k in modal else c)
        tracers = {k: fields[k] for k in st.tracers}
        return pe.State(fields["vorticity"], fields["divergence"], fields["temperature_variation"],
                        fields["log_surface_pressure"], tracers, st.sim_time)


class PrimitiveToWeatherbenchDecoder(nn.Module):
    def __init__(self, coords, physics_specs, reference_temperatures, output_pressure_levels,
                 orography: Optional[torch.Tensor] = None):
        super().__init__()
        self.coords = coords
        self.physics_specs = physics_specs
        self.ref_temps = np.asarray(reference_temperatures, dtype=np.float64)
        self.output_pressure = vi.PressureCoordinates(np.asarray(output_pressure_levels))
        if orography is not None:
            self.register_buffer("_orography", torch.as_tensor(orography), persistent=False)
        else:
            self._orography = None

    def _nodal_orography(self, like: torch.Tensor) -> torch.Tensor:
        if self._orography is None:
            return torch.zeros_like(like[..., :1, :, :])
        o = self._orography.to(like.device, like.dtype)
        if tuple(o.shape[-2:]) == tuple(self.coords.horizontal.modal_shape):
            o = self.coords.horizontal.to_nodal(o)
        return o

    def primitive_to_weatherbench(self, state: pe.State) -> Dict[str, torch.Tensor]:
        grid, vertical = self.coords.horizontal, self.coords.vertical
        cu, cv = spherical_harmonic.get_cos_lat_vector(state.vorticity, state.divergence, grid, clip=False)
        modal = {KeyWithCosLatFactor("u_component_of_wind", 1): cu, KeyWithCosLatFactor("v_component_of_wind", 1): cv,
                 KeyWithCosLatFactor("t", 0): state.temperature_variation,
                 KeyWithCosLatFactor("lnps", 0): state.log_surface_pressure}
        for k, v in state.tracers.items():
            modal[KeyWithCosLatFactor(k, 0)] = v
        from tornado_gcm_b200.neural.features import modal_features_to_nodal

        nod = modal_features_to_nodal(grid, modal)
        dtype, device = nod["t"].dtype, nod["t"].device
        t = nod.pop("t") + torch.as_tensor(self.ref_temps, dtype=dtype, device=device).reshape(-1, 1, 1)
        ps = torch.exp(nod.pop("lnps"))
        q = nod.get("specific_humidity")
        geo = pe.get_geopotential_on_sigma(t, self._nodal_orography(t), vertical, self.physics_specs.g,
                                           self.physics_specs.R, specific_humidity=q,
                                           water_vapor_gas_constant=self.physics_specs.R_vapor if q is not None
                                           else None)
        fields = {"temperature": t, "geopotential": geo, **nod}
        out = vi.interp_sigma_to_pressure(fields, self.output_pressure, vertical, ps)
        out["surface_pressure"] = ps
        return out

    def forward(self, state: pe.State) -> Dict[str, torch.Tensor]:
        return self.primitive_to_weatherbench(state)


def _add_prefix(d: Dict, prefix: str) -> Dict:
    return {prefix + k: v for k, v in d.items()}


class LearnedPrimitiveToWeatherbenchDecoder(PrimitiveToWeatherbenchDecoder):
    def __init__(self, coords, physics_specs, reference_temperatures, output_pressure_levels,
                 model_features_fn: nn.Module, correction_net: nn.Module, data_features_fn: Optional[nn.Module] = None,
                 correction_transform: Optional[nn.Module] = None, prediction_mask: Optional[Dict[str, bool]] = None,
                 randomness_fn: Optional[nn.Module] = None, perturbation_fn: Optional[nn.Module] = None,
                 diagnostic_fn: Optional[nn.Module] = None, transform_fn: Optional[nn.Module] = None,
                 orography: Optional[torch.Tensor] = None):
        super().__init__(coords, physics_specs, reference_temperatures, output_pressure_levels, orography)
        self.model_features_fn = model_features_fn
        self.data_features_fn = data_features_fn
        self.correction_net = correction_net
        self.correction_transform = correction_transform
        self.prediction_mask = prediction_mask or {}
        self.randomness_fn = randomness_fn
        self.perturbation_fn = perturbation_fn
        self.diagnostic_fn = diagnostic_fn
        self.transform_fn = transform_fn

    def forward(self, state: pe.State, forcing: Optional[Dict] = None, randomness=None) -> Dict[str, torch.Tensor]:
        noise = None
        if self.randomness_fn is not None:
            kw = {} if randomness is None else {"generator": randomness}
            rs = self.randomness_fn.unconditional_sample(device=state.vorticity.device, **kw)
            noise = rs
        if self.perturbation_fn is not None and noise is not None:
            state = self.perturbation_fn(state, noise)
        diags = self.diagnostic_fn(state) if self.diagnostic_fn is not None else None
        wb = self.primitive_to_weatherbench(state)
        if diags is not None:
            wb["diagnostics"] = diags
        kw = {"forcing": forcing}
        if noise is not None:
            kw["randomness"] = noise
        feats = self.model_features_fn(_state_dict(state), **kw)
        if self.data_features_fn is not None:
            tensors = {k: v for k, v in wb.items() if torch.is_tensor(v) and v.dim() >= 2}
            data = self.data_features_fn(batched_to_modal(self.coords.horizontal, tensors), forcing=forcing)
            feats = {**_add_prefix(data, "data_"), **_add_prefix(feats, "model_")}
        corr = self.correction_net(feats)
        if self.correction_transform is not None:
            corr = self.correction_transform(corr)
        for k in list(wb):
            c = corr.get(k)
            if c is not None and self.prediction_mask.get(k, True):
                wb[k] = wb[k] + c
        return self.transform_fn(wb) if self.transform_fn is not None else wb
