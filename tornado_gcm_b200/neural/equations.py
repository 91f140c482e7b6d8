"""Dict-state equation wrappers — reference ``neural/equations.py:35-408``.

* :func:`get_reference_temperature`: log-pressure interpolation of a
  standard-atmosphere profile onto σ, hybrid or pressure levels.
* :func:`temperature_linearize` / :func:`temperature_delinearize`.
* :class:`PrimitiveEquations`: the core σ-coordinate IMEX equations with
  ``dict`` states (``temperature`` ↔ ``temperature_variation`` handled at the
  boundary); :class:`MoistPrimitiveEquations` (humidity in the virtual
  temperature) and :class:`MoistPrimitiveEquationsWithCloudMoisture`
  (humidity plus condensate loading).  The reference's moist class reads an
  undefined ``CLOUD_KEYS`` (``neural/equations.py:372``) and its cloud class
  never passes its cloud keys to the core equations; both are wired here.
* :class:`HeldSuarezForcing` (Held & Suarez 1994): Rayleigh friction
  ``-k_v(σ)·(ζ, δ)`` applied directly to the modal fields (``k_v`` has no
  horizontal dependence, so no transform is needed) and Newtonian relaxation
  ``-k_T(φ, σ)(T - T_eq)`` with ``k_T = k_a + (k_s - k_a) max(0, (σ-σ_b)/(1-σ_b)) cos⁴φ``
  as in the paper (the reference uses ``cos²φ``).
* :class:`SimTimeEquation`.
"""

from __future__ import annotations

from typing import Dict, Optional, Sequence

import numpy as np
import torch

from tornado_gcm_b200.core import primitive_equations as pe
from tornado_gcm_b200.core import time_integration
from tornado_gcm_b200.neural import field_utils
from tornado_gcm_b200.neural.coordinates import HybridLevels, PressureLevels, SigmaLevels

# US standard atmosphere (1976) temperature at the given pressures, Pa → K
REF_PRESSURE = np.array([100, 200, 300, 500, 700, 1000, 2000, 3000, 5000, 7000, 10000, 15000, 20000, 25000, 30000,
                         40000, 50000, 60000, 70000, 85000, 100000], dtype=np.float64)
REF_TEMPERATURE = np.array([262.0, 250.9, 243.2, 233.7, 228.4, 225.9, 220.0, 226.5, 217.6, 216.6, 216.6, 216.6,
                            216.6, 221.5, 228.5, 241.5, 252.4, 262.2, 271.0, 282.4, 288.1], dtype=np.float64)
P_SURF_REF = 101_325.0

VORTICITY_KEY = "vorticity"
DIVERGENCE_KEY = "divergence"
TEMPERATURE_KEY = "temperature"
TEMPERATURE_VAR_KEY = "temperature_variation"
LOG_SP_KEY = "log_surface_pressure"
SIM_TIME_KEY = "sim_time"
CLOUD_KEYS = ("specific_cloud_liquid_water_content", "specific_cloud_ice_water_content")


def get_reference_temperature(model_levels, p_surf_ref: float = P_SURF_REF) -> np.ndarray:
    """Reference temperature at the level centres (log-pressure interpolation)."""
    if isinstance(model_levels, PressureLevels):
        p = np.asarray(model_levels.levels, dtype=np.float64)
    elif isinstance(model_levels, SigmaLevels):
        p = np.asarray(model_levels.centers) * p_surf_ref
    elif isinstance(model_levels, HybridLevels):
        a, b = np.asarray(model_levels.a_boundaries), np.asarray(model_levels.b_boundaries)
        p = 0.5 * (a[1:] + a[:-1]) + 0.5 * (b[1:] + b[:-1]) * p_surf_ref
    else:
        raise TypeError(f"Unsupported level type: {type(model_levels)}")
    return np.interp(np.log(p), np.log(REF_PRESSURE), REF_TEMPERATURE)


def temperature_linearize(state_dict: Dict, ref_temperatures, abs_key: str = TEMPERATURE_KEY,
                          del_key: str = TEMPERATURE_VAR_KEY) -> Dict:
    out = dict(state_dict)
    if abs_key in out:
        out[del_key] = field_utils.extract_1d_field_perturbation(out.pop(abs_key), ref_temperatures, axis=-3)
    return out


def temperature_delinearize(state_dict: Dict, ref_temperatures, abs_key: str = TEMPERATURE_KEY,
                            del_key: str = TEMPERATURE_VAR_KEY) -> Dict:
    out = dict(state_dict)
    if del_key in out:
        out[abs_key] = field_utils.reconstruct_1d_field_from_ref_values(out.pop(del_key), ref_temperatures, axis=-3)
    return out


def _dict_to_state(d: Dict, tracer_names: Sequence[str] = ()) -> pe.State:
    t = d.get(SIM_TIME_KEY)
    return pe.State(d[VORTICITY_KEY], d[DIVERGENCE_KEY], d[TEMPERATURE_VAR_KEY], d[LOG_SP_KEY],
                    {k: d[k] for k in tracer_names if k in d}, None if t is None else float(t))


def _state_to_dict(s: pe.State, include_tracers: bool = True) -> Dict:
    out = {VORTICITY_KEY: s.vorticity, DIVERGENCE_KEY: s.divergence, TEMPERATURE_VAR_KEY: s.temperature_variation,
           LOG_SP_KEY: s.log_surface_pressure}
    if include_tracers:
        out.update(s.tracers)
    return out


class PrimitiveEquations(time_integration.ImplicitExplicitODE):
    """Core σ-coordinate equations with ``dict`` or :class:`State` inputs."""

    def __init__(self, coords, physics_specs, reference_temperatures, orography, tracer_names: Sequence[str] = (),
                 include_vertical_advection: bool = True, humidity_key: Optional[str] = None,
                 cloud_keys: Optional[tuple] = None):
        self.tracer_names = list(tracer_names)
        self.ref_temps = np.asarray(reference_temperatures, dtype=np.float64)
        self.core = pe.PrimitiveEquationsSigma(reference_temperature=self.ref_temps, orography=orography,
                                               coords=coords, physics_specs=physics_specs,
                                               include_vertical_advection=include_vertical_advection,
                                               humidity_key=humidity_key, cloud_keys=cloud_keys)
        self._core_eq = self.core

    def _to_state(self, d: Dict) -> pe.State:
        return _dict_to_state(temperature_linearize(d, torch.as_tensor(self.ref_temps)), self.tracer_names)

    def _from_state(self, s: pe.State, is_tendency: bool = True) -> Dict:
        out = _state_to_dict(s)
        return out if is_tendency else temperature_delinearize(out, torch.as_tensor(self.ref_temps))

    def explicit_terms(self, state):
        if isinstance(state, dict):
            return self._from_state(self.core.explicit_terms(self._to_state(state)))
        return self.core.explicit_terms(state)

    def implicit_terms(self, state):
        if isinstance(state, dict):
            return self._from_state(self.core.implicit_terms(self._to_state(state)))
        return self.core.implicit_terms(state)

    def implicit_inverse(self, state, step_size):
        if isinstance(state, dict):
            return self._from_state(self.core.implicit_inverse(self._to_state(state), step_size), is_tendency=False)
        return self.core.implicit_inverse(state, step_size)


class MoistPrimitiveEquations(PrimitiveEquations):
    """Humidity enters the virtual temperature (no condensate loading)."""

    def __init__(self, coords, physics_specs, reference_temperatures, orography,
                 tracer_names: Sequence[str] = ("specific_humidity",), include_vertical_advection: bool = True):
        super().__init__(coords, physics_specs, reference_temperatures, orography, tracer_names,
                         include_vertical_advection, humidity_key="specific_humidity", cloud_keys=None)


class MoistPrimitiveEquationsWithCloudMoisture(PrimitiveEquations):
    """Humidity in the virtual temperature plus cloud liquid / ice loading."""

    CLOUD_KEYS = CLOUD_KEYS

    def __init__(self, coords, physics_specs, reference_temperatures, orography,
                 tracer_names: Sequence[str] = ("specific_humidity",) + CLOUD_KEYS,
                 include_vertical_advection: bool = True):
        super().__init__(coords, physics_specs, reference_temperatures, orography, tracer_names,
                         include_vertical_advection, humidity_key="specific_humidity", cloud_keys=self.CLOUD_KEYS)


class SimTimeEquation(time_integration.ExplicitODE):
    """``d(sim_time)/dt = 1``; every other entry has zero tendency."""

    def explicit_terms(self, state):
        if isinstance(state, dict):
            out = {k: torch.zeros_like(v) for k, v in state.items()}
            if SIM_TIME_KEY in out:
                out[SIM_TIME_KEY] = torch.ones_like(out[SIM_TIME_KEY])
            return out
        return state


class HeldSuarezForcing(time_integration.ExplicitODE):
    """Held–Suarez idealised forcing as an explicit tendency on a :class:`State`.

    Rates ``kf, ka, ks`` are non-dimensional (inverse model time units).
    """

    def __init__(self, coords, physics_specs, reference_temperatures, sigma_b: float = 0.7, kf: float = 1.0,
                 ka: float = 1.0 / 40, ks: float = 1.0 / 4, min_t: float = 200.0, max_t: float = 315.0,
                 d_ty: float = 60.0, d_thz: float = 10.0):
        self.coords = coords
        self.physics_specs = physics_specs
        self.ref_temps = np.asarray(reference_temperatures, dtype=np.float64)
        self.sigma_b, self.kf, self.ka, self.ks = sigma_b, kf, ka, ks
        self.min_t, self.max_t, self.d_ty, self.d_thz = min_t, max_t, d_ty, d_thz
        sig = np.asarray(coords.vertical.centers, dtype=np.float64)
        _, sin_lat = coords.horizontal.nodal_axes
        cos2 = 1.0 - np.asarray(sin_lat) ** 2
        ramp = np.maximum(0.0, (sig - sigma_b) / (1.0 - sigma_b))[:, None, None]      # (n,1,1)
        self._kv = kf * ramp[:, 0, 0]                                                  # (n,)
        self._kt = ka + (ks - ka) * ramp * (cos2 ** 2)[None, None, :]                  # (n,1,J)
        kappa = float(physics_specs.kappa)
        teq = (max_t - d_ty * (1.0 - cos2)[None, None, :] - d_thz * np.log(sig)[:, None, None] * cos2[None, None, :]) \
            * (sig ** kappa)[:, None, None]
        self._teq = np.maximum(min_t, teq)                                             # (n,1,J)

    def equilibrium_temperature(self) -> np.ndarray:
        return self._teq

    def explicit_terms(self, state: pe.State) -> pe.State:
        grid = self.coords.horizontal
        x = state.vorticity
        kv = torch.as_tensor(self._kv, dtype=x.dtype, device=x.device).reshape(-1, 1, 1)
        kt = torch.as_tensor(self._kt, dtype=x.dtype, device=x.device)
        teq = torch.as_tensor(self._teq, dtype=x.dtype, device=x.device)
        tref = torch.as_tensor(self.ref_temps, dtype=x.dtype, device=x.device).reshape(-1, 1, 1)
        t_full = grid.to_nodal(state.temperature_variation) + tref
        dT = grid.to_modal(-kt * (t_full - teq))
        return pe.State(-kv * state.vorticity, -kv * state.divergence, dT,
                        torch.zeros_like(state.log_surface_pressure),
                        {k: torch.zeros_like(v) for k, v in state.tracers.items()}, state.sim_time)
