"""Networks as explicit ODE terms — reference ``neural/neural_equations.py:21-211``.

``features_fn(state) → mapping → tendency_transform`` gives nodal tendencies;
they are converted to modal space in one batched analysis (the wind
tendencies of :class:`DivCurlNeuralEquations` included, as ``u·secφ``,
``v·secφ`` turned into δ, ζ tendencies by the cos-lat divergence / curl),
optionally filtered, and returned as a :class:`State` (or a dict for dict
inputs).
"""

from __future__ import annotations

from typing import Callable, Dict, Optional, Sequence

import torch
import torch.nn as nn

from tornado_gcm_b200.core import primitive_equations as pe
from tornado_gcm_b200.core import time_integration
from tornado_gcm_b200.neural.transforms import ToModalWithDivCurl, batched_to_modal


def _inputs(state) -> Dict[str, torch.Tensor]:
    if isinstance(state, pe.State):
        d = {"vorticity": state.vorticity, "divergence": state.divergence,
             "temperature_variation": state.temperature_variation,
             "log_surface_pressure": state.log_surface_pressure}
        d.update(state.tracers)
        return d
    return state


def _nodal_split(grid, tendencies: Dict) -> tuple[Dict, Dict]:
    nodal = {k: v for k, v in tendencies.items() if torch.is_tensor(v) and tuple(v.shape[-2:]) == tuple(grid.nodal_shape)}
    return nodal, {k: v for k, v in tendencies.items() if k not in nodal}


def _as_state(state, modal: Dict, keep: Optional[set] = None):
    if not isinstance(state, pe.State):
        return modal

    def get(k, like):
        if keep is not None and k not in keep:
            return torch.zeros_like(like)
        return modal.get(k, torch.zeros_like(like))

    return pe.State(get("vorticity", state.vorticity), get("divergence", state.divergence),
                    get("temperature_variation", state.temperature_variation),
                    get("log_surface_pressure", state.log_surface_pressure),
                    {k: get(k, v) for k, v in state.tracers.items()}, state.sim_time)


class DirectNeuralEquations(time_integration.ExplicitODE, nn.Module):
    def __init__(self, grid, features_fn: nn.Module, mapping: nn.Module, tendency_transform: Optional[nn.Module] = None,
                 filter_fn: Optional[Callable] = None, prediction_keys: Optional[Sequence[str]] = None):
        nn.Module.__init__(self)
        self.grid = grid
        self.features_fn = features_fn
        self.mapping = mapping
        self.tendency_transform = tendency_transform
        self.filter_fn = filter_fn
        self.prediction_keys = set(prediction_keys) if prediction_keys else None

    def _tendencies(self, state) -> Dict:
        t = self.mapping(self.features_fn(_inputs(state)))
        return self.tendency_transform(t) if self.tendency_transform is not None else t

    def _finish(self, modal: Dict) -> Dict:
        if self.filter_fn is not None:
            modal = {k: self.filter_fn(v) for k, v in modal.items()}
        return modal

    def explicit_terms(self, state):
        nodal, other = _nodal_split(self.grid, self._tendencies(state))
        modal = self._finish({**batched_to_modal(self.grid, nodal), **other})
        return _as_state(state, modal, self.prediction_keys)

    forward = explicit_terms


class DivCurlNeuralEquations(DirectNeuralEquations):
    """Wind tendencies predicted as (u, v), converted to (ζ, δ) tendencies."""

    def __init__(self, grid, features_fn: nn.Module, mapping: nn.Module, tendency_transform: Optional[nn.Module] = None,
                 filter_fn: Optional[Callable] = None, u_key: str = "u_component_of_wind",
                 v_key: str = "v_component_of_wind"):
        super().__init__(grid, features_fn, mapping, tendency_transform, filter_fn)
        self.u_key = u_key
        self.v_key = v_key
        self._to_modal = ToModalWithDivCurl(grid, u_key, v_key)

    def explicit_terms(self, state):
        modal = self._finish(self._to_modal(dict(self._tendencies(state))))
        return _as_state(state, modal)

    forward = explicit_terms
