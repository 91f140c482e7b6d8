"""Atmosphere facade — reference ``model/atmosphere.py:35-281``.

:class:`AtmosphericModel` assembles an encoder, the coupled step of
:class:`~tornado_gcm_b200.models.api.NeuralGCMModel` (which owns the IMEX-SIL3
loop, filters and conservation fix in one place) and a decoder, and exposes
``encode / decode / step / forward / assimilate / observe``.  A dynamics
equation built elsewhere (for example a :class:`PrimitiveEquationsSigma`) can
be injected; a neural equation supplies the physics tendency.
"""

from __future__ import annotations

import dataclasses
from typing import Callable, Optional

import torch
import torch.nn as nn

from tornado_gcm_b200.core import coordinate_systems
from tornado_gcm_b200.models.api import ModelConfig, NeuralGCMModel
from tornado_gcm_b200.precision.policy import PrecisionPolicy
from tornado_gcm_b200.utils.typing import ModelState


@dataclasses.dataclass
class AtmosphereConfig:
    coords: coordinate_systems.CoordinateSystem
    physics_specs: object = None
    dt: float = 1.0
    inner_steps: int = 1
    dycore_substeps: int = 8
    filter_attenuation: float = 16.0
    filter_order: int = 18
    num_substeps: int = 1
    precision_policy: PrecisionPolicy = dataclasses.field(default_factory=PrecisionPolicy)
    reference_temperature: Optional[object] = None
    orography: Optional[torch.Tensor] = None


class _NeuralEquationParameterization(nn.Module):
    """Adapts ``neural_equation(state, forcings)`` to the parameterization call."""

    def __init__(self, eq: nn.Module):
        super().__init__()
        self.eq = eq

    def forward(self, state, forcings=None, memory=None):
        try:
            return self.eq(state, forcings=forcings)
        except TypeError:
            return self.eq(state)


class AtmosphericModel(nn.Module):
    def __init__(self, config: AtmosphereConfig, dynamics_equation=None, neural_equation: Optional[nn.Module] = None,
                 encoder: Optional[nn.Module] = None, decoder: Optional[nn.Module] = None,
                 stochastic_step: Optional[nn.Module] = None, conservation_fixer: Optional[nn.Module] = None,
                 diagnostics_fn: Optional[Callable] = None):
        super().__init__()
        self.config = config
        self.encoder = encoder
        self.decoder = decoder
        core = ModelConfig(coords=config.coords, dt=config.dt, inner_steps=config.inner_steps,
                           dycore_substeps=config.dycore_substeps, physics_specs=config.physics_specs,
                           precision_policy=config.precision_policy, filter_attenuation=config.filter_attenuation,
                           filter_order=config.filter_order, reference_temperature=config.reference_temperature,
                           orography=config.orography,
                           use_dycore=dynamics_equation is None and config.physics_specs is not None)
        param = _NeuralEquationParameterization(neural_equation) if neural_equation is not None else None
        self._core = NeuralGCMModel(core, parameterization=param, conservation_fixer=conservation_fixer,
                                    encoder=encoder, decoder=decoder, stochastic_step=stochastic_step,
                                    diagnostics_fn=diagnostics_fn)
        if dynamics_equation is not None:
            self._core._dycore = dynamics_equation
            self._core._dycore_equation = dynamics_equation
            self._core._inner_dt = config.dt / config.dycore_substeps

    @property
    def core(self) -> NeuralGCMModel:
        return self._core

    def encode(self, inputs, forcing=None, forcings=None):
        """``forcing`` is the reference's keyword; ``forcings`` is accepted as well."""
        return self._core.encode(inputs, forcing if forcing is not None else forcings)

    def decode(self, state, forcing=None, forcings=None):
        return self._core.decode(state, forcing if forcing is not None else forcings)

    def step(self, state, forcings=None):
        return self._core.step(state, forcings)

    def step_model_state(self, model_state: ModelState, forcings=None) -> ModelState:
        return self._core.step_model_state(model_state, forcings)

    def initialize_model_state(self, state, **kwargs) -> ModelState:
        return self._core.initialize_model_state(state, **kwargs)

    def forward(self, initial_state, outer_steps: int, inner_steps: Optional[int] = None, forcings=None,
                post_process_fn=None, checkpoint_outer_steps: bool = False):
        return self._core(initial_state, outer_steps, inner_steps, forcings=forcings, post_process_fn=post_process_fn,
                          checkpoint_outer_steps=checkpoint_outer_steps)

    def assimilate(self, inputs, forcings=None, state=None, alpha: float = 1.0):
        """Encoded ``inputs``; with ``state``, blended as ``(1 - alpha) state + alpha encoded``."""
        encoded = self.encode(inputs, forcings=forcings)
        return encoded if (state is None or alpha >= 1.0) else state * (1.0 - alpha) + encoded * alpha

    def observe(self, state, forcing=None, forcings=None):
        return self.decode(state, forcing if forcing is not None else forcings)
