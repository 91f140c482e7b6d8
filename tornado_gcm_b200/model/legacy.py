"""Pressure-level model wrapper — reference ``model/legacy.py:20-161``.

:class:`PressureLevelModel` presents a hybrid model (pressure-level data →
σ-level state → rollout → pressure-level data) with the reference's
``PressureLevelConfig`` vocabulary.  Variable names follow the long
WeatherBench names; they are mapped onto the encoder's short field names.
"""

from __future__ import annotations

import dataclasses
from typing import Optional

import torch
import torch.nn as nn

LONG_TO_SHORT = {"u_component_of_wind": "u", "v_component_of_wind": "v", "temperature": "t",
                 "specific_humidity": "q", "geopotential": "z",
                 "specific_cloud_liquid_water_content": "clwc", "specific_cloud_ice_water_content": "ciwc"}
SHORT_TO_LONG = {v: k for k, v in LONG_TO_SHORT.items()}


@dataclasses.dataclass
class PressureLevelConfig:
    pressure_levels: list = dataclasses.field(default_factory=lambda: [100, 200, 300, 500, 700, 850, 925, 1000])
    input_variables: list = dataclasses.field(default_factory=lambda: [
        "u_component_of_wind", "v_component_of_wind", "temperature", "specific_humidity", "geopotential"])
    forcing_variables: list = dataclasses.field(default_factory=lambda: [
        "sea_surface_temperature", "sea_ice_cover", "geopotential_at_surface"])
    output_variables: list = dataclasses.field(default_factory=lambda: [
        "u_component_of_wind", "v_component_of_wind", "temperature", "specific_humidity", "geopotential"])
    dt_hours: float = 6.0


class PressureLevelModel(nn.Module):
    """``gcm`` is a :class:`~tornado_gcm_b200.models.builders.HybridGCM`."""

    def __init__(self, gcm: Optional[nn.Module] = None, config: Optional[PressureLevelConfig] = None,
                 atmosphere_model: Optional[nn.Module] = None):
        """``atmosphere_model`` is the reference's name for the wrapped model."""
        super().__init__()
        gcm = gcm if gcm is not None else atmosphere_model
        if gcm is None:
            raise ValueError("PressureLevelModel needs the model to wrap")
        self.gcm = gcm
        self.config = config or PressureLevelConfig()

    @property
    def input_variables(self) -> list:
        return list(self.config.input_variables)

    @property
    def forcing_variables(self) -> list:
        return list(self.config.forcing_variables)

    @property
    def output_variables(self) -> list:
        return list(self.config.output_variables)

    def _short(self, inputs: dict) -> dict:
        return {LONG_TO_SHORT.get(k, k): v for k, v in inputs.items()}

    def _forcings(self, forcings: Optional[dict]) -> dict:
        f = dict(forcings or {})
        if "geopotential_at_surface" in f and "orography" not in f:
            f["orography"] = f.pop("geopotential_at_surface") / 9.80616
        return f

    def encode(self, inputs: dict, forcings: Optional[dict] = None):
        return self.gcm.encoder(self._short(inputs), self.gcm.normalize_forcings(self._forcings(forcings)))

    def decode(self, state, forcings: Optional[dict] = None) -> dict:
        out = self.gcm.decoder(state, self.gcm.normalize_forcings(self._forcings(forcings)))
        return {SHORT_TO_LONG.get(k, k): v for k, v in out.items()
                if SHORT_TO_LONG.get(k, k) in self.config.output_variables}

    def advance(self, state, forcings: Optional[dict] = None):
        f = self.gcm.normalize_forcings(self._forcings(forcings))
        for _ in range(self.gcm.physics_steps_per_output):
            state = self.gcm.model.step(state, f)
        return state

    @torch.no_grad()
    def predict(self, inputs: dict, forcings: Optional[dict] = None, steps: int = 1,
                outer_steps: Optional[int] = None) -> list:
        """Decoded outputs after each of ``steps`` (the reference: ``outer_steps``) 6-h steps."""
        steps = outer_steps if outer_steps is not None else steps
        state = self.encode(inputs, forcings)
        out = []
        for _ in range(steps):
            state = self.advance(state, forcings)
            out.append(self.decode(state, forcings))
        return out

    def inputs_from_xarray(self, dataset) -> dict:
        return {k: torch.as_tensor(dataset[k].values) for k in self.config.input_variables}

    def forcings_from_xarray(self, dataset) -> dict:
        return {k: torch.as_tensor(dataset[k].values) for k in self.config.forcing_variables if k in dataset}
