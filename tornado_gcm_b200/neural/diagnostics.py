"""Trajectory diagnostics: energy / mass proxies (reference ``neural/diagnostics.py:23-182``)."""

from __future__ import annotations

import torch

from tornado_gcm_b200.core.primitive_equations import State


def total_energy_proxy(state: State) -> torch.Tensor:
    dims = (-3, -2, -1)
    return ((state.vorticity ** 2 + state.divergence ** 2).sum(dim=dims, dtype=torch.float64)
            + (state.temperature_variation ** 2).sum(dim=dims, dtype=torch.float64))


def dry_air_mass_proxy(state: State) -> torch.Tensor:
    return state.log_surface_pressure[..., 0, 0, 0].to(torch.float64)


def moisture_proxy(state: State, key: str = "specific_humidity") -> torch.Tensor:
    q = state.tracers.get(key)
    if q is None:
        return torch.zeros_like(dry_air_mass_proxy(state))
    return q[..., :, 0, 0].sum(dim=-1).to(torch.float64)


def compute_trajectory_diagnostics(trajectory: list, initial_state: State) -> dict:
    """Energies, masses and a precipitation-minus-evaporation proxy per step."""
    energies = torch.stack([total_energy_proxy(s) for s in trajectory])
    masses = torch.stack([dry_air_mass_proxy(s) for s in trajectory])
    moist = torch.stack([moisture_proxy(initial_state)] + [moisture_proxy(s) for s in trajectory])
    pme = -(moist[1:] - moist[:-1])
    return {"energies": energies, "masses": masses, "precipitation": torch.clamp(pme, min=0),
            "evaporation": torch.clamp(-pme, min=0)}


def energy_drift(trajectory: list) -> torch.Tensor:
    e = torch.stack([total_energy_proxy(s) for s in trajectory])
    return (e - e[0]) / (e[0].abs() + 1e-30)
