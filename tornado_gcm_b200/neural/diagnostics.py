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


# ── reference diagnostics API (``neural/diagnostics.py:23-182``) ─────────────
def _series(trajectory: list, initial_state: State, fn) -> torch.Tensor:
    return torch.stack([fn(initial_state)] + [fn(s) for s in trajectory])


def extract_energies(trajectory: list, initial_state: State) -> torch.Tensor:
    """Energy proxy (FP64 sum of ζ² + δ² + T'²) of the initial state and every saved step: (K+1, ...)."""
    from tornado_gcm_b200.neural.fixers import compute_total_energy

    return _series(trajectory, initial_state, compute_total_energy)


def extract_masses(trajectory: list, initial_state: State) -> torch.Tensor:
    """Dry-air mass proxy (the global mean of ln p_s) of the initial state and every saved step."""
    from tornado_gcm_b200.neural.fixers import compute_dry_air_mass

    return _series(trajectory, initial_state, compute_dry_air_mass)


def extract_precipitation_evaporation(trajectory: list, key: str = "specific_humidity") -> tuple:
    """Split the change of column humidity between saved steps into (precipitation, evaporation).

    dq_k is the change of the level-summed global-mean humidity from step k-1 to
    step k (zero for the first step, which has no predecessor here).  A decrease
    counts as precipitation (>= 0), an increase as evaporation, reported with the
    reference's sign convention (<= 0), so that precipitation + evaporation = -dq.
    The reference applies the clamps to the humidity itself rather than to its
    change; this function follows its documented meaning.
    """
    q = torch.stack([moisture_proxy(s, key) for s in trajectory])
    dq = torch.cat([torch.zeros_like(q[:1]), q[1:] - q[:-1]])
    return torch.clamp(-dq, min=0.0), torch.clamp(-dq, max=0.0)


def precipitation_rate_diagnostic(state: State, previous_state: State | None = None,
                                  key: str = "specific_humidity") -> torch.Tensor:
    """Precipitation-minus-evaporation proxy: minus the change of column humidity since
    ``previous_state`` (minus the humidity itself without one); zero without humidity."""
    if state.tracers.get(key) is None:
        return torch.zeros((), dtype=torch.float64, device=state.vorticity.device)
    now = moisture_proxy(state, key)
    return -(now - moisture_proxy(previous_state, key)) if previous_state is not None else -now


def heating_rate_diagnostic(state: State, previous_state: State | None = None) -> torch.Tensor:
    """Column heating proxy: the change of the level-summed global-mean temperature anomaly."""
    col = lambda s: s.temperature_variation[..., :, 0, 0].sum(dim=-1).to(torch.float64)  # noqa: E731
    return col(state) - col(previous_state) if previous_state is not None else col(state)


class CombinedStepDiagnostics:
    """Step diagnostics with the ``diagnostics_fn(model_state, physics_tendencies, forcing)`` signature:
    P-E and heating proxies against the model state's memory, energy and dry-air mass."""

    def __call__(self, model_state, physics_tendencies=None, forcing=None) -> dict:
        from tornado_gcm_b200.neural.fixers import compute_dry_air_mass, compute_total_energy

        state, prev = model_state.state, model_state.memory
        prev = prev if isinstance(prev, State) else None
        return {"P_minus_E_rate": precipitation_rate_diagnostic(state, prev),
                "heating_rate": heating_rate_diagnostic(state, prev),
                "total_energy": compute_total_energy(state),
                "dry_air_mass": compute_dry_air_mass(state)}
