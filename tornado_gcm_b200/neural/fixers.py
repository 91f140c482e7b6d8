"""Z2 conservation fixers (reference ``neural/fixers.py:25-326``).

Mass fixer: restore the (0,0) mode of log surface pressure.  Energy fixer:
absorb the deficit of the energy proxy Σζ²+δ²+T'² into the (0,0) mode of
T' on every level, ``Δ_k = −T_k + sign(T_k)·sqrt(T_k² + deficit)``.

Batch semantics: with leading batch dims the proxies are per sample
(summed over level, m, l), and the "skip if any discriminant ≤ 0" rule is
applied per sample with a mask instead of a host-synchronising branch.
On CUDA the reductions run in the FP64 fixer kernel of
:mod:`tornado_gcm_b200.ops.fixers` (one pass over the state, FP64
accumulation, corrections applied in the same launch).
"""

from __future__ import annotations

import torch
import torch.nn as nn

from tornado_gcm_b200.core import primitive_equations
from tornado_gcm_b200.precision.zone_cast import f64_math

State = primitive_equations.State


class KahanAccumulator:
    """Compensated (Kahan) FP64 summation."""

    def __init__(self):
        self.sum = None
        self.compensation = None

    def add(self, x: torch.Tensor) -> None:
        x = x.to(torch.float64)
        if self.sum is None:
            self.sum = x.clone()
            self.compensation = torch.zeros_like(self.sum)
            return
        y = x - self.compensation
        t = self.sum + y
        self.compensation = (t - self.sum) - y
        self.sum = t

    def reset(self) -> None:
        self.sum = None
        self.compensation = None


def kahan_sum(tensors, dim=None) -> torch.Tensor:
    acc = KahanAccumulator()
    for t in tensors:
        acc.add(t.sum(dim=dim) if dim is not None else t)
    return acc.sum


@f64_math
def _global_mean_modal(x: torch.Tensor) -> torch.Tensor:
    return x[..., 0, 0]


def compute_dry_air_mass(state: State) -> torch.Tensor:
    return _global_mean_modal(state.log_surface_pressure)


def _energy_proxy(state: State, accumulate_dtype=None) -> torch.Tensor:
    dims = (-3, -2, -1)
    kw = {} if accumulate_dtype is None else {"dtype": accumulate_dtype}
    ke = (state.vorticity ** 2 + state.divergence ** 2).sum(dim=dims, **kw)
    te = (state.temperature_variation ** 2).sum(dim=dims, **kw)
    return ke + te


def compute_total_energy(state: State) -> torch.Tensor:
    """Per-sample energy proxy in the input dtype."""
    return _energy_proxy(state)


def compute_total_energy_lite(state: State) -> torch.Tensor:
    """Per-sample energy proxy: input-precision squares, FP64 accumulation."""
    return _energy_proxy(state, torch.float64)


def _mass_fix(state: State, before: State) -> State:
    lsp = state.log_surface_pressure
    drift = lsp[..., 0, 0].to(torch.float64) - before.log_surface_pressure[..., 0, 0].to(torch.float64)
    new = lsp.clone()
    new[..., 0, 0] = lsp[..., 0, 0] - drift.to(lsp.dtype)
    return State(state.vorticity, state.divergence, state.temperature_variation, new, state.tracers, state.sim_time)


def _energy_fix(state: State, deficit: torch.Tensor, energy_split: str = "levels") -> State:
    """Restore the energy proxy through the T'(0,0) mode of every level.

    ``energy_split="levels"`` adds deficit / n to each level's T'(0,0)² (the
    proxy is then restored exactly).  ``"reference"`` is the formula of
    reference ``neural/fixers.py:171-190`` / ``:309-321``, which adds the whole
    deficit at every level, i.e. n times the deficit in total: with strong
    dissipation the global-mean temperature modes then grow until the state
    fails (1.4°, 32 levels: after about 21 simulated hours).
    """
    t = state.temperature_variation
    t00 = t[..., 0, 0].to(torch.float64)  # (..., levels)
    share = deficit / t00.shape[-1] if energy_split == "levels" else deficit
    disc = t00 * t00 + share.unsqueeze(-1)
    ok = (disc > 0).all(dim=-1, keepdim=True)
    delta = -t00 + torch.sign(t00) * torch.sqrt(torch.clamp(disc, min=0.0))
    delta = torch.where(ok, delta, torch.zeros_like(delta))
    new = t.clone()
    new[..., 0, 0] = t[..., 0, 0] + delta.to(t.dtype)
    return State(state.vorticity, state.divergence, new, state.log_surface_pressure, state.tracers, state.sim_time)


class GlobalDryAirMassFixer(nn.Module):
    def forward(self, state: State, state_before: State) -> State:
        return _mass_fix(state, state_before)


class GlobalEnergyFixer(nn.Module):
    def __init__(self, energy_split: str = "levels"):
        super().__init__()
        self.energy_split = energy_split

    def forward(self, state: State, state_before: State) -> State:
        deficit = compute_total_energy(state_before).to(torch.float64) - compute_total_energy(state).to(torch.float64)
        return _energy_fix(state, deficit, self.energy_split)


class F64ConservationFixer(nn.Module):
    """Mass then energy fix; the caller casts the state to the Z2 dtype first."""

    def __init__(self, fix_mass: bool = True, fix_energy: bool = True, dtype: torch.dtype = torch.float64,
                 energy_split: str = "levels"):
        super().__init__()
        self.dtype = dtype
        self.mass_fixer = GlobalDryAirMassFixer() if fix_mass else None
        self.energy_fixer = GlobalEnergyFixer(energy_split) if fix_energy else None

    def forward(self, state: State, state_before: State) -> State:
        if self.mass_fixer is not None:
            state = self.mass_fixer(state, state_before)
        if self.energy_fixer is not None:
            state = self.energy_fixer(state, state_before)
        return state


class LiteConservationFixer(nn.Module):
    """Z2-Lite: FP32 state, FP64 accumulation only (no full-state upcast).

    On CUDA this is one fused kernel (:func:`tornado_gcm_b200.ops.fixers.lite_fix`).
    """

    def __init__(self, fix_mass: bool = True, fix_energy: bool = True, energy_split: str = "levels"):
        super().__init__()
        self.fix_mass = fix_mass
        self.fix_energy = fix_energy
        self.energy_split = energy_split  # "levels" (exact) or "reference" (see _energy_fix)

    @property
    def bypass_upcast(self) -> bool:
        return True

    def forward_packed(self, y: torch.Tensor, y_before: torch.Tensor, n: int) -> torch.Tensor:
        """Fix a packed ``[ζ | δ | T' | ln ps | …]`` state (differentiable kernel pair)."""
        from tornado_gcm_b200.ops import fixers as fixer_ops

        return fixer_ops.packed_fix(y, y_before, n, self.fix_mass, self.fix_energy, self.energy_split)

    def forward(self, state: State, state_before: State) -> State:
        if state.vorticity.is_cuda:
            from tornado_gcm_b200.ops import fixers as fixer_ops

            return fixer_ops.lite_fix(state, state_before, self.fix_mass, self.fix_energy, self.energy_split)
        if self.fix_mass:
            state = _mass_fix(state, state_before)
        if self.fix_energy:
            deficit = compute_total_energy_lite(state_before) - compute_total_energy_lite(state)
            state = _energy_fix(state, deficit, self.energy_split)
        return state
