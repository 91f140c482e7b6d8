"""Stochastic components — reference ``neural/stochastic.py:30-307``.

* :class:`GaussianRandomField` — AR(1) process in spherical-harmonic space,
  ``U(t+1) = φ U(t) + sqrt(1-φ²) σ_l η`` (stationary variance σ_l²) with ``φ = exp(-1/τ)`` and
  ``σ_l ∝ exp(-κ l(l+1)/2)``, ``κ = (correlation_length / radius)²``.  The
  coefficients live on the grid's modal layout ``(…, 2M-1, L)`` with the
  triangular mask applied (the reference draws an ``(L, L)`` core, which is
  not its own modal shape); σ is normalised so the area-mean nodal variance
  equals ``variance``.
* :class:`NoRandomField`, :class:`ZerosRandomField` — ablation variants.
* :class:`Corrector` — forward-Euler step with non-negative humidity.
* :class:`Perturbation` — tendency perturbation.  ``mode="multiplicative"``
  scales the whole tendency by ``1 + ε·mean(noise)`` (the reference's
  behaviour, kept as the default for parity); ``mode="sppt"`` multiplies the
  nodal tendency field-wise by ``1 + ε·noise`` (stochastically perturbed
  parameterisation tendencies); ``mode="additive"`` adds ``ε·mean(noise)`` to
  the temperature tendency as in the reference.
"""

from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch
import torch.nn as nn

from tornado_gcm_b200.core import primitive_equations as pe
from tornado_gcm_b200.utils.typing import RandomnessState

EARTH_RADIUS_M = 6.37122e6


class GaussianRandomField(nn.Module):
    def __init__(self, grid, correlation_time: float = 1.0, correlation_length: float = 1.0,
                 variance: Optional[float] = 1.0, clip: float = 6.0,
                 correlation_length_km: Optional[float] = None):
        super().__init__()
        self.grid = grid
        self.correlation_time = float(correlation_time)
        if correlation_length_km is not None:  # km → model length units (radius = 1)
            correlation_length = correlation_length_km * 1e3 / EARTH_RADIUS_M * grid.radius
        self.correlation_length = float(correlation_length)
        self.variance = variance
        self.clip = float(clip)
        self._phi = math.exp(-1.0 / max(self.correlation_time, 1e-12))
        M2, L = grid.modal_shape
        l = np.arange(L, dtype=np.float64)
        kappa = (self.correlation_length / grid.radius) ** 2 if grid.radius > 0 else 0.0
        sig = np.exp(-kappa * l * (l + 1) / 2.0)
        mask = np.asarray(grid.mask, dtype=np.float64)
        if variance is None:
            sig = sig * 0.0
        else:
            # area-mean nodal variance of Σ a_ml Y_ml with a_ml ~ N(0, σ_l²)
            sh = grid.spherical_harmonics
            p = np.asarray(sh.legendre_table)                  # (Mw, J, L)
            f = np.asarray(sh.basis.f)                         # (I, M2)
            w = np.asarray(sh.basis.w)                         # (J,)
            mrow = (np.arange(M2) + 1) // 2
            y2 = np.einsum("ir,rjl->rjl", f ** 2, p[mrow] ** 2)  # Σ_i F² P² (summed over longitude)
            per_l = np.einsum("rjl,j,rl->l", y2, w, mask) / (4.0 * math.pi)
            mean_var = float(np.sum(per_l * sig ** 2))
            if mean_var > 0:
                sig = sig * math.sqrt(float(variance) / mean_var)
        self.register_buffer("_sigma", torch.tensor(sig[None, :] * mask, dtype=torch.float32), persistent=False)

    def _noise(self, lead, generator, device, dtype):
        shape = tuple(lead) + tuple(self.grid.modal_shape)
        eta = torch.randn(shape, generator=generator, device=device, dtype=torch.float32)
        return torch.clamp(eta, -self.clip, self.clip).to(dtype)

    def sample_modal(self, lead=(), generator: Optional[torch.Generator] = None, device=None,
                     dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """One stationary draw of the modal coefficients with leading shape ``lead``."""
        device = device or self._sigma.device
        # the innovation of `advance` is σ·sqrt(1-φ²), so σ² is the stationary variance
        return self._sigma.to(device, dtype) * self._noise(lead, generator, device, dtype)

    def unconditional_sample(self, device=torch.device("cpu"), dtype: torch.dtype = torch.float32,
                             generator: Optional[torch.Generator] = None, lead=()) -> RandomnessState:
        core = self.sample_modal(lead, generator, device, dtype)
        return RandomnessState(core=core, nodal_value=self.grid.to_nodal(core), modal_value=core,
                               prng_step=0)

    def advance(self, state: RandomnessState, generator: Optional[torch.Generator] = None) -> RandomnessState:
        core = state.core
        sigma = self._sigma.to(core.device, core.dtype) * math.sqrt(max(1.0 - self._phi ** 2, 0.0))
        nxt = self._phi * core + sigma * self._noise(core.shape[:-2], generator, core.device, core.dtype)
        return RandomnessState(core=nxt, nodal_value=self.grid.to_nodal(nxt), modal_value=nxt,
                               prng_step=(state.prng_step or 0) + 1)


class NoRandomField(nn.Module):
    def __init__(self, grid=None, **kwargs):
        super().__init__()

    def unconditional_sample(self, **kwargs) -> RandomnessState:
        return RandomnessState(prng_step=0)

    def advance(self, state: RandomnessState, **kwargs) -> RandomnessState:
        return RandomnessState(prng_step=(state.prng_step or 0) + 1)


class ZerosRandomField(nn.Module):
    def __init__(self, grid, prefer_nodal: bool = True, **kwargs):
        super().__init__()
        self.grid = grid
        self._prefer_nodal = prefer_nodal

    def unconditional_sample(self, device=torch.device("cpu"), dtype=torch.float32, **kwargs) -> RandomnessState:
        core_shape = self.grid.nodal_shape if self._prefer_nodal else self.grid.modal_shape
        return RandomnessState(core=torch.zeros(core_shape, dtype=dtype, device=device),
                               nodal_value=torch.zeros(self.grid.nodal_shape, dtype=dtype, device=device),
                               prng_step=0)

    def advance(self, state: RandomnessState, **kwargs) -> RandomnessState:
        return RandomnessState(core=None if state.core is None else torch.zeros_like(state.core),
                               nodal_value=None if state.nodal_value is None else torch.zeros_like(state.nodal_value),
                               prng_step=(state.prng_step or 0) + 1)


class Corrector(nn.Module):
    def __init__(self, dt: float, humidity_key: str = "specific_humidity"):
        super().__init__()
        self.dt = dt
        self.humidity_key = humidity_key

    def forward(self, state: pe.State, tendency: pe.State, forcing=None) -> pe.State:
        nxt = state + self.dt * tendency
        if self.humidity_key in nxt.tracers:
            tr = dict(nxt.tracers)
            tr[self.humidity_key] = torch.clamp(tr[self.humidity_key], min=0.0)
            nxt = pe.State(nxt.vorticity, nxt.divergence, nxt.temperature_variation, nxt.log_surface_pressure,
                           tr, nxt.sim_time)
        return nxt


class Perturbation(nn.Module):
    def __init__(self, mode: str = "multiplicative", epsilon: float = 1.0, grid=None):
        super().__init__()
        if mode not in ("multiplicative", "additive", "sppt"):
            raise ValueError(f"unknown perturbation mode {mode!r}")
        if mode == "sppt" and grid is None:
            raise ValueError("sppt perturbations need the grid")
        self.mode = mode
        self.epsilon = epsilon
        self.grid = grid

    def forward(self, tendency: pe.State, randomness: Optional[RandomnessState] = None) -> pe.State:
        if randomness is None or randomness.nodal_value is None:
            return tendency
        noise = randomness.nodal_value
        if self.mode == "multiplicative":
            return tendency * (1.0 + self.epsilon * noise.mean())
        if self.mode == "additive":
            return pe.State(tendency.vorticity, tendency.divergence,
                            tendency.temperature_variation + self.epsilon * noise.mean(),
                            tendency.log_surface_pressure, tendency.tracers, tendency.sim_time)
        g = self.grid
        fac = 1.0 + self.epsilon * noise
        f = lambda t: g.to_modal(g.to_nodal(t) * fac)
        return tendency.tree_map(f)


class StochasticPhysicsParameterizationStep(nn.Module):
    """Sub-stepped stochastic physics — reference ``neural/stochastic.py:314-391``.

    Each of ``num_substeps``: tendency of ``physics_parameterization``,
    perturbed by ``perturbation`` with the current random field, a
    :class:`Corrector` Euler step, then the AR(1) random field advances.
    """

    def __init__(self, physics_parameterization: nn.Module, corrector: Corrector,
                 random_field: Optional[GaussianRandomField] = None, perturbation: Optional[Perturbation] = None,
                 num_substeps: int = 1):
        super().__init__()
        self.physics_param = physics_parameterization
        self.corrector = corrector
        self.random_field = random_field
        self.perturbation = perturbation
        self.num_substeps = int(num_substeps)

    def forward(self, state: pe.State, forcing=None, randomness: Optional[RandomnessState] = None,
                generator: Optional[torch.Generator] = None):
        rand = randomness
        for _ in range(self.num_substeps):
            tend = self.physics_param(state)
            if self.perturbation is not None and rand is not None:
                tend = self.perturbation(tend, rand)
            state = self.corrector(state, tend, forcing)
            if self.random_field is not None and rand is not None:
                rand = self.random_field.advance(rand, generator=generator)
        return state, rand

    def initialize_randomness(self, device=torch.device("cpu"), dtype: torch.dtype = torch.float32,
                              generator: Optional[torch.Generator] = None) -> Optional[RandomnessState]:
        if self.random_field is None:
            return None
        return self.random_field.unconditional_sample(device=device, dtype=dtype, generator=generator)
