"""NeuralGCM model API — reference ``model/api.py:54-1337``.

``NeuralGCMModel.step`` is one outer physics step:

1. neural tendency from the parameterization (Z3, BF16 on tcgen05);
2. ``dycore_substeps`` IMEX-SIL3 substeps of dycore + constant physics
   tendency, each followed by the dycore and stability spectral filters
   and the inner-state sanitiser (Z1);
3. conservation fix every ``fixer_cadence`` steps (Z2, FP64 accumulation).

On CUDA the substep runs through :class:`tornado_gcm_b200.ops.dycore.FusedSIL3`
(fused explicit-terms pipeline + one kernel for each SIL3 stage combine /
implicit solve / filters / sanitise); on CPU it runs the reference-semantics
torch steppers in :mod:`tornado_gcm_b200.core.time_integration`.

Differences from the reference by design: batch-first tensors; the zone
casts are explicit (no global autocast); the implicit inverse is cached on
device; ``VectorizedModel`` computes ``sim_time`` arithmetically instead of
re-running member 0.
"""

from __future__ import annotations

import dataclasses
import logging
from typing import Any, Callable, Optional

import numpy as np
import torch
import torch.nn as nn
import torch.utils.checkpoint as torch_checkpoint
from tornado_gcm_b200.utils.tracing import zone_range as record_function

from tornado_gcm_b200.core import coordinate_systems, filtering, primitive_equations, time_integration
from tornado_gcm_b200.precision.monitor import PrecisionMonitor
from tornado_gcm_b200.precision.policy import PrecisionPolicy, PrecisionZone
from tornado_gcm_b200.utils.typing import ModelState, RandomnessState

logger = logging.getLogger(__name__)
State = primitive_equations.State
ForcingFn = Callable[[dict, float], dict]


_EPD_MEMORY_FIELDS = frozenset(("vorticity", "divergence", "temperature_variation", "log_surface_pressure"))


def _physics_memory_ok_for_epd(memory, state: State) -> bool:
    """Whether ``memory`` supplies every ``memory_*`` feature the physics network was built with.

    A :class:`State` (or any object that is not a dict) is used as it is.  A dict
    qualifies when it holds the four core spectral fields and, for a state with
    tracers, a tracer dict covering all of them; an empty or partial dict (a
    forcing-only blob, say) would narrow the packed feature vector below the
    trained width, so the caller falls back to the current state.
    """
    if memory is None:
        return False
    if not isinstance(memory, dict):
        return True
    if not _EPD_MEMORY_FIELDS.issubset(memory):
        return False
    wanted = set(state.tracers or ())
    have = memory.get("tracers")
    return not wanted or (isinstance(have, dict) and wanted.issubset(have))


@dataclasses.dataclass
class ModelConfig:
    """Model configuration (field names/defaults as the reference ``ModelConfig``)."""

    coords: coordinate_systems.CoordinateSystem
    dt: float = 1.0
    inner_steps: int = 1
    dycore_substeps: int = 8
    physics_specs: Any = None
    reference_temperature: Optional[np.ndarray] = None
    orography: Optional[torch.Tensor] = None
    precision_policy: PrecisionPolicy = dataclasses.field(default_factory=PrecisionPolicy)
    filter_attenuation: float = 16.0
    filter_order: int = 18
    filter_cutoff: float = 0.0
    stability_filter_attenuation: Optional[float] = None
    stability_filter_order: int = 10
    stability_filter_cutoff: float = 0.4
    diffusion_tau: float = 0.01
    use_dycore: bool = True
    checkpoint_inner_steps: bool = False
    humidity_key: Optional[str] = "specific_humidity"
    cloud_keys: Optional[tuple] = None
    # hyperdiffusion step filter (order, tau in model time units); None = off
    hyperdiffusion_order: Optional[int] = None
    hyperdiffusion_tau: Optional[float] = None


class NeuralGCMModel(nn.Module):
    def __init__(self, config: ModelConfig, parameterization: nn.Module | None = None,
                 conservation_fixer: nn.Module | None = None, monitor: PrecisionMonitor | None = None,
                 forcing_fn: ForcingFn | None = None, encoder: nn.Module | None = None,
                 decoder: nn.Module | None = None, stochastic_step: nn.Module | None = None,
                 perturbation_fn: nn.Module | None = None, random_field: nn.Module | None = None,
                 diagnostics_fn: Callable | None = None):
        super().__init__()
        self.config = config
        self.parameterization = parameterization
        self.conservation_fixer = conservation_fixer
        self.monitor = monitor
        self.forcing_fn = forcing_fn
        self.encoder = encoder
        self.decoder = decoder
        self.stochastic_step = stochastic_step
        self.perturbation_fn = perturbation_fn
        self.random_field = random_field
        self.diagnostics_fn = diagnostics_fn
        self._fixer_cadence = 1
        self._step_count = 0
        self._sanitize_inner_enabled = True
        self._sanitize_inner_clamp_abs = 1.0e12
        self._nanoscope_ctx = None
        self._cached_diagnostics: dict = {}
        self._diagnostics_enabled = False
        self.policy = config.precision_policy
        # wavenumber/latitude sharding over ranks (parallel.spectral_shard.ShardContext)
        self.shard = None
        # run the packed (kernel-table) step on CPU tensors too (the kernels' CPU twins)
        self.packed_on_cpu = False

        grid = config.coords.horizontal
        self.exp_filter = filtering.exponential_filter(grid, config.filter_attenuation, config.filter_order,
                                                       config.filter_cutoff)
        self.stability_filter = None
        if config.stability_filter_attenuation is not None:
            self.stability_filter = filtering.exponential_filter(
                grid, config.stability_filter_attenuation, config.stability_filter_order,
                config.stability_filter_cutoff)
        self.hyperdiffusion_filter = None
        self._dycore_equation = None
        self._dycore = None
        self._fused = None
        if config.use_dycore and config.physics_specs is not None:
            ref_temp = config.reference_temperature
            if ref_temp is None:
                ref_temp = np.full(config.coords.vertical.layers, 250.0)
            oro = config.orography
            if oro is None:
                oro = torch.zeros(config.coords.modal_shape[1:], dtype=torch.float32)
            self._dycore = primitive_equations.PrimitiveEquationsSigma(
                ref_temp, oro, config.coords, config.physics_specs,
                humidity_key=config.humidity_key, cloud_keys=config.cloud_keys)
            self._dycore_equation = self._dycore
            self._inner_dt = config.dt / config.dycore_substeps
            if config.hyperdiffusion_order is not None and config.hyperdiffusion_tau is not None:
                eig = grid.laplacian_eigenvalues
                # negative: filtering.horizontal_diffusion_filter applies exp(scale · (-λ)^order), so
                # this damps the truncation wavenumber by exp(-dt / τ) per step (see
                # core.time_integration.horizontal_diffusion_step_filter for the reference's sign)
                scale = -self._inner_dt / (config.hyperdiffusion_tau * abs(eig[-1]) ** config.hyperdiffusion_order)
                self.hyperdiffusion_filter = filtering.horizontal_diffusion_filter(
                    grid, scale, config.hyperdiffusion_order)
        self.use_fused_dycore = True

    # ── runtime knobs ─────────────────────────────────────────────────
    @property
    def dycore(self):
        return self._dycore

    def set_precision_policy(self, policy: PrecisionPolicy) -> None:
        self.policy = policy

    def set_fixer(self, fixer: nn.Module | None) -> None:
        self.conservation_fixer = fixer

    def set_fixer_cadence(self, cadence: int) -> None:
        if cadence < 1:
            raise ValueError(f"fixer_cadence must be >= 1, got {cadence}")
        self._fixer_cadence = cadence

    def enable_diagnostics(self, enabled: bool = True) -> None:
        self._diagnostics_enabled = enabled
        if not enabled:
            self._cached_diagnostics.clear()

    def get_diagnostics(self) -> dict:
        d = dict(self._cached_diagnostics)
        self._cached_diagnostics.clear()
        return d

    def set_transform_precision(self, precision: str) -> None:
        """Switch the spherical-harmonic transforms of the step to ``precision``
        ("tf32" kernels, "float32", or "highest" = FP64 torch contractions).

        The dycore equation is rebuilt on the re-precisioned grid; the fused
        packed path (TF32 kernels) is used only for "tf32".
        """
        cfg = self.config
        grid = cfg.coords.horizontal.with_precision(precision)
        cfg.coords = dataclasses.replace(cfg.coords, horizontal=grid)
        if self._dycore is not None:
            old = self._dycore
            self._dycore = primitive_equations.PrimitiveEquationsSigma(
                old.reference_temperature, old.orography, cfg.coords, cfg.physics_specs,
                humidity_key=cfg.humidity_key, cloud_keys=cfg.cloud_keys)
            self._dycore_equation = self._dycore
        self._fused = None
        self.use_fused_dycore = precision == "tf32"
        if self.parameterization is not None and hasattr(self.parameterization, "grid"):
            self.parameterization.grid = grid

    def set_inner_state_safeguard(self, enabled: bool, clamp_abs: float = 1.0e12) -> None:
        self._sanitize_inner_enabled = bool(enabled)
        self._sanitize_inner_clamp_abs = float(clamp_abs)

    def attach_nanoscope(self, ctx: Any) -> None:
        self._nanoscope_ctx = ctx

    def detach_nanoscope(self) -> None:
        self._nanoscope_ctx = None

    # ── zones ─────────────────────────────────────────────────────────
    def _apply_parameterization(self, state: State, forcings=None, memory=None) -> State:
        if self.parameterization is None:
            return state.tree_map(torch.zeros_like)
        z1 = self.policy.compute_dtype(PrecisionZone.Z1_DYNAMICS_CORE)
        z3_mem = memory if _physics_memory_ok_for_epd(memory, state) else state
        tend = self.parameterization(state, forcings=forcings, memory=z3_mem)
        out = tend.tree_map(lambda t: t.to(z1))
        if self.monitor is not None:
            self.monitor.audit_zone_transfer("Z3_to_Z1", tend.vorticity, out.vorticity)
        return out

    def _packed_parameterization(self, state: State, y: torch.Tensor, keys: tuple, forcings, memory):
        """Physics tendency in the packed layout of ``y``.

        Parameterizations with a ``forward_packed`` method stay in the packed
        layout end to end; others run on the :class:`State` and are packed.
        """
        p = self.parameterization
        z1 = self.policy.compute_dtype(PrecisionZone.Z1_DYNAMICS_CORE)
        if p is not None and hasattr(p, "forward_packed") and self.monitor is None and y.ndim == 4:
            return p.forward_packed(y, keys, forcings).to(z1)
        from tornado_gcm_b200.ops import spectral

        return spectral.pack_state(self._apply_parameterization(state, forcings=forcings, memory=memory), keys)

    def _apply_conservation_fix(self, state: State, before: State) -> State:
        if self.conservation_fixer is None:
            return state
        if getattr(self.conservation_fixer, "bypass_upcast", False):
            fixed = self.conservation_fixer(state, before)
        else:
            z2 = self.policy.compute_dtype(PrecisionZone.Z2_CONSERVATION_FIXER)
            z1 = self.policy.compute_dtype(PrecisionZone.Z1_DYNAMICS_CORE)
            fixed = self.conservation_fixer(state.tree_map(lambda t: t.to(z2)),
                                            before.tree_map(lambda t: t.to(z2))).tree_map(lambda t: t.to(z1))
        if self._diagnostics_enabled:
            with torch.no_grad():
                self._cached_diagnostics["last_fixer"] = {
                    "vorticity_drift_max": (fixed.vorticity.double() - state.vorticity.double()).abs().max().item(),
                    "divergence_drift_max": (fixed.divergence.double() - state.divergence.double()).abs().max().item(),
                }
        return fixed

    def _filter_state(self, state: State) -> State:
        return state.tree_map(self.exp_filter)

    def _sanitize_inner_state(self, state: State) -> State:
        if not self._sanitize_inner_enabled:
            return state
        c = self._sanitize_inner_clamp_abs

        def fix(t):
            if not torch.is_floating_point(t):
                return t
            return torch.clamp(torch.nan_to_num(t, nan=0.0, posinf=c, neginf=-c), -c, c)
        return state.tree_map(fix)

    def combined_filter_scaling(self) -> np.ndarray:
        """Product of all per-substep spectral filters as one l-vector."""
        s = self.exp_filter.scaling.copy()
        if self.stability_filter is not None:
            s = s * self.stability_filter.scaling
        if self.hyperdiffusion_filter is not None:
            s = s * self.hyperdiffusion_filter.scaling
        return s

    # ── inner step ────────────────────────────────────────────────────
    def _fused_stepper(self, tracer_keys):
        if self._fused is None:
            self._fused = {}
        st = self._fused.get(tracer_keys)
        if st is None:
            from tornado_gcm_b200.ops import dycore as dycore_ops

            st = dycore_ops.PackedSIL3(self._dycore, self._inner_dt, self.combined_filter_scaling(), tracer_keys,
                                       clamp_abs=self._sanitize_inner_clamp_abs if self._sanitize_inner_enabled
                                       else float("inf"),
                                       grid=self.shard.grid if self.shard is not None else None)
            self._fused[tracer_keys] = st
        return st

    def _build_inner_step_fn(self, physics_tendency: State):
        eq = self._dycore
        phys = physics_tendency

        class _Combined(time_integration.ImplicitExplicitODE):
            def explicit_terms(self_, x):
                return time_integration.tree_add(eq.explicit_terms(x), phys)

            def implicit_terms(self_, x):
                return eq.implicit_terms(x)

            def implicit_inverse(self_, x, s):
                return eq.implicit_inverse(x, s)

        step_hook = None
        if self._nanoscope_ctx is not None:
            ctx = self._nanoscope_ctx

            def step_hook(i, y):
                try:
                    ctx.snapshot_manager.push_state(step=self._step_count, t=i * self._inner_dt, y=y)
                except Exception as exc:  # pragma: no cover - optional integration
                    logger.debug("nanoscope push failed: %s", exc)
        raw = time_integration.imex_rk_sil3(_Combined(), self._inner_dt, step_hook=step_hook)
        filters = [time_integration.runge_kutta_step_filter(lambda s: s.tree_map(self.exp_filter))]
        if self.stability_filter is not None:
            filters.append(time_integration.runge_kutta_step_filter(lambda s: s.tree_map(self.stability_filter)))
        if self.hyperdiffusion_filter is not None:
            filters.append(time_integration.runge_kutta_step_filter(lambda s: s.tree_map(self.hyperdiffusion_filter)))
        return time_integration.step_with_filters(raw, filters)

    def _use_fused(self, state: State) -> bool:
        if self.shard is not None:
            return True  # the sharded model exists only as the packed step
        return ((state.vorticity.is_cuda or self.packed_on_cpu) and self.use_fused_dycore
                and self._nanoscope_ctx is None and getattr(self._dycore, "use_fused", True))

    # ── outer step ────────────────────────────────────────────────────
    def step(self, state: State, forcings: dict | None = None, memory=None) -> State:
        before = state
        if self.forcing_fn is not None and forcings is not None:
            forcings = self.forcing_fn(forcings, state.sim_time if state.sim_time is not None else 0.0)
        fused = self._dycore is not None and self._use_fused(state)
        fixed_in_packed = False
        if fused:
            from tornado_gcm_b200.ops import spectral

            keys = tuple(sorted(state.tracers))
            stepper = self._fused_stepper(keys)
            y = spectral.pack_state(state, keys)
            y_start = y
            with record_function("Z3_neural_net"):
                P = self._packed_parameterization(state, y, keys, forcings, memory)
        else:
            with record_function("Z3_neural_net"):
                phys = self._apply_parameterization(state, forcings=forcings, memory=memory)
        if self._dycore is not None:
            with record_function("Z1_dycore"):
                if fused:
                    P = P + stepper.orography_packed(y.device)
                    for _ in range(self.config.dycore_substeps):
                        if self.config.checkpoint_inner_steps and self.training:
                            y = torch_checkpoint.checkpoint(stepper.step_packed, y, P, use_reentrant=False)
                        else:
                            y = stepper.step_packed(y, P)
                    self._step_count += 1
                    fixer = self.conservation_fixer
                    if (self._step_count % self._fixer_cadence == 0 and fixer is not None
                            and hasattr(fixer, "forward_packed") and not self._diagnostics_enabled):
                        with record_function("Z2_physics_bridge"):
                            n_lev = self.config.coords.vertical.layers
                            if self.shard is not None:
                                from tornado_gcm_b200.parallel.spectral_shard import sharded_packed_fix

                                y = sharded_packed_fix(y, y_start, n_lev, self.shard.group, fixer.fix_mass,
                                                       fixer.fix_energy, fixer.energy_split)
                            else:
                                y = fixer.forward_packed(y, y_start, n_lev)
                        fixed_in_packed = True
                    elif (self.shard is not None and fixer is not None
                          and self._step_count % self._fixer_cadence == 0):
                        raise NotImplementedError("a sharded model step needs a fixer with a packed form "
                                                  "(LiteConservationFixer)")
                    state = spectral.unpack_state(y, self.config.coords.vertical.layers, keys, state.sim_time)
                else:
                    inner = self._build_inner_step_fn(phys)
                    for _ in range(self.config.dycore_substeps):
                        if self.config.checkpoint_inner_steps and self.training:
                            state = torch_checkpoint.checkpoint(inner, state, use_reentrant=False)
                        else:
                            state = inner(state)
                        state = self._sanitize_inner_state(state)
        else:
            with record_function("Z1_dycore"):
                state = state + self.config.dt * phys
            with record_function("Z0_spectral"):
                state = self._filter_state(state)
        if not fused:
            self._step_count += 1
        if self._step_count % self._fixer_cadence == 0 and not fixed_in_packed:
            with record_function("Z2_physics_bridge"):
                state = self._apply_conservation_fix(state, before)
        if state.sim_time is not None:
            from tornado_gcm_b200.ops.spectral import carry_packed

            state = carry_packed(state, dataclasses.replace(state, sim_time=state.sim_time + self.config.dt))
        if self.monitor is not None:
            self.monitor.step()
        return state

    def step_model_state(self, model_state: ModelState, forcings: dict | None = None) -> ModelState:
        if isinstance(model_state, State):
            model_state = ModelState(state=model_state)
        state, memory = model_state.state, model_state.memory
        diagnostics, randomness = model_state.diagnostics, model_state.randomness
        nxt = self.step(state, forcings=forcings, memory=memory)
        nrand = randomness
        if self.stochastic_step is not None:
            rin = randomness if randomness.core is not None else None
            nxt, rraw = self.stochastic_step(nxt, forcing=forcings, randomness=rin)
            if rraw is not None:
                nrand = rraw
        elif self.random_field is not None and randomness.core is not None:
            nrand = self.random_field.advance(randomness)
        nmem = state.tree_map(torch.clone) if memory is not None else None
        ndiag = {}
        if self.diagnostics_fn is not None:
            ndiag = self.diagnostics_fn(ModelState(nxt, nmem, diagnostics, nrand), physics_tendencies=None,
                                        forcing=forcings)
        elif isinstance(diagnostics, dict):
            ndiag = diagnostics
        return ModelState(state=nxt, memory=nmem, diagnostics=ndiag, randomness=nrand)

    def initialize_model_state(self, state: State, with_memory: bool = True, device=None,
                               dtype: torch.dtype = torch.float32) -> ModelState:
        memory = state.tree_map(torch.clone) if with_memory else None
        randomness = RandomnessState()
        if self.random_field is not None:
            r = self.random_field.unconditional_sample(device=device or state.vorticity.device, dtype=dtype)
            randomness = RandomnessState(core=r.core, nodal_value=r.nodal_value)
        return ModelState(state=state, memory=memory, diagnostics={}, randomness=randomness)

    def _advance(self, s, forcings):
        return self.step_model_state(s, forcings) if isinstance(s, ModelState) else self.step(s, forcings)

    def forward(self, initial_state, outer_steps: int, inner_steps: int | None = None, forcings=None,
                post_process_fn=None, checkpoint_outer_steps: bool = False):
        inner_steps = self.config.inner_steps if inner_steps is None else inner_steps
        self.policy.apply_tf32_setting()
        cur = initial_state
        traj = []

        def block(s):
            for _ in range(inner_steps):
                s = self._advance(s, forcings)
            return s

        for _ in range(outer_steps):
            if checkpoint_outer_steps and self.training:
                cur = torch_checkpoint.checkpoint(block, cur, use_reentrant=False)
            else:
                cur = block(cur)
            s = cur.state if isinstance(cur, ModelState) else cur
            traj.append(post_process_fn(s) if post_process_fn is not None else s)
        return cur, traj

    @torch.no_grad()
    def forward_streaming(self, initial_state, outer_steps: int, inner_steps: int | None = None, forcings=None,
                          post_process_fn=None):
        inner_steps = self.config.inner_steps if inner_steps is None else inner_steps
        self.policy.apply_tf32_setting()
        cur = initial_state
        for _ in range(outer_steps):
            for _ in range(inner_steps):
                cur = self._advance(cur, forcings)
            s = cur.state if isinstance(cur, ModelState) else cur
            yield post_process_fn(s) if post_process_fn is not None else s
        return cur

    @torch.no_grad()
    def forward_chunked(self, initial_state, chunk_size: int, inner_steps: int | None = None, forcings=None,
                        post_process_fn=None):
        return self.forward(initial_state, chunk_size, inner_steps, forcings=forcings,
                            post_process_fn=post_process_fn)

    def forward_nested(self, initial_state, forcings: list, frequencies: dict, dt=1, collect_every: int = 1,
                       checkpoint_level: int = -1, post_process_fn=None):
        from tornado_gcm_b200.core.scan_utils import nested_rollout

        self.policy.apply_tf32_setting()
        final, raw = nested_rollout(step_fn=lambda s, f: self._advance(s, f), initial_state=initial_state,
                                    forcings=forcings, frequencies=frequencies, dt=dt,
                                    checkpoint_level=checkpoint_level, collect_every=collect_every)
        ext = lambda s: s.state if isinstance(s, ModelState) else s
        traj = [post_process_fn(ext(s)) for s in raw] if post_process_fn is not None else raw
        return final, traj

    # ── encode / decode ───────────────────────────────────────────────
    def encode(self, inputs, forcings=None):
        if self.encoder is None:
            raise ValueError("model has no encoder")
        return self.encoder(inputs, forcings) if forcings is not None else self.encoder(inputs)

    def decode(self, state, forcings=None):
        if self.decoder is None:
            raise ValueError("model has no decoder")
        return self.decoder(state, forcings) if forcings is not None else self.decoder(state)


class InferenceModel(nn.Module):
    """Assimilate → rollout → observe wrapper (reference ``model/api.py:1005-1133``).

    ``forward`` rolls a model-space state (or :class:`ModelState`) forward and returns
    the trajectory through ``post_process_fn``; :meth:`assimilate` maps raw inputs into
    model space (optionally blended into an existing state); :meth:`observe` decodes.
    """

    def __init__(self, model: NeuralGCMModel, post_process_fn: Callable | None = None):
        super().__init__()
        self.model = model
        self.post_process_fn = post_process_fn

    def assimilate(self, inputs, forcings=None, state: State | None = None, alpha: float = 1.0,
                   return_model_state: bool = False):
        """Encode ``inputs`` (or take them as a model-space :class:`State` when the model has no
        encoder); with ``state``, return ``(1 - alpha) state + alpha encoded``."""
        if self.model.encoder is not None:
            encoded = self.model.encode(inputs, forcings)
        elif isinstance(inputs, State):
            encoded = inputs
        else:
            raise ValueError("the model has no encoder: pass a model-space State as inputs")
        out = encoded if (state is None or alpha >= 1.0) else state * (1.0 - alpha) + encoded * alpha
        return self.model.initialize_model_state(out) if return_model_state else out

    def observe(self, state, forcings=None):
        """Decoded fields of ``state``; the state itself when the model has no decoder."""
        return self.model.decode(state, forcings) if self.model.decoder is not None else state

    @torch.no_grad()
    def forward(self, initial_state, outer_steps: int, inner_steps: int | None = None, forcings=None) -> list:
        self.model.eval()
        _, traj = self.model.forward(initial_state, outer_steps, inner_steps, forcings=forcings,
                                     post_process_fn=self.post_process_fn)
        return traj


class VectorizedModel(nn.Module):
    """Ensemble wrapper: members as a leading batch dimension (or a loop)."""

    def __init__(self, model: NeuralGCMModel, mode: str | None = None, use_vmap: bool = True):
        """``mode``: ``batch`` (members as the leading dimension of every kernel) or ``loop``
        (one member at a time); without it ``use_vmap`` (the reference's switch) picks batch."""
        super().__init__()
        mode = mode if mode is not None else ("batch" if use_vmap else "loop")
        if mode not in ("batch", "loop", "vmap"):
            raise ValueError(f"unknown mode {mode}")
        self.model = model
        self.mode = "batch" if mode == "vmap" else mode

    def step(self, states: State, forcings=None) -> State:
        if self.mode == "batch":
            return self.model.step(states, forcings)
        n = states.vorticity.shape[0]
        outs = [self.model.step(states.tree_map(lambda t: t[i]), forcings) for i in range(n)]
        stacked = State(*(torch.stack([getattr(o, f) for o in outs]) for f in
                          ("vorticity", "divergence", "temperature_variation", "log_surface_pressure")),
                        {k: torch.stack([o.tracers[k] for o in outs]) for k in outs[0].tracers},
                        None if states.sim_time is None else states.sim_time + self.model.config.dt)
        return stacked

    def forward(self, initial_states: State, outer_steps: int, inner_steps: int | None = None, forcings=None,
                post_process_fn=None):
        inner_steps = self.model.config.inner_steps if inner_steps is None else inner_steps
        cur, traj = initial_states, []
        for _ in range(outer_steps):
            for _ in range(inner_steps):
                cur = self.step(cur, forcings)
            traj.append(post_process_fn(cur) if post_process_fn is not None else cur)
        return cur, traj
