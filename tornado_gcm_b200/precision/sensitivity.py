"""Hierarchical precision sensitivity (HPS level 1) — reference ``precision/sensitivity.py:74-902``.

:class:`SensitivityProfiler` measures how much a rollout's physics metrics
(by default the conservation proxies, accumulated in FP64) drift when one
module — or one precision zone — is run at a lower precision:

* ``run_coarse``: every top-level child module in turn;
* ``run_refine``: the children of modules whose drift exceeds a threshold;
* ``run_hierarchical``: both;
* ``profile_module_multi_dtype``: one module at several dtypes (the precision
  curve);
* ``run_zone_perturbation``: an all-FP64 baseline, then one PZHA zone
  lowered at a time through the model's :class:`PrecisionPolicy`.

Two ways to lower a module's precision:

* ``mode="emulate"`` (default): parameters and buffers are rounded through
  the test dtype and kept in their storage dtype (``p ← p.to(bf16).to(p.dtype)``).
  The forward code is unchanged, so the drift measures the information lost
  to the narrower format, not dtype-plumbing failures.
* ``mode="cast"``: parameters are cast to the test dtype as in the reference;
  a forward that cannot run in that dtype counts as infinitely sensitive.

Drift per metric is ``|m_test - m_base| / (|m_base| + 1e-30)``; the module's
drift is the largest finite one.  Recommendations: ``critical`` (> 0.1, FP64),
``moderate`` (> 1e-3, FP32/TF32), ``tolerant`` (BF16), ``invalid_baseline``
(non-finite).
"""

from __future__ import annotations

import dataclasses
import logging
import math
import time
from typing import Callable, Optional, Protocol

import torch
import torch.nn as nn

from tornado_gcm_b200.core.primitive_equations import State
from tornado_gcm_b200.precision.policy import PrecisionPolicy, PrecisionZone

logger = logging.getLogger(__name__)

ValidatorFn = Callable[[State], dict]


class PhysicsValidator(Protocol):
    def __call__(self, state: State) -> dict: ...


def default_conservation_validator(state: State) -> dict:
    """Energy proxy ``Σζ² + Σδ²`` and mass proxy ``Σ ln ps`` (FP64 sums)."""
    with torch.no_grad():
        vor = state.vorticity.detach().double()
        div = state.divergence.detach().double()
        return {"energy_proxy": float((vor * vor).sum() + (div * div).sum()),
                "mass_proxy": float(state.log_surface_pressure.detach().double().sum())}


def _finite(v) -> bool:
    try:
        return math.isfinite(float(v))
    except (TypeError, ValueError):
        return False


def _hps_baseline_metrics_usable(metrics: dict) -> bool:
    return any(_finite(v) for v in metrics.values())


@dataclasses.dataclass
class ModuleSensitivity:
    module_name: str
    drift: float
    metric_drifts: dict = dataclasses.field(default_factory=dict)
    test_dtype: torch.dtype = torch.bfloat16
    elapsed_s: float = 0.0
    n_children_profiled: int = 0


@dataclasses.dataclass
class SensitivityMap:
    modules: dict = dataclasses.field(default_factory=dict)
    baseline_metrics: dict = dataclasses.field(default_factory=dict)
    n_steps: int = 0
    refine_threshold: float = 0.0
    total_elapsed_s: float = 0.0

    @property
    def sensitivity_ranking(self) -> list:
        def key(item):
            d = item[1]
            if not _finite(d):
                return (1, 0.0)
            return (0, -float(d))

        return sorted(((n, ms.drift) for n, ms in self.modules.items()), key=key)

    def get_zone_recommendation(self) -> dict:
        rec = {}
        for name, ms in self.modules.items():
            d = ms.drift
            if not _finite(d):
                rec[name] = "invalid_baseline"
            elif d > 0.1:
                rec[name] = "critical"
            elif d > 1e-3:
                rec[name] = "moderate"
            else:
                rec[name] = "tolerant"
        return rec

    def summary_str(self) -> str:
        rec = self.get_zone_recommendation()
        lines = [f"SensitivityMap: {len(self.modules)} modules, {self.n_steps} steps, "
                 f"{self.total_elapsed_s:.1f}s total", f"Baseline metrics: {self.baseline_metrics}", "",
                 "Ranking (highest sensitivity first):"]
        for i, (name, drift) in enumerate(self.sensitivity_ranking, 1):
            ms = self.modules[name]
            kids = f" ({ms.n_children_profiled} sub-modules)" if ms.n_children_profiled else ""
            lines.append(f"  {i}. {name}: drift={float(drift):.6e} [{rec[name]}]{kids}")
        return "\n".join(lines)


class SensitivityProfiler:
    _ZONE_TARGETS = [
        ("Z1_dynamics", ("z1_compute_dtype", "z1_storage_dtype"), False),
        ("Z2_fixer", ("z2_compute_dtype", "z2_storage_dtype"), False),
        ("Z3_neural", ("z3_compute_dtype", "z3_param_dtype"), True),
    ]

    def __init__(self, model: nn.Module, baseline_policy: Optional[PrecisionPolicy] = None,
                 validator: Optional[ValidatorFn] = None, step_fn: Optional[Callable] = None, device=None,
                 mode: str = "emulate"):
        if mode not in ("emulate", "cast"):
            raise ValueError("mode must be 'emulate' or 'cast'")
        self.model = model
        self.baseline_policy = baseline_policy or getattr(model, "policy", None) or PrecisionPolicy()
        self.validator = validator or default_conservation_validator
        self.step_fn = step_fn
        params = list(model.parameters())
        self.device = device or (params[0].device if params else torch.device("cpu"))
        self.mode = mode

    # ── rollout and drift ──
    def _run_forward(self, state: State, n_steps: int, forcings=None) -> State:
        was_training = self.model.training
        self.model.eval()
        try:
            with torch.no_grad():
                for _ in range(n_steps):
                    state = (self.step_fn(self.model, state, forcings) if self.step_fn is not None
                             else self.model.step(state, forcings=forcings))
        finally:
            self.model.train(was_training)
        return state

    @staticmethod
    def _measure_drift(base: dict, test: dict) -> tuple:
        per = {}
        for k, b in base.items():
            t = test.get(k, float("nan"))
            if not _finite(b):
                per[k] = float("nan")
            elif not _finite(t):
                per[k] = float("inf")
            else:
                per[k] = abs(float(t) - float(b)) / (abs(float(b)) + 1e-30)
        finite = [v for v in per.values() if math.isfinite(v)]
        if finite:
            return max(finite), per
        return (float("inf") if any(v == float("inf") for v in per.values()) else float("nan")), per

    # ── module precision patching ──
    def _get_top_level_modules(self) -> list:
        return [(n, m) for n, m in self.model.named_children() if isinstance(m, nn.Module)]

    def _get_submodules(self, parent_name: str) -> list:
        parent = dict(self.model.named_modules()).get(parent_name)
        if parent is None:
            return []
        return [(f"{parent_name}.{n}", m) for n, m in parent.named_children()]

    @torch.no_grad()
    def _downcast_module(self, module_name: str, dtype: torch.dtype) -> dict:
        """Lower ``module_name``'s tensors; returns the originals for :meth:`_restore_module`."""
        mod = dict(self.model.named_modules()).get(module_name)
        if mod is None:
            return {}
        saved = {}
        tensors = [(f"p:{n}", t) for n, t in mod.named_parameters()] + \
                  [(f"b:{n}", t) for n, t in mod.named_buffers() if t is not None and t.is_floating_point()]
        for key, t in tensors:
            saved[key] = t.data
            t.data = t.data.to(dtype) if self.mode == "cast" else t.data.to(dtype).to(t.dtype)
        return saved

    @torch.no_grad()
    def _restore_module(self, module_name: str, saved: dict) -> None:
        mod = dict(self.model.named_modules()).get(module_name)
        if mod is None:
            return
        for n, t in mod.named_parameters():
            if f"p:{n}" in saved:
                t.data = saved[f"p:{n}"]
        for n, t in mod.named_buffers():
            if t is not None and f"b:{n}" in saved:
                t.data = saved[f"b:{n}"]

    def profile_module(self, module_name: str, test_dtype: torch.dtype, init_state: State, baseline_metrics: dict,
                       n_steps: int, forcings=None) -> ModuleSensitivity:
        t0 = time.perf_counter()
        saved = self._downcast_module(module_name, test_dtype)
        if not saved:
            return ModuleSensitivity(module_name, 0.0, test_dtype=test_dtype, elapsed_s=time.perf_counter() - t0)
        try:
            metrics = self.validator(self._run_forward(init_state, n_steps, forcings))
            drift, per = self._measure_drift(baseline_metrics, metrics)
        except (RuntimeError, TypeError) as exc:
            logger.info("module %s failed at %s (%s): counted as critical", module_name, test_dtype, exc)
            drift, per = float("inf"), {k: float("inf") for k in baseline_metrics}
        finally:
            self._restore_module(module_name, saved)
        return ModuleSensitivity(module_name, drift, per, test_dtype, time.perf_counter() - t0)

    # ── passes ──
    def run_baseline(self, init_state: State, n_steps: int, forcings=None) -> dict:
        return self.validator(self._run_forward(init_state, n_steps, forcings))

    def run_coarse(self, init_state: State, n_steps: int = 200, test_dtype: torch.dtype = torch.bfloat16,
                   forcings=None, baseline_metrics: Optional[dict] = None) -> SensitivityMap:
        t0 = time.perf_counter()
        base = baseline_metrics if baseline_metrics is not None else self.run_baseline(init_state, n_steps, forcings)
        smap = SensitivityMap(baseline_metrics=base, n_steps=n_steps)
        for name, _ in self._get_top_level_modules():
            smap.modules[name] = self.profile_module(name, test_dtype, init_state, base, n_steps, forcings)
        smap.total_elapsed_s = time.perf_counter() - t0
        return smap

    def run_refine(self, coarse_map: SensitivityMap, init_state: State, refine_threshold: float = 0.01,
                   n_steps: Optional[int] = None, test_dtype: torch.dtype = torch.bfloat16,
                   forcings=None) -> SensitivityMap:
        n_steps = coarse_map.n_steps if n_steps is None else n_steps
        t0 = time.perf_counter()
        hot = [n for n, ms in coarse_map.modules.items() if _finite(ms.drift) and ms.drift > refine_threshold
               or ms.drift == float("inf")]
        if not hot:
            return coarse_map
        out = SensitivityMap(baseline_metrics=coarse_map.baseline_metrics, n_steps=n_steps,
                             refine_threshold=refine_threshold)
        for name, ms in coarse_map.modules.items():
            if name not in hot:
                out.modules[name] = ms
                continue
            count = 0
            for child, mod in self._get_submodules(name):
                if sum(p.numel() for p in mod.parameters()) == 0:
                    continue
                out.modules[child] = self.profile_module(child, test_dtype, init_state,
                                                         coarse_map.baseline_metrics, n_steps, forcings)
                count += 1
            out.modules[name] = dataclasses.replace(ms, n_children_profiled=count)
        out.total_elapsed_s = time.perf_counter() - t0
        return out

    def run_hierarchical(self, init_state: State, n_steps: int = 200, refine_threshold: float = 0.01,
                         test_dtype: torch.dtype = torch.bfloat16, forcings=None) -> SensitivityMap:
        coarse = self.run_coarse(init_state, n_steps, test_dtype, forcings)
        return self.run_refine(coarse, init_state, refine_threshold, n_steps, test_dtype, forcings)

    def profile_module_multi_dtype(self, module_name: str, test_dtypes: list, init_state: State,
                                   baseline_metrics: dict, n_steps: int, forcings=None) -> list:
        return [self.profile_module(module_name, d, init_state, baseline_metrics, n_steps, forcings)
                for d in test_dtypes]

    # ── zone level ──
    def run_zone_perturbation(self, init_state: State, n_steps: int = 200, test_dtype: torch.dtype = torch.bfloat16,
                              use_fp64_baseline: bool = True, forcings=None,
                              zone_targets: Optional[list] = None) -> SensitivityMap:
        """Lower one PZHA zone at a time via ``model.set_precision_policy``; entries ``zone:<name>``."""
        if not hasattr(self.model, "set_precision_policy"):
            raise AttributeError("zone perturbation needs a model with set_precision_policy()")
        t0 = time.perf_counter()
        targets = zone_targets or self._ZONE_TARGETS
        original = self.model.policy
        saved = {n: p.data for n, p in self.model.named_parameters()}
        try:
            base_pol = original
            if use_fp64_baseline:
                base_pol = dataclasses.replace(
                    original, z0_dtype=torch.float64, z1_compute_dtype=torch.float64, z1_use_tf32=False,
                    z1_storage_dtype=torch.float64, z2_compute_dtype=torch.float64, z2_storage_dtype=torch.float64,
                    z3_compute_dtype=torch.float64, z3_param_dtype=torch.float64, z3_master_dtype=torch.float64)
                self._set_params(torch.float64)
            self.model.set_precision_policy(base_pol)
            z1 = base_pol.compute_dtype(PrecisionZone.Z1_DYNAMICS_CORE)
            s0 = init_state.tree_map(lambda t: t.to(z1))
            base = self.validator(self._run_forward(s0, n_steps, forcings))
            smap = SensitivityMap(baseline_metrics=base, n_steps=n_steps)
            for zone, fields, recast in targets:
                name = f"zone:{zone}"
                if not _hps_baseline_metrics_usable(base):
                    smap.modules[name] = ModuleSensitivity(name, float("nan"), test_dtype=test_dtype)
                    continue
                t1 = time.perf_counter()
                pol = dataclasses.replace(base_pol, **{f: test_dtype for f in fields})
                if recast:
                    self._set_params(test_dtype, emulate=self.mode == "emulate")
                self.model.set_precision_policy(pol)
                try:
                    drift, per = self._measure_drift(base, self.validator(self._run_forward(s0, n_steps, forcings)))
                except (RuntimeError, TypeError):
                    drift, per = float("inf"), {}
                finally:
                    self.model.set_precision_policy(base_pol)
                    if recast:
                        self._set_params(torch.float64 if use_fp64_baseline else None, saved=saved)
                smap.modules[name] = ModuleSensitivity(name, drift, per, test_dtype, time.perf_counter() - t1)
            smap.total_elapsed_s = time.perf_counter() - t0
            return smap
        finally:
            self.model.set_precision_policy(original)
            with torch.no_grad():
                for n, p in self.model.named_parameters():
                    p.data = saved[n]

    @torch.no_grad()
    def _set_params(self, dtype, emulate: bool = False, saved: Optional[dict] = None) -> None:
        for n, p in self.model.named_parameters():
            src = saved[n] if saved is not None else p.data
            if dtype is None:
                p.data = src
            elif emulate:
                p.data = src.to(dtype).to(p.dtype)
            else:
                p.data = src.to(dtype)
