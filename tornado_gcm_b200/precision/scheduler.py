"""Precision-phase scheduler of the SDA loop.

Behaviour parity: reference ``precision/scheduler.py:33-399`` (modes
``milestone`` / ``loss_aware`` / ``stability_aware``, the three training
phases with 60/30/10 % step budgets and rollouts 4/16/32, a deferred and
optionally ramped rollout increase after a phase change).  The design here
is a small state machine:

* :data:`PHASES` — the phase table (policy overrides, rollout, budget).
* Triggers — objects with ``check(view) -> reason | None`` that read one
  :class:`MetricsView` (the metrics stream as seen at a check) and propose
  moving to the next phase.  A mode is just a list of triggers
  (:data:`MODE_TRIGGERS`); the first trigger that fires wins.
* :class:`TrendPlateauTest` — the loss plateau test: an ordinary
  least-squares line through the last ``window`` losses; the loss has
  plateaued when the change of the fitted line across the window,
  relative to the window mean, is below ``threshold`` in magnitude.  The
  test has to pass at ``patience`` consecutive checks.
* :class:`RolloutPlan` — the rollout changes that follow a phase switch,
  as an explicit list of ``(step_offset, rollout)`` events (deferred by
  ``warmup_steps_after_switch``, then a linear ramp over
  ``rollout_ramp_steps``), consumed one step at a time by
  :meth:`PrecisionScheduler.tick_warmup`.
* A minimum spacing between switches (``min_switch_spacing`` checks worth
  of steps) keeps a noisy metric from racing through the phases.
"""

from __future__ import annotations

import dataclasses
import logging
import math
from collections import deque
from typing import Optional, Sequence

import torch

from tornado_gcm_b200.precision.policy import PrecisionPolicy

logger = logging.getLogger(__name__)


@dataclasses.dataclass(frozen=True)
class Phase:
    name: str
    overrides: dict
    rollout: int
    budget: float  # fraction of the training steps (milestone mode)


# The reference's documented three-phase training schedule.
PHASES: tuple[Phase, ...] = (
    Phase("low_precision_pretrain",
          dict(z3_compute_dtype=torch.bfloat16, z1_use_tf32=True, z2_compute_dtype=torch.float32), 4, 0.60),
    Phase("mixed_precision_train",
          dict(z3_compute_dtype=torch.bfloat16, z1_use_tf32=True, z2_compute_dtype=torch.float64), 16, 0.30),
    Phase("high_precision_finetune",
          dict(z3_compute_dtype=torch.float32, z3_param_dtype=torch.float32, z1_use_tf32=True,
               z2_compute_dtype=torch.float64), 32, 0.10),
)
# Flat views of the table under the reference's names (public constants there).
PHASE_CONFIGS = [p.overrides for p in PHASES]
PHASE_ROLLOUTS = [p.rollout for p in PHASES]
PHASE_BUDGETS = tuple(p.budget for p in PHASES)


@dataclasses.dataclass
class SchedulerDecision:
    policy_changed: bool = False
    new_policy: Optional[PrecisionPolicy] = None
    rollout_changed: bool = False
    new_rollout: Optional[int] = None
    reason: str = ""


@dataclasses.dataclass
class MetricsView:
    """What a trigger may look at during one check."""

    step: int
    total_steps: int
    phase: int
    losses: Sequence[float]          # the scheduler's loss window (oldest first)
    nan_count: int                   # cumulative, as reported by the profiler
    new_nans: int                    # NaN events since the previous check
    grad_max_abs: float
    spectral_tail: float
    config: object


# ── tests and triggers ─────────────────────────────────────────────────────
class TrendPlateauTest:
    """Least-squares trend test for a loss plateau.

    For losses y_0..y_{n-1} the fitted slope is
    ``b = Σ (i - ī)(y_i - ȳ) / Σ (i - ī)²`` and the fitted change across the
    window is ``b · (n - 1)``.  The window is a plateau when
    ``|b · (n - 1)| < threshold · |ȳ|``.  Windows shorter than
    ``min_points`` never count as a plateau.
    """

    def __init__(self, threshold: float, min_points: int = 20):
        self.threshold = float(threshold)
        self.min_points = int(min_points)

    @staticmethod
    def relative_trend(values: Sequence[float]) -> float:
        n = len(values)
        if n < 2:
            return math.inf
        xm = (n - 1) / 2.0
        ym = sum(values) / n
        sxx = sum((i - xm) ** 2 for i in range(n))
        sxy = sum((i - xm) * (v - ym) for i, v in enumerate(values))
        change = sxy / sxx * (n - 1)
        if ym == 0.0:
            return math.inf
        return abs(change) / abs(ym)

    def is_plateau(self, values: Sequence[float]) -> tuple[bool, float]:
        if len(values) < self.min_points:
            return False, math.inf
        rel = self.relative_trend(values)
        return rel < self.threshold, rel


class NaNTrigger:
    """Fires when the profiler's cumulative NaN count reaches the configured count with new NaNs seen."""

    def check(self, v: MetricsView) -> Optional[str]:
        if v.new_nans > 0 and v.nan_count >= v.config.nan_trigger_count:
            return f"NaN events: {v.nan_count}"
        return None


class PlateauTrigger:
    """Fires after ``loss_plateau_patience`` consecutive plateau verdicts of :class:`TrendPlateauTest`."""

    def __init__(self):
        self.streak = 0

    def reset(self) -> None:
        self.streak = 0

    def check(self, v: MetricsView) -> Optional[str]:
        test = TrendPlateauTest(v.config.loss_plateau_threshold)
        flat, rel = test.is_plateau(v.losses)
        self.streak = self.streak + 1 if flat else 0
        if self.streak >= v.config.loss_plateau_patience:
            self.streak = 0
            return f"loss plateau (fitted relative change {rel:.4g} over {len(v.losses)} losses)"
        return None


class InstabilityTrigger:
    """Fires on NaNs, a gradient magnitude above ``grad_var_threshold`` or a
    spectral energy tail above ``spectral_tail_threshold``; the reason lists every cause."""

    def check(self, v: MetricsView) -> Optional[str]:
        cfg = v.config
        causes = []
        if v.nan_count >= cfg.nan_trigger_count:
            causes.append(f"NaN events {v.nan_count}")
        if v.grad_max_abs > cfg.grad_var_threshold:
            causes.append(f"max |grad| {v.grad_max_abs:.3g}")
        if v.spectral_tail > cfg.spectral_tail_threshold:
            causes.append(f"spectral tail {v.spectral_tail:.3g}")
        return ("instability: " + "; ".join(causes)) if causes else None


class BudgetTrigger:
    """Milestone mode: the phase whose cumulative budget contains step / total_steps.

    Returns the reason and stores the target phase (may skip phases).
    """

    def __init__(self, phases: Sequence[Phase]):
        self.bounds = []
        acc = 0.0
        for p in phases:
            acc += p.budget
            self.bounds.append(acc)
        self.target = 0

    def phase_for(self, frac: float) -> int:
        for i, b in enumerate(self.bounds):
            if frac < b:
                return i
        return len(self.bounds) - 1

    def check(self, v: MetricsView) -> Optional[str]:
        frac = v.step / max(v.total_steps, 1)
        self.target = self.phase_for(frac)
        if self.target > v.phase:
            return f"milestone: {frac:.1%} of {v.total_steps} steps"
        return None


MODE_TRIGGERS = {
    "milestone": lambda phases: [BudgetTrigger(phases)],
    "loss_aware": lambda phases: [NaNTrigger(), PlateauTrigger()],
    "stability_aware": lambda phases: [InstabilityTrigger()],
}


# ── rollout plan after a switch ────────────────────────────────────────────
class RolloutPlan:
    """Rollout events after a phase switch: ``events[k] = (steps after the switch, rollout)``."""

    def __init__(self, start: int, target: int, defer: int, ramp: int):
        self.events: deque = deque()
        self.elapsed = 0
        if defer <= 0 and ramp <= 0:
            return
        if ramp <= 0:
            self.events.append((defer, target, "deferred rollout after warm-up"))
            return
        first = max(defer, 1)  # the ramp starts on the step the warm-up ends
        for k in range(1, ramp + 1):
            frac = k / ramp
            r = target if k == ramp else max(1, int(round(start + frac * (target - start))))
            self.events.append((first + k - 1, r, f"rollout ramp {frac:.0%}"))

    def tick(self) -> Optional[tuple[int, str]]:
        """Advance one step; the rollout change due at this step, if any."""
        if not self.events:
            return None
        self.elapsed += 1
        due = None
        while self.events and self.events[0][0] <= self.elapsed:
            _, r, why = self.events.popleft()
            due = (r, why)
        return due

    @property
    def pending(self) -> bool:
        return bool(self.events)


# ── the scheduler ──────────────────────────────────────────────────────────
class PrecisionScheduler:
    """Decides phase switches from profiler metrics; see the module docstring."""

    def __init__(self, config, base_policy: PrecisionPolicy, total_steps: int = 100_000,
                 phases: Sequence[Phase] = PHASES) -> None:
        self.config = config
        self.base_policy = base_policy
        self.total_steps = total_steps
        self.phases = tuple(phases)
        self.current_phase = 0
        self.max_phase = len(self.phases) - 1
        self._policies = [dataclasses.replace(base_policy, **p.overrides) for p in self.phases]
        self._window: deque = deque(maxlen=int(getattr(config, "loss_window", 200)))
        self._triggers = MODE_TRIGGERS.get(config.mode, lambda ph: [])(self.phases)
        self._seen_nans = 0
        self._last_switch: Optional[int] = None
        self._plan = RolloutPlan(0, 0, 0, 0)
        self.last_decision = SchedulerDecision()

    # spacing between switches, in steps
    def _spacing(self) -> int:
        checks = int(getattr(self.config, "min_switch_spacing", 2))
        return checks * max(int(self.config.check_interval), 1)

    def _view(self, metrics, step: int) -> MetricsView:
        for x in getattr(metrics, "recent_losses", ()) or ():
            if x == x:  # NaN losses are counted by the profiler, not averaged
                self._window.append(float(x))
        nan_count = int(getattr(metrics, "nan_count", 0))
        new = max(0, nan_count - self._seen_nans)
        self._seen_nans = max(self._seen_nans, nan_count)
        stats = getattr(metrics, "gradient_stats", None) or {}
        gmax = max((float(g.max_abs) for g in stats.values()), default=0.0)
        return MetricsView(step, self.total_steps, self.current_phase, tuple(self._window), nan_count, new, gmax,
                           float(getattr(metrics, "spectral_energy_tail", 0.0)), self.config)

    def decide(self, metrics, step: int) -> SchedulerDecision:
        if not self._triggers:
            d = SchedulerDecision(reason=f"unknown mode: {self.config.mode}")
            self.last_decision = d
            return d
        view = self._view(metrics, step)
        d = SchedulerDecision()
        if self.current_phase < self.max_phase:
            spaced = self._last_switch is None or step - self._last_switch > self._spacing()
            milestone = self.config.mode == "milestone"
            for trig in self._triggers:
                reason = trig.check(view)
                if reason is None:
                    continue
                if not (spaced or milestone):
                    break
                target = trig.target if isinstance(trig, BudgetTrigger) else self.current_phase + 1
                d = self._switch(target, step, reason)
                break
        self.last_decision = d
        return d

    def _switch(self, target: int, step: int, reason: str) -> SchedulerDecision:
        target = min(target, self.max_phase)
        if target <= self.current_phase:
            return SchedulerDecision()
        start = self.phases[self.current_phase].rollout
        self.current_phase = target
        self._last_switch = step
        self._window.clear()
        for t in self._triggers:
            if hasattr(t, "reset"):
                t.reset()
        new_rollout = self.phases[target].rollout
        defer = int(self.config.warmup_steps_after_switch)
        ramp = int(getattr(self.config, "rollout_ramp_steps", 0))
        logger.info("precision phase -> %s at step %d (%s)", self.phases[target].name, step, reason)
        if defer <= 0 and ramp <= 0:
            self._plan = RolloutPlan(0, 0, 0, 0)
            return SchedulerDecision(True, self._policies[target], True, new_rollout, reason)
        self._plan = RolloutPlan(start, new_rollout, defer, ramp)
        return SchedulerDecision(True, self._policies[target], False, None, reason)

    def tick_warmup(self) -> SchedulerDecision:
        """Per-step call: emits the rollout change of the plan that is due at this step."""
        due = self._plan.tick()
        if due is None:
            return SchedulerDecision()
        return SchedulerDecision(rollout_changed=True, new_rollout=due[0], reason=due[1])

    @property
    def current_policy(self) -> PrecisionPolicy:
        return self._policies[self.current_phase]

    @property
    def current_rollout(self) -> int:
        return self.phases[self.current_phase].rollout
