"""Adaptive precision scheduler (reference ``precision/scheduler.py:33-399``).

Modes: ``milestone`` (fixed 60/30/10 budget fractions), ``loss_aware``
(advance on loss plateau or repeated NaN) and ``stability_aware``
(escalate on NaN, gradient explosion or spectral-tail growth).  A phase
change swaps the policy immediately and defers the rollout increase by
``warmup_steps_after_switch`` steps, optionally ramping it linearly over
``rollout_ramp_steps``.
"""

from __future__ import annotations

import dataclasses
import logging
from collections import deque
from typing import Optional

import torch

from tornado_gcm_b200.precision.policy import PrecisionPolicy

logger = logging.getLogger(__name__)

PHASE_CONFIGS = [
    dict(z3_compute_dtype=torch.bfloat16, z1_use_tf32=True, z2_compute_dtype=torch.float32),
    dict(z3_compute_dtype=torch.bfloat16, z1_use_tf32=True, z2_compute_dtype=torch.float64),
    dict(z3_compute_dtype=torch.float32, z3_param_dtype=torch.float32, z1_use_tf32=True,
         z2_compute_dtype=torch.float64),
]
PHASE_ROLLOUTS = [4, 16, 32]
PHASE_BUDGETS = (0.60, 0.30, 0.10)


@dataclasses.dataclass
class SchedulerDecision:
    policy_changed: bool = False
    new_policy: Optional[PrecisionPolicy] = None
    rollout_changed: bool = False
    new_rollout: Optional[int] = None
    reason: str = ""


class PrecisionScheduler:
    def __init__(self, config, base_policy: PrecisionPolicy, total_steps: int = 100_000) -> None:
        self.config = config
        self.base_policy = base_policy
        self.total_steps = total_steps
        self.current_phase = 0
        self.max_phase = len(PHASE_CONFIGS) - 1
        self._phase_policies = [dataclasses.replace(base_policy, **c) for c in PHASE_CONFIGS]
        self._phase_rollouts = list(PHASE_ROLLOUTS)
        self._loss_window: deque = deque(maxlen=200)
        self._plateau_count = 0
        self._nan_count = 0
        self._last_switch_step = 0
        self._warmup_remaining = 0
        self._pending_rollout: Optional[int] = None
        self._ramp_remaining = 0
        self._ramp_start = PHASE_ROLLOUTS[0]
        self._ramp_target = PHASE_ROLLOUTS[0]
        self._ramp_total = 0
        self.last_decision = SchedulerDecision()

    def decide(self, metrics, step: int) -> SchedulerDecision:
        mode = self.config.mode
        if mode == "milestone":
            d = self._milestone(step)
        elif mode == "loss_aware":
            d = self._loss_aware(metrics, step)
        elif mode == "stability_aware":
            d = self._stability(metrics, step)
        else:
            d = SchedulerDecision(reason=f"unknown mode: {mode}")
        self.last_decision = d
        return d

    def _milestone(self, step: int) -> SchedulerDecision:
        frac = step / max(self.total_steps, 1)
        acc, target = 0.0, self.max_phase
        for i, b in enumerate(PHASE_BUDGETS):
            acc += b
            if frac < acc:
                target = i
                break
        if target > self.current_phase:
            return self._advance_to(target, step, reason="milestone")
        return SchedulerDecision()

    def _loss_aware(self, metrics, step: int) -> SchedulerDecision:
        for v in metrics.recent_losses:
            self._loss_window.append(v)
        if metrics.nan_count > self._nan_count:
            self._nan_count = metrics.nan_count
            if metrics.nan_count >= self.config.nan_trigger_count and self.current_phase < self.max_phase:
                return self._advance_to(self.current_phase + 1, step, reason=f"NaN detected ({metrics.nan_count}x)")
        n = len(self._loss_window)
        if n < 20:
            return SchedulerDecision()
        w = list(self._loss_window)
        h = n // 2
        old, new = sum(w[:h]) / h, sum(w[h:]) / (n - h)
        if old == 0:
            return SchedulerDecision()
        rel = abs(new - old) / (abs(old) + 1e-30)
        self._plateau_count = self._plateau_count + 1 if rel < self.config.loss_plateau_threshold \
            else max(0, self._plateau_count - 1)
        if (self._plateau_count >= self.config.loss_plateau_patience and self.current_phase < self.max_phase
                and step - self._last_switch_step > self.config.check_interval * 3):
            self._plateau_count = 0
            self._loss_window.clear()
            return self._advance_to(self.current_phase + 1, step, reason=f"loss plateau (rel_change={rel:.4f})")
        return SchedulerDecision()

    def _stability(self, metrics, step: int) -> SchedulerDecision:
        reasons = []
        if metrics.nan_count >= self.config.nan_trigger_count:
            reasons.append(f"NaN×{metrics.nan_count}")
        if metrics.gradient_stats:
            gmax = max((g.max_abs for g in metrics.gradient_stats.values()), default=0.0)
            if gmax > self.config.grad_var_threshold:
                reasons.append(f"grad_max={gmax:.1e}")
        if metrics.spectral_energy_tail > self.config.spectral_tail_threshold:
            reasons.append(f"spectral_tail={metrics.spectral_energy_tail:.3f}")
        if reasons and self.current_phase < self.max_phase and \
                step - self._last_switch_step > self.config.check_interval * 2:
            return self._advance_to(self.current_phase + 1, step, reason="stability: " + ", ".join(reasons))
        return SchedulerDecision()

    def _advance_to(self, target: int, step: int, *, reason: str) -> SchedulerDecision:
        target = min(target, self.max_phase)
        if target <= self.current_phase:
            return SchedulerDecision()
        self.current_phase = target
        self._last_switch_step = step
        pol, rollout = self._phase_policies[target], self._phase_rollouts[target]
        if self.config.warmup_steps_after_switch > 0:
            self._warmup_remaining = self.config.warmup_steps_after_switch
            self._pending_rollout = rollout
            return SchedulerDecision(True, pol, False, None, reason)
        return SchedulerDecision(True, pol, True, rollout, reason)

    def tick_warmup(self) -> SchedulerDecision:
        if self._warmup_remaining > 0:
            self._warmup_remaining -= 1
            if self._warmup_remaining == 0 and self._pending_rollout is not None:
                target = self._pending_rollout
                self._pending_rollout = None
                ramp = self.config.rollout_ramp_steps
                if ramp > 0:
                    self._ramp_start = self._phase_rollouts[max(0, self.current_phase - 1)]
                    self._ramp_target = target
                    self._ramp_total = ramp
                    self._ramp_remaining = ramp
                    return self._ramp_tick()
                return SchedulerDecision(rollout_changed=True, new_rollout=target,
                                         reason="deferred rollout after warmup")
            return SchedulerDecision()
        if self._ramp_remaining > 0:
            return self._ramp_tick()
        return SchedulerDecision()

    def _ramp_tick(self) -> SchedulerDecision:
        self._ramp_remaining -= 1
        prog = 1.0 - self._ramp_remaining / max(self._ramp_total, 1)
        k = max(1, round(self._ramp_start + prog * (self._ramp_target - self._ramp_start)))
        if self._ramp_remaining == 0:
            k = self._ramp_target
        return SchedulerDecision(rollout_changed=True, new_rollout=k, reason=f"rollout ramp ({prog:.0%})")

    @property
    def current_policy(self) -> PrecisionPolicy:
        return self._phase_policies[self.current_phase]

    @property
    def current_rollout(self) -> int:
        return self._phase_rollouts[self.current_phase]
