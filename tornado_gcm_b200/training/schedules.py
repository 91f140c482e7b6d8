"""Rollout and learning-rate schedules (reference ``training/schedules.py:33-270``).

The learning-rate schedules follow the optax definitions of the same names
(cosine with linear warmup, exponential decay, warmup + exponential decay,
piecewise constant by scales / by rates, delayed constant, joined).
"""

from __future__ import annotations

import bisect
import dataclasses
import math
from typing import Optional, Sequence


@dataclasses.dataclass
class ProgressiveRolloutSchedule:
    total_steps: int
    milestones: tuple = (0.20, 0.50, 0.80)
    rollout_lengths: tuple = (4, 8, 16, 32)

    def __post_init__(self):
        if len(self.rollout_lengths) != len(self.milestones) + 1:
            raise ValueError(f"rollout_lengths ({len(self.rollout_lengths)}) must be "
                             f"len(milestones)+1 ({len(self.milestones) + 1})")

    def get_rollout(self, step: int, max_available: Optional[int] = None) -> int:
        k = self.rollout_lengths[bisect.bisect_right(self.milestones, step / max(self.total_steps, 1))]
        if max_available is not None:
            k = min(k, max_available)
        return max(k, 1)


@dataclasses.dataclass
class CosineDecaySchedule:
    base_lr: float = 1e-3
    warmup_steps: int = 1000
    total_steps: int = 100_000
    min_lr: float = 1e-6

    def __call__(self, step: int) -> float:
        if step < self.warmup_steps:
            return self.base_lr * step / max(self.warmup_steps, 1)
        p = min((step - self.warmup_steps) / max(self.total_steps - self.warmup_steps, 1), 1.0)
        return self.min_lr + 0.5 * (self.base_lr - self.min_lr) * (1.0 + math.cos(math.pi * p))


LearningRateSchedule = CosineDecaySchedule


def _exponent(count: int, steps: int, staircase: bool) -> float:
    return count // max(steps, 1) if staircase else count / max(steps, 1)


@dataclasses.dataclass
class ExponentialDecaySchedule:
    init_value: float = 1e-4
    transition_steps: int = 100_000
    decay_rate: float = 0.1
    transition_begin: int = 0
    staircase: bool = False
    end_value: float = 0.0

    def __call__(self, step: int) -> float:
        c = max(step - self.transition_begin, 0)
        return max(self.init_value * self.decay_rate ** _exponent(c, self.transition_steps, self.staircase),
                   self.end_value)


@dataclasses.dataclass
class WarmupExponentialDecaySchedule:
    init_value: float = 0.0
    peak_value: float = 1e-4
    warmup_steps: int = 1000
    transition_steps: int = 100_000
    decay_rate: float = 0.1
    transition_begin: int = 0
    staircase: bool = False
    end_value: float = 0.0

    def __call__(self, step: int) -> float:
        if step < self.warmup_steps:
            return self.init_value + step / max(self.warmup_steps, 1) * (self.peak_value - self.init_value)
        if step < self.warmup_steps + self.transition_begin:
            return self.peak_value
        c = max(step - self.warmup_steps - self.transition_begin, 0)
        return max(self.peak_value * self.decay_rate ** _exponent(c, self.transition_steps, self.staircase),
                   self.end_value)


@dataclasses.dataclass
class PiecewiseConstantSchedule:
    init_value: float = 1e-4
    boundaries_and_scales: dict = dataclasses.field(default_factory=dict)

    def __call__(self, step: int) -> float:
        lr = self.init_value
        for b in sorted(self.boundaries_and_scales):
            if step < b:
                break
            lr *= self.boundaries_and_scales[b]
        return lr


@dataclasses.dataclass
class PiecewiseConstantByRatesSchedule:
    rates: Sequence = (0.0, 1e-4)
    boundaries: Sequence = (1000,)

    def __post_init__(self):
        if len(self.rates) != len(self.boundaries) + 1:
            raise ValueError(f"len(rates)={len(self.rates)} must be len(boundaries)+1={len(self.boundaries) + 1}")

    def __call__(self, step: int) -> float:
        return float(self.rates[bisect.bisect_right(list(self.boundaries), step)])


@dataclasses.dataclass
class DelayedConstantSchedule:
    turn_on_step: int = 0
    rate: float = 1e-4

    def __call__(self, step: int) -> float:
        return self.rate if step >= self.turn_on_step else 0.0


@dataclasses.dataclass
class JoinedSchedule:
    schedules: Sequence = dataclasses.field(default_factory=list)
    boundaries: Sequence = dataclasses.field(default_factory=list)

    def __call__(self, step: int) -> float:
        i = bisect.bisect_right(list(self.boundaries), step)
        off = 0 if i == 0 else self.boundaries[i - 1]
        return float(self.schedules[i](step - off))


def apply_lr(optimizer, lr: float) -> None:
    """Set the learning rate of every parameter group."""
    for g in optimizer.param_groups:
        if isinstance(g.get("lr"), float) or not hasattr(g.get("lr"), "fill_"):
            g["lr"] = lr
        else:
            g["lr"].fill_(lr)
