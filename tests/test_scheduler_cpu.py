"""Precision scheduler: scripted metric traces through the state machine."""

import math
from types import SimpleNamespace

import torch

from tornado_gcm_b200.precision.policy import PrecisionPolicy
from tornado_gcm_b200.precision.scheduler import (PHASE_ROLLOUTS, PrecisionScheduler, RolloutPlan,
                                                  TrendPlateauTest)
from tornado_gcm_b200.precision.sda import SchedulerConfig


def metrics(losses=(), nan=0, gmax=0.0, tail=0.0):
    stats = {"w": SimpleNamespace(max_abs=gmax)} if gmax else {}
    return SimpleNamespace(recent_losses=list(losses), nan_count=nan, gradient_stats=stats,
                           spectral_energy_tail=tail)


def sched(**kw):
    cfg = SchedulerConfig(**{"warmup_steps_after_switch": 0, **kw})
    return PrecisionScheduler(cfg, PrecisionPolicy(), total_steps=kw.get("total_steps", 1000))


def test_trend_test_separates_decreasing_and_flat_series():
    t = TrendPlateauTest(threshold=0.01)
    dec = [10.0 * math.exp(-0.05 * i) for i in range(40)]
    flat = [1.0 + 0.001 * ((-1) ** i) for i in range(40)]
    assert not t.is_plateau(dec)[0]
    assert t.is_plateau(flat)[0]
    assert not t.is_plateau(flat[:10])[0]  # too few points
    # exact slope: y = 2 + 0.1 i over 11 points changes by 1.0 on a mean of 2.5
    assert abs(TrendPlateauTest.relative_trend([2 + 0.1 * i for i in range(11)]) - 0.4) < 1e-12


def test_milestone_follows_budgets_and_can_skip():
    s = sched(mode="milestone", total_steps=100)
    assert not s.decide(metrics(), 10).policy_changed
    d = s.decide(metrics(), 60)
    assert d.policy_changed and d.rollout_changed and d.new_rollout == PHASE_ROLLOUTS[1]
    assert s.current_phase == 1
    s2 = sched(mode="milestone", total_steps=100)
    d2 = s2.decide(metrics(), 95)  # straight to the last phase
    assert s2.current_phase == 2 and d2.new_rollout == PHASE_ROLLOUTS[2]
    assert s2.current_policy.z3_compute_dtype == torch.float32


def test_loss_aware_needs_patience_and_spacing():
    s = sched(mode="loss_aware", check_interval=10, loss_plateau_patience=3, loss_plateau_threshold=0.01)
    flat = [1.0] * 25
    assert not s.decide(metrics(flat), 10).policy_changed
    assert not s.decide(metrics(), 20).policy_changed
    d = s.decide(metrics(), 30)
    assert d.policy_changed and "loss plateau" in d.reason and s.current_phase == 1
    # window cleared on the switch; a new plateau must build up, and switches are spaced
    assert not s.decide(metrics(flat), 35).policy_changed
    assert not s.decide(metrics(), 40).policy_changed
    assert not s.decide(metrics(), 45).policy_changed  # patience reached, but within 2 checks of the switch
    s._triggers[1].streak = 2
    assert s.decide(metrics(), 60).policy_changed and s.current_phase == 2


def test_loss_aware_decreasing_loss_never_switches():
    s = sched(mode="loss_aware", check_interval=1, loss_plateau_patience=2)
    for step in range(1, 60):
        assert not s.decide(metrics([5.0 * math.exp(-0.1 * step)]), step).policy_changed
    assert s.current_phase == 0


def test_nan_trigger_counts_new_events_only():
    s = sched(mode="loss_aware", nan_trigger_count=2)
    assert not s.decide(metrics(nan=1), 1).policy_changed
    d = s.decide(metrics(nan=2), 500)
    assert d.policy_changed and "NaN" in d.reason
    assert not s.decide(metrics(nan=2), 2000).policy_changed  # no new NaN since the last check


def test_stability_reports_every_cause():
    s = sched(mode="stability_aware", grad_var_threshold=10.0, spectral_tail_threshold=0.1)
    assert not s.decide(metrics(gmax=5.0, tail=0.05), 300).policy_changed
    d = s.decide(metrics(gmax=50.0, tail=0.5), 600)
    assert d.policy_changed and "max |grad|" in d.reason and "spectral tail" in d.reason


def test_deferred_and_ramped_rollout_plan():
    cfg = SchedulerConfig(mode="milestone", warmup_steps_after_switch=3, rollout_ramp_steps=4)
    s = PrecisionScheduler(cfg, PrecisionPolicy(), total_steps=100)
    d = s.decide(metrics(), 60)
    assert d.policy_changed and not d.rollout_changed
    seen = []
    for _ in range(10):
        t = s.tick_warmup()
        seen.append(t.new_rollout if t.rollout_changed else None)
    # nothing for two steps, then 4 -> 16 in four even steps starting when the warm-up ends
    assert seen[:2] == [None, None]
    assert seen[2:6] == [7, 10, 13, 16]
    assert all(v is None for v in seen[6:])


def test_rollout_plan_without_ramp():
    p = RolloutPlan(4, 16, defer=2, ramp=0)
    assert p.tick() is None and p.tick() == (16, "deferred rollout after warm-up") and p.tick() is None


def test_unknown_mode_is_inert():
    s = sched(mode="bogus")
    d = s.decide(metrics([1.0] * 50, nan=10), 99)
    assert not d.policy_changed and "unknown mode" in d.reason
