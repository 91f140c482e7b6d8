"""Multi-frequency nested rollouts (reference ``core/scan_utils.py:43-355``)."""

from __future__ import annotations

import dataclasses
import math
from typing import Any, Callable

import torch
import torch.utils.checkpoint as checkpoint_util


def compute_nested_steps(frequencies: dict, dt=1, total_steps: int | None = None) -> tuple:
    """Steps per nesting level, innermost first (e.g. {'atmos': 6, 'ocean': 24}, 72 → (6, 4, 3))."""
    if not frequencies:
        return (total_steps,) if total_steps is not None else ()
    intervals = sorted(int(v / dt) for v in frequencies.values())
    intervals = sorted(set(intervals))
    steps, prev = [], 1
    for iv in intervals:
        n, rem = divmod(iv, prev)
        if rem:
            raise ValueError(f"Forcing intervals are not congruent: {iv} is not divisible by {prev}.")
        steps.append(n)
        prev = iv
    if total_steps is not None:
        inner = math.prod(steps)
        n_out, rem = divmod(total_steps, inner)
        if rem:
            raise ValueError(f"total_steps={total_steps} is not divisible by the product of nested intervals "
                             f"({inner}).")
        steps.append(n_out)
    return tuple(steps)


def frequency_groups(frequencies: dict, dt=1) -> list:
    groups: dict = {}
    for name, f in frequencies.items():
        groups.setdefault(int(f / dt), []).append(name)
    return sorted(groups.items(), key=lambda kv: kv[0])


@dataclasses.dataclass
class NestedForcingLevel:
    steps: int
    var_names: list
    data: list
    stride: int


def nest_forcings(forcings: list, frequencies: dict, dt=1, total_steps: int | None = None) -> list:
    total_steps = len(forcings) if total_steps is None else total_steps
    steps = compute_nested_steps(frequencies, dt, total_steps)
    groups = frequency_groups(frequencies, dt)
    levels = [NestedForcingLevel(steps[0], [], [], 1)]
    stride = steps[0]
    for li, (_, names) in enumerate(groups, start=1):
        n = steps[li] if li < len(steps) else 1
        data = []
        for s in range(n):
            gi = s * stride
            src = forcings[gi] if gi < len(forcings) else {}
            data.append({k: src[k] for k in names if k in src})
        levels.append(NestedForcingLevel(n, list(names), data, stride))
        stride *= n
    if len(steps) > len(levels):
        levels.append(NestedForcingLevel(steps[len(levels)], [], [], stride))
    return levels


def nested_scan(step_fn: Callable, initial_state: Any, levels: list, checkpoint_level: int = -1,
                collect_every: int = 1) -> tuple[Any, list]:
    """Recursive unroll; forcings of outer levels stay active while inner levels run."""
    traj: list = []
    counter = [0]

    def run(state, li, ctx):
        lvl = levels[li]
        for s in range(lvl.steps):
            local = dict(ctx)
            if lvl.data:
                local.update(lvl.data[s])
            if li == 0:
                state = step_fn(state, local if local else None)
                counter[0] += 1
                if counter[0] % collect_every == 0:
                    traj.append(state)
            elif li == checkpoint_level:
                state = _ckpt(lambda st, _li=li, _c=local: run(st, _li - 1, _c), state)
            else:
                state = run(state, li - 1, local)
        return state

    final = run(initial_state, len(levels) - 1, {})
    return final, traj


def _ckpt(fn, state):
    from tornado_gcm_b200.training.trainer import _flatten, _unflatten

    flat, meta = _flatten(state)
    holder = {}

    def seg(*a):
        out = fn(_unflatten(a, meta))
        f, m = _flatten(out)
        holder["m"] = m
        return f

    res = checkpoint_util.checkpoint(seg, *flat, use_reentrant=False)
    res = (res,) if isinstance(res, torch.Tensor) else res
    return _unflatten(res, holder["m"])


def nested_rollout(step_fn: Callable, initial_state: Any, forcings: list, frequencies: dict, dt=1,
                   checkpoint_level: int = -1, collect_every: int = 1) -> tuple[Any, list]:
    levels = nest_forcings(forcings, frequencies, dt)
    return nested_scan(step_fn, initial_state, levels, checkpoint_level, collect_every)
