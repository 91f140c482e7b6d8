"""Optimisers and gradient tools (reference ``training/optimization.py:36-261``)."""

from __future__ import annotations

import re
from typing import Sequence

import torch
import torch.nn as nn

from tornado_gcm_b200.core.primitive_equations import State


def _normalize_param_name(name: str) -> str:
    for p in ("module.", "_orig_mod.", "_fsdp_wrapped_module."):
        name = name.replace(p, "")
    return name


def multi_adam(model: nn.Module, top_level_keys: Sequence[str] = (), learning_rates: Sequence[float] = (),
               default_learning_rate: float = 1e-4, b1: float = 0.9, b2: float = 0.95, eps: float = 1e-6,
               weight_decay: float = 0.0, raise_if_keys_not_found: bool = True, fused: bool | None = None,
               capturable: bool = False) -> torch.optim.Optimizer:
    """AdamW with per-group learning rates matched by module prefix or ``REGEX_<pattern>``."""
    if len(top_level_keys) != len(learning_rates):
        raise ValueError(f"top_level_keys ({len(top_level_keys)}) and learning_rates ({len(learning_rates)}) "
                         "must have same length")
    matchers = []
    for key in top_level_keys:
        if key.startswith("REGEX_"):
            pat = re.compile(key[6:])
            matchers.append(lambda n, p=pat: p.search(n) is not None or p.search(_normalize_param_name(n)) is not None)
        else:
            matchers.append(lambda n, k=key: any(x == k or x.startswith(k + ".")
                                                 for x in (n, _normalize_param_name(n))))
    groups = [[] for _ in top_level_keys]
    default = []
    hit = set()
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        for i, m in enumerate(matchers):
            if m(name):
                groups[i].append(p)
                hit.add(i)
                break
        else:
            default.append(p)
    if raise_if_keys_not_found:
        for i, k in enumerate(top_level_keys):
            if i not in hit:
                raise ValueError(f"Parameter group key '{k}' matched no parameters")
    pg = [{"params": g, "lr": lr, "name": k} for g, lr, k in zip(groups, learning_rates, top_level_keys) if g]
    if default:
        pg.append({"params": default, "lr": default_learning_rate, "name": "default"})
    if fused is None:
        fused = all(p.is_cuda for g in pg for p in g["params"])
    return torch.optim.AdamW(pg, lr=default_learning_rate, betas=(b1, b2), eps=eps, weight_decay=weight_decay,
                             fused=fused, capturable=capturable)


def _detach_state(state):
    if isinstance(state, State):
        return state.tree_map(lambda t: t.detach().requires_grad_(t.requires_grad))
    if isinstance(state, dict):
        return {k: _detach_state(v) for k, v in state.items()}
    if isinstance(state, torch.Tensor):
        return state.detach().requires_grad_(state.requires_grad)
    return state


class StopGradientTrajectory:
    """Rollout with gradient cuts at the given outer steps."""

    def __init__(self, stop_gradient_outer_steps: Sequence[int] = ()):
        self.stops = sorted(stop_gradient_outer_steps)

    def rollout(self, step_fn, initial_state, total_outer_steps: int, inner_steps: int = 1) -> list:
        bounds = [0] + [s for s in self.stops if 0 < s < total_outer_steps] + [total_outer_steps]
        traj = []
        state = initial_state
        for leg in range(len(bounds) - 1):
            if leg > 0:
                state = _detach_state(state)
            for _ in range(bounds[leg], bounds[leg + 1]):
                for _ in range(inner_steps):
                    state = step_fn(state)
                traj.append(state)
        return traj


class MixedPrecisionBackward(torch.autograd.Function):
    """Low-precision forward, fp32 backward ("recompute": re-run forward in fp32;
    "stash": differentiate the low-precision graph)."""

    @staticmethod
    def forward(ctx, module: nn.Module, x: torch.Tensor, fwd_dtype: torch.dtype = torch.bfloat16,
                mode: str = "recompute"):
        ctx.module, ctx.mode, ctx.fwd_dtype = module, mode, fwd_dtype
        ctx.save_for_backward(x)
        with torch.no_grad():
            y = module(x.to(fwd_dtype))
        return y.to(x.dtype)

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        dtype = torch.float32 if ctx.mode == "recompute" else ctx.fwd_dtype
        with torch.enable_grad():
            xi = x.detach().to(dtype).requires_grad_(True)
            params = [p for p in ctx.module.parameters() if p.requires_grad]
            y = ctx.module(xi)
            grads = torch.autograd.grad(y, [xi] + params, g.to(y.dtype), allow_unused=True)
        for p, gp in zip(params, grads[1:]):
            if gp is None:
                continue
            gp = gp.to(p.dtype)
            p.grad = gp if p.grad is None else p.grad + gp
        return None, grads[0].to(x.dtype), None, None
