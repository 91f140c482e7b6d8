"""Zone-boundary casts (reference ``precision/zone_cast.py:85-262``)."""

from __future__ import annotations

import functools
from typing import Any, Callable, Optional

import torch

from tornado_gcm_b200.precision.policy import PrecisionPolicy, PrecisionZone

_DTYPE_RANK = {torch.bfloat16: 0, torch.float16: 0, torch.float32: 1, torch.float64: 2}


def _dtype_rank(dtype: torch.dtype) -> int:
    return _DTYPE_RANK.get(dtype, 1)


def zone_cast(x: torch.Tensor, src_zone: PrecisionZone, dst_zone: PrecisionZone, policy: PrecisionPolicy, *,
              monitor: Optional[Any] = None, name: str = "") -> torch.Tensor:
    """Cast to the destination zone's compute dtype; audit downcasts if a monitor is given."""
    if src_zone == dst_zone:
        return x
    dst = policy.compute_dtype(dst_zone)
    if x.dtype == dst:
        return x
    out = x.to(dst)
    if (monitor is not None and policy.enable_precision_audit
            and _dtype_rank(dst) < _dtype_rank(policy.compute_dtype(src_zone))):
        monitor.audit_zone_transfer(name or f"{src_zone.value}→{dst_zone.value}", x, out)
    return out


def tree_zone_cast(tree: Any, src_zone, dst_zone, policy, **kw) -> Any:
    if isinstance(tree, torch.Tensor):
        return zone_cast(tree, src_zone, dst_zone, policy, **kw)
    if isinstance(tree, dict):
        return {k: tree_zone_cast(v, src_zone, dst_zone, policy, **kw) for k, v in tree.items()}
    if isinstance(tree, (list, tuple)):
        return type(tree)(tree_zone_cast(v, src_zone, dst_zone, policy, **kw) for v in tree)
    if hasattr(tree, "tree_map"):
        return tree.tree_map(lambda t: zone_cast(t, src_zone, dst_zone, policy, **kw)
                             if isinstance(t, torch.Tensor) else t)
    return tree


def _cast_any(obj: Any, dtype: torch.dtype) -> Any:
    if isinstance(obj, torch.Tensor):
        return obj.to(dtype) if obj.is_floating_point() else obj
    if isinstance(obj, tuple):
        return tuple(_cast_any(o, dtype) for o in obj)
    if isinstance(obj, list):
        return [_cast_any(o, dtype) for o in obj]
    if isinstance(obj, dict):
        return {k: _cast_any(v, dtype) for k, v in obj.items()}
    if hasattr(obj, "tree_map"):
        return obj.tree_map(lambda t: t.to(dtype) if isinstance(t, torch.Tensor) else t)
    return obj


def zone_boundary(src: PrecisionZone, dst: PrecisionZone, policy: PrecisionPolicy, *, cast_output: bool = True):
    """Decorator: inputs cast src→dst, outputs cast back dst→src."""
    def deco(fn):
        @functools.wraps(fn)
        def wrapper(*args, **kwargs):
            a = tuple(tree_zone_cast(x, src, dst, policy) for x in args)
            k = {n: tree_zone_cast(v, src, dst, policy) for n, v in kwargs.items()}
            out = fn(*a, **k)
            return tree_zone_cast(out, dst, src, policy) if cast_output else out
        return wrapper
    return deco


def f64_math(fn: Callable) -> Callable:
    """Run ``fn`` on FP64 copies of its tensor arguments; cast results back."""
    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        dtypes = [a.dtype for a in args if isinstance(a, torch.Tensor) and a.is_floating_point()]
        out_dtype = max(dtypes, key=_dtype_rank) if dtypes else torch.float32
        out = fn(*[_cast_any(a, torch.float64) for a in args],
                 **{k: _cast_any(v, torch.float64) for k, v in kwargs.items()})
        return _cast_any(out, out_dtype)
    return wrapper


def einsum_highest(subscripts: str, *operands: torch.Tensor) -> torch.Tensor:
    """FP64-intermediate einsum; result in the highest input floating dtype."""
    if not operands:
        raise ValueError("einsum_highest requires at least one operand")
    fl = [o for o in operands if o.is_floating_point()]
    if not fl:
        return torch.einsum(subscripts, *operands)
    out_dtype = max(fl, key=lambda t: _dtype_rank(t.dtype)).dtype
    return torch.einsum(subscripts, *[o.to(torch.float64) for o in operands]).to(out_dtype)
