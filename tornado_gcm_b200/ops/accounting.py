"""Algorithmic bytes and FLOPs of the native ops, for step-level rooflines.

While :func:`counting` is active, :func:`tornado_gcm_b200.ops._ext.require`
hands out a proxy of ``torch.ops.tgcm`` that records, per op name, the
number of calls, the bytes of every tensor argument and result (each tensor
read or written once: the traffic of an ideal kernel with that interface),
and for the GEMM-shaped ops the arithmetic (2·M·N·K, triangular Legendre
sums counted exactly) by precision class.  Run one eager step under it and
compare the totals with the measured HBM bandwidth and tensor-core peaks::

    with accounting.counting() as acc:
        step()
    print(accounting.summary(acc, hbm_gbs=6554.6, bf16_tflops=1690.5))

A CUDA-graph replay launches the captured kernels without calling the ops,
so the step has to run eagerly while counting.
"""

from __future__ import annotations

import contextlib
from typing import Dict, Optional

import torch

_ACTIVE: Optional[dict] = None


def active() -> Optional[dict]:
    return _ACTIVE


@contextlib.contextmanager
def counting():
    """Record the ops called inside the block; yields the per-op table."""
    global _ACTIVE
    prev = _ACTIVE
    table: Dict[str, dict] = {}
    _ACTIVE = table
    try:
        yield table
    finally:
        _ACTIVE = prev


def _device_bytes(x) -> int:
    """Bytes of device tensors only (host-side tables such as peer pointer lists are not traffic)."""
    if isinstance(x, torch.Tensor):
        return x.numel() * x.element_size() if x.is_cuda else 0
    if isinstance(x, (list, tuple)):
        return sum(_device_bytes(v) for v in x)
    return 0


def _tri(L: int, Mw: int) -> int:
    """Σ_{m < Mw} max(L - m, 0): Legendre coefficients per (cos or sin) row pair."""
    return sum(max(L - m, 0) for m in range(Mw))


def _flops(name: str, args) -> tuple:
    """(flops, precision class) of a GEMM-shaped op, or (0, None)."""
    try:
        if name == "linear_fwd":
            X, W = args[0], args[1]
            return 2 * X.shape[0] * X.shape[1] * W.shape[0], "bf16"
        if name == "linear_fwd_gathered":
            X, O = args[0], int(args[3])
            return 2 * X.shape[0] * X.shape[1] * O, "bf16"
        if name in ("linear_dgrad", "linear_wgrad"):
            dY, other = args[0], args[1]
            return 2 * dY.shape[0] * dY.shape[1] * other.shape[1], "bf16"
        if name == "bgemm_tf32":
            A, B = args[0], args[1]
            return 2 * A.shape[0] * A.shape[1] * A.shape[2] * B.shape[1], "tf32"
        if name == "dgemm_strided":
            M, N, K, G = (int(a) for a in args[3:7])
            return 2 * M * N * K * G, "fp64"
        if name == "sht_synth":
            x, L, P, F = args[0], int(args[1]), args[2], args[3]
            S = x.shape[0]
            Mw, J = P.shape[0], P.shape[1]
            I, M2 = F.shape[0], 2 * Mw - 1
            return 2 * S * J * (2 * _tri(L, Mw)) + 2 * S * J * I * M2, "tf32"
        if name == "sht_anal":
            N, Ft, Pt, Lo = args[0], args[1], args[2], int(args[3])
            S = N.shape[0]
            Mw = Pt.shape[0]
            J = N.shape[1] if args[7] else N.shape[2]
            I = N.shape[2] if args[7] else N.shape[1]
            M2 = 2 * Mw - 1
            return 2 * S * J * I * M2 + 2 * S * J * (2 * _tri(Lo, Mw)), "tf32"
        if name == "column_attention_fwd":
            q, k = args[0], args[1]
            return 4 * q.shape[0] * q.shape[1] * k.shape[1] * q.shape[2], "fp32"
        if name == "column_attention_bwd":
            q, k = args[0], args[1]
            return 8 * q.shape[0] * q.shape[1] * k.shape[1] * q.shape[2], "fp32"
    except (AttributeError, IndexError, TypeError, ValueError):
        pass
    return 0, None


def record(name: str, args, kwargs, result) -> None:
    table = _ACTIVE
    if table is None:
        return
    row = table.setdefault(name, {"calls": 0, "bytes": 0, "flops": 0, "cls": None})
    row["calls"] += 1
    row["bytes"] += _device_bytes(list(args) + list(kwargs.values())) + _device_bytes(result)
    fl, cls = _flops(name, args)
    if fl:
        row["flops"] += fl
        row["cls"] = cls


class CountingOps:
    """Attribute-compatible stand-in for ``torch.ops.tgcm`` that records each call."""

    def __init__(self, ops):
        self._ops = ops

    def __getattr__(self, name):
        fn = getattr(self._ops, name)
        if not callable(fn):
            return fn

        def call(*args, **kwargs):
            out = fn(*args, **kwargs)
            record(name, args, kwargs, out)
            return out

        return call


def summary(table: dict, hbm_gbs: float, bf16_tflops: float, tf32_tflops: Optional[float] = None,
            fp64_tflops: float = 40.0, fp32_tflops: float = 80.0) -> dict:
    """Totals and the roofline time of the recorded ops.

    ``tf32_tflops`` defaults to half the BF16 rate (the tensor-core TF32 rate
    is half the BF16 one); ``fp64_tflops`` is the nominal FP64 tensor rate and
    ``fp32_tflops`` the nominal CUDA-core FP32 rate.  Eager framework ops (adds,
    copies, fills) are not counted: their traffic is overhead, not part of the
    minimum.
    """
    tf32 = tf32_tflops if tf32_tflops is not None else bf16_tflops / 2
    rate = {"bf16": bf16_tflops, "tf32": tf32, "fp64": fp64_tflops, "fp32": fp32_tflops}
    total_bytes = sum(r["bytes"] for r in table.values())
    flops = {}
    for r in table.values():
        if r["flops"]:
            flops[r["cls"]] = flops.get(r["cls"], 0) + r["flops"]
    t_hbm = total_bytes / (hbm_gbs * 1e9) * 1e3
    t_flop = sum(f / (rate[c] * 1e12) * 1e3 for c, f in flops.items())
    return {
        "calls": sum(r["calls"] for r in table.values()),
        "alg_bytes_gb": total_bytes / 1e9,
        "tflop": {c: f / 1e12 for c, f in flops.items()},
        "t_hbm_ms": t_hbm,
        "t_flop_ms": t_flop,
        "roofline_ms": max(t_hbm, t_flop),
    }


def table_lines(table: dict, hbm_gbs: float) -> list:
    """Per-op rows (largest traffic first): calls, GB, ms at the HBM rate, GFLOP and class."""
    rows = sorted(table.items(), key=lambda kv: -kv[1]["bytes"])
    out = ["op  calls  GB  ms_at_hbm  GFLOP  class"]
    for name, r in rows:
        out.append(f"{name}  {r['calls']}  {r['bytes'] / 1e9:.3f}  {r['bytes'] / (hbm_gbs * 1e6):.3f}  "
                   f"{r['flops'] / 1e9:.1f}  {r['cls'] or '-'}")
    return out
