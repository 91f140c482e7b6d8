"""Zone-named trace ranges and a JSON-lines throughput log.

``zone_range(name)`` opens a ``torch.profiler.record_function`` range and,
when ``TGCM_NVTX=1`` (or :func:`enable_nvtx`), an NVTX range with the same
name, so the PZHA zones (``Z3_neural_net``, ``Z1_dycore``, ``Z0_spectral``,
``Z2_physics_bridge``) show up in the PyTorch profiler and in Nsight tools.
NVTX ranges are host-side markers: inside a captured CUDA graph they cover
the capture, not the replays.

:class:`ThroughputLog` appends one JSON object per line (step, device-timed
milliseconds as the max over ranks, samples/s and extra fields).
"""

from __future__ import annotations

import contextlib
import json
import os
import time
from typing import Optional

import torch
from torch.profiler import record_function

_NVTX = os.environ.get("TGCM_NVTX", "0") not in ("", "0")


def enable_nvtx(on: bool = True) -> None:
    global _NVTX
    _NVTX = bool(on)


def nvtx_enabled() -> bool:
    return _NVTX


@contextlib.contextmanager
def zone_range(name: str):
    use_nvtx = _NVTX and torch.cuda.is_available()
    if use_nvtx:
        torch.cuda.nvtx.range_push(name)
    try:
        with record_function(name):
            yield
    finally:
        if use_nvtx:
            torch.cuda.nvtx.range_pop()


class ThroughputLog:
    """Append-only JSON-lines log of step timings (rank 0 writes)."""

    def __init__(self, path: str, rank: int = 0):
        self.path = path
        self.rank = rank

    def record(self, step: int, ms_per_step: float, samples: Optional[float] = None, **extra) -> dict:
        rec = {"step": int(step), "ms_per_step": float(ms_per_step), "time": time.time()}
        if samples is not None and ms_per_step > 0:
            rec["samples_per_s"] = float(samples) * 1000.0 / float(ms_per_step)
        rec.update(extra)
        if self.rank == 0:
            d = os.path.dirname(os.path.abspath(self.path))
            os.makedirs(d, exist_ok=True)
            with open(self.path, "a", encoding="utf-8") as f:
                f.write(json.dumps(rec) + "\n")
        return rec


def device_time_max_over_ranks(ms: float, device=None) -> float:
    """Max of a per-rank device time over the default process group (identity without one)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(ms)
    dev = device if device is not None else (torch.device("cuda", torch.cuda.current_device())
                                             if dist.get_backend() == "nccl" else torch.device("cpu"))
    t = torch.tensor([float(ms)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
