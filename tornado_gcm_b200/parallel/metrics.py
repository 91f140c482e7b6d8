"""Cross-rank metric reduction: one packed all-reduce (reference
``distributed/ddp.py:369-409`` issues one collective and one host sync per
scalar)."""

from __future__ import annotations

import torch
import torch.distributed as dist


def all_reduce_metrics(metrics: dict, op: str = "mean") -> dict[str, float]:
    """Average (or max) scalar metrics over ranks with a single collective.

    Values may be python numbers or 0-d tensors; the result is a dict of
    python floats (one device→host copy in total).
    """
    if not metrics:
        return {}
    keys = list(metrics)
    vals = []
    device = None
    for k in keys:
        v = metrics[k]
        if torch.is_tensor(v):
            device = device or v.device
            vals.append(v.detach().float().reshape(()))
        else:
            vals.append(torch.tensor(float(v)))
    device = device or torch.device("cpu")
    packed = torch.stack([v.to(device) for v in vals])
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        backend = dist.get_backend()
        if backend == "nccl" and packed.device.type != "cuda":
            packed = packed.cuda()
        if backend == "gloo" and packed.device.type != "cpu":
            packed = packed.cpu()
        if op == "max":
            dist.all_reduce(packed, op=dist.ReduceOp.MAX)
        else:
            dist.all_reduce(packed, op=dist.ReduceOp.SUM)
            packed = packed / dist.get_world_size()
    host = packed.cpu().tolist()
    return dict(zip(keys, host))
