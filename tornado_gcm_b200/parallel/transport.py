"""Communication backends behind one interface: NVLink peer memory, NCCL, gloo.

Every multi-rank component of the framework asks a :class:`Transport` for
what it needs instead of calling a library directly:

* ``all_reduce_sum`` / ``all_gather`` / ``barrier`` — the plain collectives
  (metrics, host-side checks, the sharded fixer's partial sums);
* ``gradient_reducer(numel, device)`` — the object that averages (or sums) a
  flat gradient buffer after backward;
* ``spectral_engine(layout)`` — the transform engine of the model sharded
  over wavenumbers and latitudes.

Three transports implement it:

* :class:`NVLinkTransport` — symmetric memory (``torch.distributed.
  _symmetric_memory``) and this framework's kernels: the one-launch fused
  gradient all-reduce (``csrc/comm.cu``), the routed Legendre epilogues of
  the sharded transforms with the bounded peer barrier.  Plain peer loads,
  stores and reductions only (no multicast objects are used);
* :class:`NcclTransport` — ``torch.distributed`` over NCCL (the baseline the
  fused paths are measured against);
* :class:`GlooTransport` — CPU ranks (tests of the host-side logic).

:func:`get_transport` picks one: ``auto`` = NVLink on CUDA when the
extension is loaded and the group spans one node, NCCL on CUDA otherwise,
gloo on the CPU; the environment variable ``TGCM_TRANSPORT`` overrides it.
"""

from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist


class Transport:
    name = "base"

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0

    # ── plain collectives ──
    def all_reduce_sum(self, t: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        return t

    def all_gather(self, t: torch.Tensor) -> list:
        if self.world == 1:
            return [t]
        parts = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(parts, t.contiguous(), group=self.group)
        return parts

    def barrier(self) -> None:
        if self.world > 1:
            dist.barrier(group=self.group)

    # ── component factories ──
    def gradient_reducer(self, numel: int, device):
        """Reducer of a flat fp32 gradient buffer: ``.flat`` plus ``all_reduce_mean/sum(flat)``."""
        return _CollectiveReducer(numel, device, self)

    def spectral_engine(self, layout):
        from tornado_gcm_b200.parallel.spectral_shard import CollectiveTransforms

        return CollectiveTransforms(layout, self.group)


class _CollectiveReducer:
    def __init__(self, numel: int, device, transport: Transport):
        self.flat = torch.zeros(numel, dtype=torch.float32, device=device)
        self.t = transport

    def all_reduce_sum(self, flat: torch.Tensor) -> None:
        self.t.all_reduce_sum(flat)

    def all_reduce_mean(self, flat: torch.Tensor) -> None:
        self.t.all_reduce_sum(flat)
        flat.mul_(1.0 / self.t.world)


class NcclTransport(Transport):
    name = "nccl"


class GlooTransport(Transport):
    name = "gloo"


class NVLinkTransport(Transport):
    """Peer memory over NVLink / NVSwitch with this framework's kernels."""

    name = "nvlink"

    def gradient_reducer(self, numel: int, device):
        from tornado_gcm_b200.parallel import fused_allreduce

        return fused_allreduce.make_reducer(numel, torch.device(device), self.group)

    def spectral_engine(self, layout):
        from tornado_gcm_b200.parallel.spectral_shard import FusedTransforms

        return FusedTransforms(layout, self.group)


_KINDS = {"nvlink": NVLinkTransport, "nccl": NcclTransport, "gloo": GlooTransport}


def get_transport(kind: str = "auto", group=None, device=None) -> Transport:
    """The transport for ``group`` on ``device`` (see the module docstring)."""
    kind = os.environ.get("TGCM_TRANSPORT", kind) if kind == "auto" else kind
    if kind == "auto":
        dev = torch.device(device) if device is not None else None
        if dev is not None and dev.type == "cuda":
            from tornado_gcm_b200.ops import _ext

            kind = "nvlink" if _ext.available() and _single_node(group) else "nccl"
        else:
            kind = "gloo"
    if kind not in _KINDS:
        raise ValueError(f"unknown transport {kind!r}; known: {sorted(_KINDS)}")
    return _KINDS[kind](group)


def _single_node(group) -> bool:
    """All ranks of ``group`` on this node (peer memory needs NVLink reachability)."""
    if not dist.is_initialized():
        return True
    local = int(os.environ.get("LOCAL_WORLD_SIZE", "0") or 0)
    return local == 0 or dist.get_world_size(group) <= local


def describe(t: Optional[Transport]) -> str:
    return "none" if t is None else f"{t.name} ({t.world} ranks)"
