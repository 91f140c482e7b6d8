"""Sharded checkpoints for row-sharded (FSDP-style) weights: save per rank, gather.

A row-sharded parameter keeps rows ``[r·R, (r+1)·R)`` of its full tensor on
rank ``r`` (``R`` rows per rank, recorded per tensor: ``ceil(rows / W)``
rounded up to a multiple of 16 by default; the last ranks may hold fewer or
no rows) — the layout of the fused all-gather linear layers
(``parallel/fsdp_gather.GatheredLinear``).  This module

* splits a full state dict into the rank's shards (:func:`shard_state_dict`),
* writes one file per rank plus a metadata file (:func:`save_sharded`) — no
  rank ever holds the full model,
* assembles the full state dict again, either offline from the files
  (:func:`gather_sharded`, e.g. to export the reference's single-file ``.pt``
  checkpoint) or online over a process group (:func:`all_gather_state_dict`),
* loads a full checkpoint into a sharded model (each rank slices its rows).

Reference ``training/checkpointing.py:20-95`` defines the single-file format
kept here; the reference wraps torch FSDP (``distributed/ddp.py:245-361``)
without a sharded save path.
"""

from __future__ import annotations

import json
import os
import pathlib
from typing import Callable, Dict, Iterable, Optional

import torch
import torch.distributed as dist

from tornado_gcm_b200.training.checkpointing import _atomic_save

META_NAME = "shards.json"


def shard_rows(n_rows: int, world: int, row_multiple: int = 16) -> int:
    """Rows per rank for ``n_rows`` split over ``world`` ranks."""
    per = -(-n_rows // world)
    return -(-per // row_multiple) * row_multiple


def row_range(n_rows: int, rank: int, per: int) -> tuple:
    """Rows of ``rank`` when every rank holds ``per`` rows (the last ones may hold fewer)."""
    lo = min(rank * per, n_rows)
    return lo, min(lo + per, n_rows)


def default_sharded(name: str, t: torch.Tensor) -> bool:
    """Matrices (weights of linear layers) are sharded; vectors and buffers stay whole."""
    return t.dim() >= 2 and name.endswith("weight")


def shard_state_dict(sd: Dict[str, torch.Tensor], rank: int, world: int,
                     is_sharded: Callable[[str, torch.Tensor], bool] = default_sharded,
                     row_multiple: int = 16) -> tuple:
    """(local state dict, metadata) of ``rank``: sharded tensors cut to the rank's rows,
    replicated ones kept whole on rank 0 only."""
    local, meta = {}, {}
    for k, v in sd.items():
        if is_sharded(k, v):
            per = shard_rows(v.shape[0], world, row_multiple)
            lo, hi = row_range(v.shape[0], rank, per)
            local[k] = v[lo:hi].detach().clone()
            meta[k] = {"sharded": True, "shape": list(v.shape), "dtype": str(v.dtype).replace("torch.", ""),
                       "rows": per}
        else:
            if rank == 0:
                local[k] = v.detach().clone()
            meta[k] = {"sharded": False, "shape": list(v.shape), "dtype": str(v.dtype).replace("torch.", "")}
    return local, meta


def _shard_path(directory: pathlib.Path, rank: int) -> pathlib.Path:
    return directory / f"shard_{rank:05d}.pt"


def save_sharded(directory, local_sd: Dict[str, torch.Tensor], meta: dict, rank: int, world: int,
                 extra: Optional[dict] = None) -> None:
    """Write this rank's shard file; rank 0 also writes the metadata (world, rows per rank, shapes)."""
    d = pathlib.Path(directory)
    _atomic_save({"rank": rank, "world": world, "state": {k: v.cpu() for k, v in local_sd.items()}},
                 _shard_path(d, rank))
    if rank == 0:
        doc = {"world": world, "tensors": meta, "extra": extra or {}}
        d.mkdir(parents=True, exist_ok=True)
        tmp = d / (META_NAME + ".tmp")
        tmp.write_text(json.dumps(doc, indent=1))
        os.replace(tmp, d / META_NAME)


def gather_sharded(directory) -> Dict[str, torch.Tensor]:
    """Full state dict assembled from the files of :func:`save_sharded` (one process)."""
    d = pathlib.Path(directory)
    doc = json.loads((d / META_NAME).read_text())
    world = int(doc["world"])
    shards = [torch.load(_shard_path(d, r), map_location="cpu", weights_only=True)["state"] for r in range(world)]
    full = {}
    for k, m in doc["tensors"].items():
        if m["sharded"]:
            parts = []
            for r in range(world):
                lo, hi = row_range(m["shape"][0], r, int(m["rows"]))
                if hi > lo:
                    parts.append(shards[r][k])
            full[k] = torch.cat(parts, dim=0)
            if list(full[k].shape) != m["shape"]:
                raise ValueError(f"gathered {k} has shape {list(full[k].shape)}, expected {m['shape']}")
        else:
            full[k] = shards[0][k]
    return full


def all_gather_state_dict(local_sd: Dict[str, torch.Tensor], meta: dict, group=None,
                          keys: Optional[Iterable[str]] = None) -> Dict[str, torch.Tensor]:
    """Full state dict on every rank of ``group`` from the ranks' shards (collectives:
    one all-gather per sharded tensor, one broadcast per replicated one)."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    src0 = dist.get_global_rank(group, 0) if (dist.is_initialized() and group is not None) else 0
    full = {}
    for k in (keys if keys is not None else meta.keys()):
        m = meta[k]
        shape = m["shape"]
        dtype = getattr(torch, m["dtype"])
        dev = next(iter(local_sd.values())).device if local_sd else torch.device("cpu")
        if m["sharded"]:
            per = int(m["rows"])
            mine = local_sd[k]
            buf = torch.zeros((per,) + tuple(shape[1:]), dtype=dtype, device=dev)
            buf[: mine.shape[0]] = mine
            parts = [torch.empty_like(buf) for _ in range(world)]
            if world > 1:
                dist.all_gather(parts, buf, group=group)
            else:
                parts = [buf]
            full[k] = torch.cat(parts, dim=0)[: shape[0]].contiguous()
        else:
            t = local_sd[k].to(dev) if rank == 0 else torch.empty(shape, dtype=dtype, device=dev)
            if world > 1:
                dist.broadcast(t, src=src0, group=group)
            full[k] = t
    return full


def load_full_into_shards(full_sd: Dict[str, torch.Tensor], meta: dict, rank: int) -> Dict[str, torch.Tensor]:
    """This rank's shards of a full state dict (e.g. a reference single-file checkpoint)."""
    out = {}
    for k, m in meta.items():
        v = full_sd[k]
        if m["sharded"]:
            lo, hi = row_range(v.shape[0], rank, int(m["rows"]))
            out[k] = v[lo:hi].clone()
        else:
            out[k] = v.clone()
    return out
