"""Fused mean all-reduce of the flat gradient buffer over NVLink peer memory.

The buffer and a small signal area are allocated in symmetric memory
(``torch.distributed._symmetric_memory``): after a one-time rendezvous every
rank holds device pointers to all peers' copies.  One sm_100a kernel
(``csrc/comm.cu``) then performs the whole mean all-reduce — barrier,
reduce-scatter with the 1/W scaling fused, all-gather by pushing into peer
memory, barrier — with plain peer loads/stores and bounded waits.  It is a
single graph-capturable launch with no NCCL call.

This replaces the bucketed NCCL all-reduce of reference
``distributed/ddp.py:203-237`` (DDP ``bucket_cap_mb=25``) for the gradients
of :class:`~tornado_gcm_b200.training.trainer.GCMTrainer`.
"""

from __future__ import annotations

import logging

import torch
import torch.distributed as dist

from tornado_gcm_b200.ops import _ext

logger = logging.getLogger(__name__)

_MAX_RANKS = 8


def _blocks_for(numel: int, world: int) -> int:
    per_rank = (numel + world - 1) // world
    return int(max(1, min(128, (per_rank + 4095) // 4096)))


class FusedMeanAllReducer:
    """Owns a symmetric flat fp32 buffer and reduces it in place."""

    def __init__(self, numel: int, device: torch.device, group=None):
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > _MAX_RANKS:
            raise ValueError(f"fused all-reduce supports up to {_MAX_RANKS} ranks")
        self.blocks = _blocks_for(numel, self.world)
        self.flat = symm_mem.empty(numel, dtype=torch.float32, device=device)
        self.flat.zero_()
        self.pads = symm_mem.empty(2 * _MAX_RANKS * self.blocks, dtype=torch.int32, device=device)
        self.pads.zero_()
        gname = self.group.group_name
        h_buf = symm_mem.rendezvous(self.flat, gname)
        h_pad = symm_mem.rendezvous(self.pads, gname)
        self.buf_ptrs = torch.tensor([int(p) for p in h_buf.buffer_ptrs], dtype=torch.int64)
        self.pad_ptrs = torch.tensor([int(p) for p in h_pad.buffer_ptrs], dtype=torch.int64)
        self._handles = (h_buf, h_pad)
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)

    def all_reduce_mean(self, flat: torch.Tensor) -> None:
        if flat.data_ptr() != self.flat.data_ptr():
            raise ValueError("all_reduce_mean works on the reducer's own symmetric buffer")
        ops = _ext.require("fused all-reduce")
        ops.fused_allreduce_mean(self.flat, self.buf_ptrs, self.pad_ptrs, self.rank, self.blocks,
                                 _ext.error_flag(self.flat.device))

    def all_reduce_sum(self, flat: torch.Tensor) -> None:
        """Same kernel with the scale set to 1 (plain sum over ranks)."""
        if flat.data_ptr() != self.flat.data_ptr():
            raise ValueError("all_reduce_sum works on the reducer's own symmetric buffer")
        ops = _ext.require("fused all-reduce")
        ops.fused_allreduce_mean(self.flat, self.buf_ptrs, self.pad_ptrs, self.rank, self.blocks,
                                 _ext.error_flag(self.flat.device), 1.0)


def make_reducer(numel: int, device: torch.device, group=None) -> FusedMeanAllReducer:
    """Symmetric-memory reducer for a flat buffer of ``numel`` fp32 elements."""
    if not torch.cuda.is_available() or not _ext.available():
        raise RuntimeError("fused all-reduce needs CUDA and the extension")
    return FusedMeanAllReducer(numel, device, group)


def _bench_main() -> None:  # pragma: no cover - needs several GPUs
    """``torchrun --nproc-per-node N -m tornado_gcm_b200.parallel.fused_allreduce [--mb 4.8]``.

    Checks the fused mean all-reduce against NCCL and times both (CUDA events,
    max over ranks).  Prints one JSON line on rank 0.
    """
    import argparse
    import datetime
    import json
    import os

    ap = argparse.ArgumentParser()
    ap.add_argument("--mb", type=float, default=4.8)
    ap.add_argument("--iters", type=int, default=50)
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    n = int(args.mb * 1e6 / 4) // 4 * 4
    red = make_reducer(n, dev)
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    errs = []
    for it in range(3):
        src = torch.randn(n, device=dev, generator=g)
        ref = src.clone()
        dist.all_reduce(ref)
        ref /= world
        red.flat.copy_(src)
        red.all_reduce_mean(red.flat)
        torch.cuda.synchronize()
        errs.append(float((red.flat - ref).abs().max()))
    flag = int(_ext.error_flag(dev).item())

    def timed(fn):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b) / args.iters], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    buf = torch.randn(n, device=dev)
    t_fused = timed(lambda: red.all_reduce_mean(red.flat))
    t_nccl = timed(lambda: dist.all_reduce(buf))
    bytes_bus = 2.0 * (world - 1) / world * n * 4
    if rank == 0:
        print(json.dumps({"case": "fused_allreduce_mean", "world": world, "mb": n * 4 / 1e6,
                          "max_abs_err_vs_nccl": max(errs), "error_flag": flag,
                          "fused_ms": t_fused, "nccl_ms": t_nccl,
                          "fused_busbw_gbs": bytes_bus / (t_fused * 1e-3) / 1e9,
                          "nccl_busbw_gbs": bytes_bus / (t_nccl * 1e-3) / 1e9}), flush=True)
    del red
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    _bench_main()
