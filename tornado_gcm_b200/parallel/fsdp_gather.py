"""FSDP-style weight sharding with the all-gather fused into the consuming GEMM.

Each rank keeps only ``rows = ceil(O / W)`` rows (rounded up to 16) of a
linear layer's ``(O, K)`` BF16 weight, in symmetric memory.  The forward GEMM
(:func:`linear_fwd_gathered`, ``csrc/gemm.cu``) reads the weight directly
from the shards that own it — plain, non-multicast TMA loads from the peers'
memory over NVLink — so the full weight is never materialised and there is no
separate all-gather launch.  Every CTA of the persistent kernel owns one
64-row column block of the output and loads that block of the weight into
shared memory ONCE (up to K = 768), then streams its activation tiles; a
remote weight row therefore crosses NVLink once per CTA, not once per tile.  This is the reference's FSDP all-gather
(``distributed/ddp.py:245-361``, parameters gathered before each wrapped
unit) done inside the GEMM's producer warp.

:class:`GatheredLinear` wraps one layer (inference / forward);
:func:`shard_mlp` converts the linear layers of an :class:`~tornado_gcm_b200.neural.standard_layers.Mlp`.
The baseline for comparisons is ``all_gather_into_tensor`` + the ordinary
tcgen05 linear kernel (:func:`baseline_forward`).

    torchrun --nproc-per-node 2 -m tornado_gcm_b200.parallel.fsdp_gather --tokens 32768 --width 384
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
from typing import Optional

import torch
import torch.distributed as dist

from tornado_gcm_b200.ops import _ext
from tornado_gcm_b200.ops.linear import ACT_CODES as _ACT


# Crossover between reading the shards inside the GEMM and pulling them first, in
# GEMM rows x padded input width (2 x B200: the in-GEMM read wins at 8192 x 384,
# the pulled weight from 16384 x 384 and from 8192 x 768 on).
PULL_MIN_WORK = 16384 * 384


def _pad8(k: int) -> int:
    return (k + 7) // 8 * 8


class GatheredLinear:
    """``y = act(x W^T + b)`` with ``W`` row-sharded over the ranks in symmetric memory."""

    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor] = None, act: str = "none", group=None,
                 pad_out: bool = False):
        """``pad_out``: round the output width up to a multiple of 8 (zero weight rows), so that the
        BF16 output rows are 16-byte aligned for the next kernel; ``out_features`` stays the layer's."""
        import torch.distributed._symmetric_memory as symm_mem

        _ext.require("fused all-gather linear")
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > 8:
            raise ValueError("at most 8 shards")
        dev = weight.device
        self.out_features, K = weight.shape
        self.in_features = K
        if pad_out and self.out_features % 8:
            weight = torch.cat([weight, weight.new_zeros(_pad8(self.out_features) - self.out_features, K)], 0)
            if bias is not None:
                bias = torch.cat([bias, bias.new_zeros(_pad8(self.out_features) - self.out_features)], 0)
        self.O = weight.shape[0]
        self.Kp = _pad8(K)
        # shards of a multiple of 16 rows in rank order; trailing ranks may own no row
        self.rows = -(-self.O // self.world)
        self.rows = (self.rows + 15) // 16 * 16
        self.act = _ACT[act]
        shard = symm_mem.empty(self.rows * self.Kp, dtype=torch.bfloat16, device=dev)
        shard.zero_()
        r0 = self.rank * self.rows
        r1 = min(self.O, r0 + self.rows)
        if r1 > r0:
            shard.view(self.rows, self.Kp)[: r1 - r0, :K].copy_(weight[r0:r1].to(torch.bfloat16))
        h = symm_mem.rendezvous(shard, self.group.group_name)
        self.shard = shard
        self._handle = h
        self.w_ptrs = torch.tensor([int(p) for p in h.buffer_ptrs], dtype=torch.int64)
        self.bias = None if bias is None else bias.detach().float().contiguous().to(dev)
        # GEMM size (rows x Kp) from which the weight is pulled locally before the GEMM (see __call__)
        self.pull_min_work = int(os.environ.get("TGCM_GATHER_PULL_MIN_WORK", str(PULL_MIN_WORK)))
        torch.cuda.synchronize(dev)
        dist.barrier(group=self.group)

    def local_weight(self) -> torch.Tensor:
        return self.shard.view(self.rows, self.Kp)

    def local_rows(self) -> torch.Tensor:
        """This rank's rows of the (out_features, in_features) weight, without padding."""
        r0 = min(self.rank * self.rows, self.out_features)
        r1 = min(self.out_features, r0 + self.rows)
        return self.local_weight()[: r1 - r0, : self.in_features]

    def __call__(self, x: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """Dispatch on the GEMM's size: below ``pull_min_work`` (token rows x padded input
        width) the GEMM reads the shards in place (:meth:`fused_forward`); from it on the
        weight is pulled into this GPU's memory first (:meth:`pull_forward`), so that the
        128-row tiles of the ordinary kernel apply."""
        rows = x.numel() // x.shape[-1]
        if rows * self.Kp >= self.pull_min_work:
            return self.pull_forward(x, out_dtype)
        return self.fused_forward(x, out_dtype)

    def _rows_in(self, x: torch.Tensor) -> torch.Tensor:
        x = x.to(torch.bfloat16)
        if x.shape[-1] != self.Kp:
            x = torch.nn.functional.pad(x, (0, self.Kp - x.shape[-1]))
        return x.reshape(-1, self.Kp).contiguous()

    def fused_forward(self, x: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """The GEMM's producer warp loads every weight block from the rank that owns it."""
        ops = _ext.require("fused all-gather linear")
        x2 = self._rows_in(x)
        out = torch.empty(x2.shape[0], self.O, dtype=out_dtype, device=x2.device)
        ops.linear_fwd_gathered(x2, self.w_ptrs, self.rows, self.O, self.bias, self.act, out, None,
                                _ext.error_flag(x2.device))
        return out.reshape(x.shape[:-1] + (self.O,))

    def pull_forward(self, x: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """One copy kernel pulls every shard over NVLink (16-byte peer loads) into a transient
        local buffer, then the ordinary tcgen05 linear kernel runs: for large token counts the
        weight is reused by so many tiles that reading it once and locally wins."""
        ops = _ext.require("pulled all-gather linear")
        full = torch.empty(self.world * self.rows, self.Kp, dtype=torch.bfloat16, device=self.shard.device)
        ops.pull_peer_buffers(full, self.w_ptrs, self.rows * self.Kp * 2)
        x2 = self._rows_in(x)
        out = torch.empty(x2.shape[0], self.O, dtype=out_dtype, device=x2.device)
        ops.linear_fwd(x2, full[: self.O], self.bias, self.act, out, None, _ext.error_flag(x2.device))
        return out.reshape(x.shape[:-1] + (self.O,))

    def baseline_forward(self, x: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """NCCL all-gather of the shards, then the ordinary tcgen05 linear kernel."""
        ops = _ext.require("linear")
        full = torch.empty(self.world * self.rows, self.Kp, dtype=torch.bfloat16, device=self.shard.device)
        dist.all_gather_into_tensor(full, self.local_weight().contiguous(), group=self.group)
        x = x.to(torch.bfloat16)
        if x.shape[-1] != self.Kp:
            x = torch.nn.functional.pad(x, (0, self.Kp - x.shape[-1]))
        x2 = x.reshape(-1, self.Kp).contiguous()
        out = torch.empty(x2.shape[0], self.O, dtype=out_dtype, device=x2.device)
        ops.linear_fwd(x2, full[: self.O].contiguous(), self.bias, self.act, out, None, _ext.error_flag(x2.device))
        return out.reshape(x.shape[:-1] + (self.O,))


def shard_mlp(mlp, act: Optional[str] = None, group=None, pad_out: bool = True) -> list:
    """GatheredLinear for every layer of an Mlp (its own activations unless ``act`` is given)."""
    layers = list(mlp.layers)
    acts = mlp.layer_activations() if act is None else [act] * (len(layers) - 1) + ["none"]
    return [GatheredLinear(l.weight.detach(), l.bias.detach() if l.bias is not None else None,
                           acts[i] or "none", group, pad_out=pad_out) for i, l in enumerate(layers)]


def local_state_dict(layers: list, names: list, dtype: torch.dtype = torch.float32) -> tuple:
    """(this rank's weight rows, metadata) of sharded layers under their module names
    ``names[i] + ".weight"``, in the format of ``training/sharded_checkpoint`` (biases stay
    whole, on rank 0): a sharded tower is saved without any rank holding its full weights."""
    local, meta = {}, {}
    for lin, name in zip(layers, names):
        key = name + ".weight"
        local[key] = lin.local_rows().to(dtype).cpu()
        meta[key] = {"sharded": True, "shape": [lin.out_features, lin.in_features],
                     "dtype": str(dtype).replace("torch.", ""), "rows": lin.rows}
        if lin.bias is not None:
            bkey = name + ".bias"
            if lin.rank == 0:
                local[bkey] = lin.bias[: lin.out_features].to(dtype).cpu()
            meta[bkey] = {"sharded": False, "shape": [lin.out_features], "dtype": str(dtype).replace("torch.", "")}
    return local, meta


def gathered_mlp_forward(layers: list, x: torch.Tensor) -> torch.Tensor:
    """BF16 token rows through sharded layers; returns the last layer's padded BF16 rows."""
    h = x
    for lin in layers:
        h = lin(h)
    return h


def _time(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main(argv=None) -> None:  # pragma: no cover - needs several GPUs
    ap = argparse.ArgumentParser(description="fused all-gather linear vs NCCL all-gather + linear")
    ap.add_argument("--tokens", type=int, nargs="+", default=[8192, 16384, 32768])
    ap.add_argument("--width", type=int, nargs="+", default=[384, 768])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        for width in args.width:
            torch.manual_seed(0)
            w = (torch.randn(width, width, device="cuda") / width ** 0.5)
            b = torch.randn(width, device="cuda") * 0.1
            lin = GatheredLinear(w, b, "gelu_tanh")
            for T in args.tokens:
                x = torch.randn(T, width, device="cuda").to(torch.bfloat16)
                fused = _time(lambda: lin.fused_forward(x), args.iters, args.warmup)
                pull = _time(lambda: lin.pull_forward(x), args.iters, args.warmup)
                auto = _time(lambda: lin(x), args.iters, args.warmup)
                base = _time(lambda: lin.baseline_forward(x), args.iters, args.warmup)
                flops = 2.0 * T * width * width
                wbytes = 2.0 * width * width * (lin.world - 1) / lin.world
                ref = lin.baseline_forward(x).float()
                err = float((lin.fused_forward(x).float() - ref).abs().max())
                err_pull = float((lin.pull_forward(x).float() - ref).abs().max())
                if dist.get_rank() == 0:
                    print(json.dumps({"tokens": T, "width": width, "gpus": lin.world, "fused_ms": fused,
                                      "pull_ms": pull, "dispatch_ms": auto, "nccl_gather_ms": base,
                                      "dispatch_path": "pull" if T * lin.Kp >= lin.pull_min_work else "fused",
                                      "dispatch_tflops": flops / auto / 1e9, "remote_weight_bytes": wbytes,
                                      "max_abs_diff": err, "max_abs_diff_pull": err_pull}), flush=True)
    finally:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
