"""Sharded data parallelism for rollout training: gradients and AdamW state split over the ranks.

This is the framework's FSDP training path (reference ``distributed/ddp.py:245-361``,
``wrap_fsdp`` with ``FULL_SHARD``), laid out for backprop-through-rollout:

* every parameter of the model is a view of ONE flat fp32 buffer ``P`` and its
  ``.grad`` a view of one flat fp32 buffer ``G`` (both padded to a multiple of
  ``4 * world`` elements); chunk ``r`` of the flat buffers belongs to rank ``r``;
* backward accumulates the full local gradient in ``G`` (a tower weight is used
  at every physics step, so its gradient is complete only when backward has
  gone through the first step: there is nothing to reduce earlier);
* :meth:`ShardedAdamW.step` then (1) reduce-scatters ``G``: rank ``r`` ends with the
  mean over ranks of chunk ``r``; (2) clips by the global gradient norm (the
  squared norms of the chunks summed over ranks); (3) runs fused AdamW on chunk
  ``r`` of ``P`` only, so the two moment buffers are ``1/world`` of the model;
  (4) all-gathers ``P`` so that every rank holds the updated weights for the
  next rollout.

The parameters stay gathered while a step runs, as in FSDP's ``SHARD_GRAD_OP``
strategy: a rollout applies every weight dozens of times per step, and
``FULL_SHARD``'s gather before each use (and again in backward) would move the
weights over NVLink once per physics step instead of once per optimizer step.

On NVLink (the ``nvlink`` transport) ``P``, ``G`` and a signal pad live in
symmetric memory and the two collectives are this framework's kernels
(``csrc/comm.cu``: ``fused_reduce_scatter`` and ``fused_all_gather``, plain
16-byte peer loads, bounded barriers, one launch each, graph-capturable).  With
NCCL or gloo the same steps run as ``reduce_scatter_tensor`` and
``all_gather_into_tensor`` on the chunks.
"""

from __future__ import annotations

from typing import Optional, Sequence

import torch
import torch.distributed as dist

_MAX_RANKS = 8


def _blocks_for(chunk: int) -> int:
    return int(max(1, min(128, (chunk + 4095) // 4096)))


class _FusedChunkComm:
    """Symmetric P and G buffers with the fused reduce-scatter / all-gather kernels."""

    kind = "fused NVLink peer-memory kernels (csrc/comm.cu)"

    def __init__(self, numel: int, device: torch.device, group):
        import torch.distributed._symmetric_memory as symm_mem

        from tornado_gcm_b200.ops import _ext
        from tornado_gcm_b200.parallel.fused_allreduce import make_reducer

        self._ext = _ext
        self.ops = _ext.require("sharded optimizer collectives")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _MAX_RANKS:
            raise ValueError(f"at most {_MAX_RANKS} ranks")
        self.blocks = _blocks_for(numel // self.world)
        self.P = symm_mem.empty(numel, dtype=torch.float32, device=device)
        self.G = symm_mem.empty(numel, dtype=torch.float32, device=device)
        self.pads = symm_mem.empty(2 * _MAX_RANKS * self.blocks, dtype=torch.int32, device=device)
        self.P.zero_()
        self.G.zero_()
        self.pads.zero_()
        gname = group.group_name
        hp = symm_mem.rendezvous(self.P, gname)
        hg = symm_mem.rendezvous(self.G, gname)
        hs = symm_mem.rendezvous(self.pads, gname)
        self.p_ptrs = torch.tensor([int(x) for x in hp.buffer_ptrs], dtype=torch.int64)
        self.g_ptrs = torch.tensor([int(x) for x in hg.buffer_ptrs], dtype=torch.int64)
        self.pad_ptrs = torch.tensor([int(x) for x in hs.buffer_ptrs], dtype=torch.int64)
        self._handles = (hp, hg, hs)
        # a separate small reducer sums the per-rank squared gradient norms
        self.norm_red = make_reducer(4 * self.world, device, group)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)

    def reduce_scatter_mean(self) -> None:
        self.ops.fused_reduce_scatter(self.G, self.g_ptrs, self.pad_ptrs, self.rank, self.blocks,
                                      self._ext.error_flag(self.G.device), 0.0)

    def all_gather_params(self) -> None:
        self.ops.fused_all_gather(self.P, self.p_ptrs, self.pad_ptrs, self.rank, self.blocks,
                                  self._ext.error_flag(self.P.device))

    def sum_scalar(self, x: torch.Tensor) -> torch.Tensor:
        buf = self.norm_red.flat
        buf.zero_()
        buf[:1].copy_(x.reshape(1))
        self.norm_red.all_reduce_sum(buf)
        return buf[0]


class _CollectiveChunkComm:
    """The same steps on ``torch.distributed`` collectives (NCCL on CUDA, gloo on the CPU)."""

    def __init__(self, numel: int, device: torch.device, group):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.P = torch.zeros(numel, dtype=torch.float32, device=device)
        self.G = torch.zeros(numel, dtype=torch.float32, device=device)
        self.chunk = numel // self.world
        self._tmp = torch.empty(self.chunk, dtype=torch.float32, device=device)
        self._scalar = torch.zeros(1, dtype=torch.float32, device=device)
        self.kind = "nccl" if device.type == "cuda" else (dist.get_backend(group) if dist.is_initialized() else "none")

    def _own(self, t: torch.Tensor) -> torch.Tensor:
        return t[self.rank * self.chunk:(self.rank + 1) * self.chunk]

    def reduce_scatter_mean(self) -> None:
        if self.world > 1:
            dist.reduce_scatter_tensor(self._tmp, self.G, group=self.group)
            self._own(self.G).copy_(self._tmp).mul_(1.0 / self.world)

    def all_gather_params(self) -> None:
        if self.world > 1:
            self._tmp.copy_(self._own(self.P))
            dist.all_gather_into_tensor(self.P, self._tmp, group=self.group)

    def sum_scalar(self, x: torch.Tensor) -> torch.Tensor:
        self._scalar.copy_(x.reshape(1))
        if self.world > 1:
            dist.all_reduce(self._scalar, group=self.group)
        return self._scalar[0]


class ShardedAdamW:
    """AdamW whose gradients and moments are sharded over the ranks (see the module docstring).

    Typical use (what :class:`~tornado_gcm_b200.training.trainer.GCMTrainer` does with
    ``data_parallel="sharded"``)::

        opt = ShardedAdamW(model.parameters(), lr=1e-4)
        opt.zero_grad()              # G = 0, .grad views attached
        loss.backward()              # full local gradients accumulate in G
        opt.step()                   # reduce-scatter, clip, AdamW on own chunk, all-gather
    """

    def __init__(self, params: Sequence[torch.nn.Parameter], lr: float = 1e-4, weight_decay: float = 0.0,
                 betas=(0.9, 0.95), eps: float = 1e-6, max_grad_norm: Optional[float] = 1.0,
                 capturable: bool = False, group=None, transport: str = "auto"):
        self.params = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("no trainable parameters")
        if any(p.dtype != torch.float32 for p in self.params):
            raise ValueError("the sharded optimizer keeps fp32 master weights: pass fp32 parameters")
        dev = self.params[0].device
        self.device = dev
        self.group = group or (dist.group.WORLD if dist.is_initialized() else None)
        self.world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        n = sum(p.numel() for p in self.params)
        q = 4 * self.world
        self.numel = n
        self.numel_padded = (n + q - 1) // q * q
        self.chunk = self.numel_padded // self.world
        self.comm = self._make_comm(transport, dev)
        self.backend = self.comm.kind if self.world > 1 else "none (one rank)"
        P, G = self.comm.P, self.comm.G
        # every rank starts from rank 0's weights
        off = 0
        with torch.no_grad():
            for p in self.params:
                P[off:off + p.numel()].copy_(p.detach().reshape(-1).float())
                off += p.numel()
            if self.world > 1:
                dist.broadcast(P, src=0, group=self.group)
        self._views_p, self._views_g = [], []
        off = 0
        for p in self.params:
            k = p.numel()
            self._views_p.append(P[off:off + k].view_as(p))
            self._views_g.append(G[off:off + k].view_as(p))
            off += k
        for p, v in zip(self.params, self._views_p):
            p.data = v
        c0 = self.rank * self.chunk
        self.shard = torch.nn.Parameter(P[c0:c0 + self.chunk], requires_grad=True)
        self.shard.grad = G[c0:c0 + self.chunk]
        self.max_grad_norm = max_grad_norm
        self.optimizer = torch.optim.AdamW([self.shard], lr=lr, weight_decay=weight_decay, betas=betas, eps=eps,
                                           fused=dev.type == "cuda", capturable=capturable and dev.type == "cuda")

    def _make_comm(self, transport: str, dev: torch.device):
        from tornado_gcm_b200.parallel.transport import get_transport

        if self.world == 1:
            return _CollectiveChunkComm(self.numel_padded, dev, self.group)
        t = get_transport(transport, group=self.group, device=dev)
        if t.name == "nvlink":
            return _FusedChunkComm(self.numel_padded, dev, self.group)
        return _CollectiveChunkComm(self.numel_padded, dev, self.group)

    @property
    def flat_grad(self) -> torch.Tensor:
        return self.comm.G

    @property
    def flat_params(self) -> torch.Tensor:
        return self.comm.P

    @property
    def param_groups(self):
        return self.optimizer.param_groups

    def attach(self) -> None:
        """Point every parameter's ``.grad`` at its view of the flat gradient buffer."""
        for p, v in zip(self.params, self._views_g):
            if p.grad is None or p.grad.data_ptr() != v.data_ptr():
                p.grad = v
        self.shard.grad = self.comm.G[self.rank * self.chunk:(self.rank + 1) * self.chunk]

    def zero_grad(self, set_to_none: bool = False) -> None:  # noqa: ARG002 - the views are kept
        self.comm.G.zero_()
        self.attach()

    def clip_shard(self) -> torch.Tensor:
        """Scale the own gradient chunk by min(1, max_norm / global_norm); returns the global norm."""
        g = self.shard.grad
        total = self.comm.sum_scalar(torch.sum(g * g)).sqrt()
        if self.max_grad_norm is not None:
            coef = torch.clamp(self.max_grad_norm / (total + 1e-6), max=1.0)
            g.mul_(coef)
        return total

    def step(self) -> torch.Tensor:
        """Reduce-scatter, clip, AdamW on the own chunk, all-gather; returns the global grad norm."""
        for p, v in zip(self.params, self._views_g):
            if p.grad is not None and p.grad.data_ptr() != v.data_ptr():
                v.add_(p.grad)  # autograd replaced a view (a .grad that was None)
                p.grad = v
        self.comm.reduce_scatter_mean()
        total = self.clip_shard()
        self.optimizer.step()
        self.comm.all_gather_params()
        return total

    def _gather_flat(self, chunk: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return chunk.detach().clone()
        parts = [torch.empty_like(chunk) for _ in range(self.world)]
        dist.all_gather(parts, chunk.detach().contiguous(), group=self.group)
        return torch.cat(parts)

    def full_state_dict(self) -> dict:
        """The optimizer state as a ``torch.optim.AdamW`` over the model's parameters would
        hold it (moments shaped like each parameter, in parameter order), gathered from
        every rank.  Collective: every rank calls it; every rank gets the result."""
        st = self.optimizer.state.get(self.shard, {})
        if "exp_avg" not in st:
            return {"state": {}, "param_groups": self._full_groups()}
        m1, m2 = self._gather_flat(st["exp_avg"]), self._gather_flat(st["exp_avg_sq"])
        step = st["step"].detach().clone() if torch.is_tensor(st["step"]) else torch.tensor(float(st["step"]))
        state, off = {}, 0
        for i, p in enumerate(self.params):
            k = p.numel()
            state[i] = {"step": step.clone(), "exp_avg": m1[off:off + k].view_as(p).clone(),
                        "exp_avg_sq": m2[off:off + k].view_as(p).clone()}
            off += k
        return {"state": state, "param_groups": self._full_groups()}

    def _full_groups(self) -> list:
        g = {k: v for k, v in self.optimizer.param_groups[0].items() if k != "params"}
        g["params"] = list(range(len(self.params)))
        return [g]

    def load_full_state_dict(self, sd: dict) -> None:
        """Take this rank's chunk of a full (replicated-layout) AdamW state dict."""
        if not sd.get("state"):
            return
        flat1 = torch.zeros(self.numel_padded, dtype=torch.float32, device=self.device)
        flat2 = torch.zeros_like(flat1)
        off = 0
        for i, p in enumerate(self.params):
            k = p.numel()
            flat1[off:off + k] = sd["state"][i]["exp_avg"].reshape(-1).to(flat1)
            flat2[off:off + k] = sd["state"][i]["exp_avg_sq"].reshape(-1).to(flat2)
            off += k
        c0 = self.rank * self.chunk
        step = sd["state"][0]["step"]
        own = {"step": torch.as_tensor(step, dtype=torch.float32).clone(),
               "exp_avg": flat1[c0:c0 + self.chunk].clone(), "exp_avg_sq": flat2[c0:c0 + self.chunk].clone()}
        groups = [dict(sd["param_groups"][0], params=[0])]
        self.optimizer.load_state_dict({"state": {0: own}, "param_groups": groups})

    def state_dict(self) -> dict:
        """This rank's optimizer state (its chunk's moments) with the layout needed to merge shards."""
        return {"optimizer": self.optimizer.state_dict(), "rank": self.rank, "world": self.world,
                "chunk": self.chunk, "numel": self.numel}

    def load_state_dict(self, sd: dict) -> None:
        if sd["world"] != self.world or sd["chunk"] != self.chunk:
            raise ValueError("optimizer shard was saved with a different world size or model")
        self.optimizer.load_state_dict(sd["optimizer"])
