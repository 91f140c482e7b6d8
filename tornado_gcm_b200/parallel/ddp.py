"""Data parallelism — reference ``distributed/ddp.py:47-475``.

Process-group bootstrap (``setup_distributed``), the reference's
``wrap_ddp`` / ``wrap_fsdp`` entry points (torch DDP / FSDP with the
reference's configuration), the FP32 spectral-gradient hooks, the
distributed sampler helper, and :class:`GradientAllReducer`: this
framework's own DP engine for the hybrid-GCM trainer.

``GradientAllReducer`` packs every gradient into one flat fp32 buffer
(parameters are assigned to contiguous views of it, so backward writes in
place) and reduces it with a single collective per bucket after
backward-through-rollout; on NVLink it uses the fused symmetric-memory
reduce kernels of :mod:`tornado_gcm_b200.parallel.fused_allreduce` when
available, otherwise NCCL.  Scaling by 1/world is fused into the reduce.
"""

from __future__ import annotations

import dataclasses
import datetime
import logging
import os
from typing import Optional, Sequence

import torch
import torch.distributed as dist
import torch.nn as nn

logger = logging.getLogger(__name__)

DISTRIBUTED_AVAILABLE = dist.is_available()


@dataclasses.dataclass
class DDPConfig:
    backend: str = "nccl"
    find_unused_parameters: bool = False
    bucket_cap_mb: int = 25
    static_graph: bool = True
    gradient_as_bucket_view: bool = True
    fp32_spectral_grads: bool = False


@dataclasses.dataclass
class FSDPConfig:
    sharding_strategy: str = "FULL_SHARD"
    min_num_params: int = 100_000
    wrap_policy: str = "size"
    param_dtype: torch.dtype = torch.float32
    reduce_dtype: torch.dtype = torch.float32
    buffer_dtype: torch.dtype = torch.float32
    backward_prefetch: str = "BACKWARD_PRE"
    forward_prefetch: bool = True
    limit_all_gathers: bool = True
    use_orig_params: bool = True
    cpu_offload: bool = False

    @classmethod
    def from_env(cls) -> "FSDPConfig":
        c = cls()
        env = os.environ
        if "NEURALGCM_FSDP_STRATEGY" in env:
            c.sharding_strategy = env["NEURALGCM_FSDP_STRATEGY"]
        if "NEURALGCM_FSDP_MIN_PARAMS" in env:
            c.min_num_params = int(env["NEURALGCM_FSDP_MIN_PARAMS"])
        if "NEURALGCM_FSDP_WRAP_POLICY" in env:
            c.wrap_policy = env["NEURALGCM_FSDP_WRAP_POLICY"]
        if "NEURALGCM_FSDP_CPU_OFFLOAD" in env:
            c.cpu_offload = env["NEURALGCM_FSDP_CPU_OFFLOAD"] not in ("0", "false", "False")
        return c


def is_distributed() -> bool:
    return dist.is_available() and dist.is_initialized()


def get_rank() -> int:
    return dist.get_rank() if is_distributed() else 0


def get_world_size() -> int:
    return dist.get_world_size() if is_distributed() else 1


def get_local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK", "0"))


def is_main_process() -> bool:
    return get_rank() == 0


def setup_distributed(backend: Optional[str] = None, init_method: Optional[str] = None,
                      world_size: Optional[int] = None, rank: Optional[int] = None,
                      timeout_s: float = 600.0) -> tuple[int, int, int]:
    """Initialise the default process group; returns ``(rank, world, local rank)``.

    ``world_size`` / ``rank`` default to the launcher's WORLD_SIZE / RANK; ``init_method``
    defaults to ``env://`` (MASTER_ADDR / MASTER_PORT, 127.0.0.1:29500 when unset)."""
    if is_distributed():
        return get_rank(), get_world_size(), get_local_rank()
    world = int(world_size if world_size is not None else os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return 0, 1, 0
    rank = int(rank if rank is not None else os.environ.get("RANK", "0"))
    if init_method is None or init_method.startswith("env://"):
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29500")
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    local = get_local_rank()
    if backend == "nccl":
        torch.cuda.set_device(local)
    dist.init_process_group(backend=backend, init_method=init_method or "env://", world_size=world, rank=rank,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist.get_rank(), dist.get_world_size(), local


def cleanup_distributed() -> None:
    if is_distributed():
        dist.destroy_process_group()


def wrap_ddp(model: nn.Module, config: DDPConfig | None = None, device_id: Optional[int] = None,
             device_ids=None) -> nn.Module:
    """torch DDP with the reference's settings (baseline path); ``device_id`` (the reference's
    argument) or ``device_ids`` pick the GPU, else the current device."""
    config = config or DDPConfig()
    if not is_distributed():
        return model
    from torch.nn.parallel import DistributedDataParallel as DDP

    if device_ids is None and device_id is not None:
        device_ids = [device_id]
    if device_ids is None and torch.cuda.is_available() and next(model.parameters()).is_cuda:
        device_ids = [torch.cuda.current_device()]
    wrapped = DDP(model, device_ids=device_ids, find_unused_parameters=config.find_unused_parameters,
                  bucket_cap_mb=config.bucket_cap_mb, static_graph=config.static_graph,
                  gradient_as_bucket_view=config.gradient_as_bucket_view)
    if config.fp32_spectral_grads:
        register_fp32_spectral_grad_hooks(wrapped)
    return wrapped


def wrap_fsdp(model: nn.Module, config: FSDPConfig | None = None) -> nn.Module:
    """torch FSDP with size / transformer auto-wrap (reference ``ddp.py:245-361``)."""
    config = config or FSDPConfig.from_env()
    if not is_distributed():
        return model
    import functools

    from torch.distributed.fsdp import BackwardPrefetch, CPUOffload, MixedPrecision, ShardingStrategy
    from torch.distributed.fsdp import FullyShardedDataParallel as FSDP
    from torch.distributed.fsdp.wrap import size_based_auto_wrap_policy, transformer_auto_wrap_policy

    if config.wrap_policy == "transformer":
        from tornado_gcm_b200.neural.transformer_layers import TransformerBlock

        policy = functools.partial(transformer_auto_wrap_policy, transformer_layer_cls={TransformerBlock})
    else:
        policy = functools.partial(size_based_auto_wrap_policy, min_num_params=config.min_num_params)
    mp = MixedPrecision(param_dtype=config.param_dtype, reduce_dtype=config.reduce_dtype,
                        buffer_dtype=config.buffer_dtype)
    return FSDP(model, sharding_strategy=getattr(ShardingStrategy, config.sharding_strategy),
                auto_wrap_policy=policy, mixed_precision=mp,
                backward_prefetch=getattr(BackwardPrefetch, config.backward_prefetch),
                forward_prefetch=config.forward_prefetch, limit_all_gathers=config.limit_all_gathers,
                use_orig_params=config.use_orig_params, cpu_offload=CPUOffload(offload_params=config.cpu_offload),
                device_id=torch.cuda.current_device() if torch.cuda.is_available() else None)


def register_fp32_spectral_grad_hooks(model: nn.Module, keywords: Sequence[str] = ("spectral", "modal", "sht")):
    """Accumulate gradients of spectral parameters in fp32."""
    handles = []
    for name, p in model.named_parameters():
        if any(k in name.lower() for k in keywords) and p.dtype != torch.float32:
            handles.append(p.register_hook(lambda g: g.float()))
    return handles


def register_spectral_grad_hooks(model: nn.Module, spectral_param_patterns: Sequence[str] = ("dynamics",)) -> list:
    """Reference-named variant of :func:`register_fp32_spectral_grad_hooks`: parameters whose
    name matches one of the regular expressions get their gradients in fp32."""
    import re

    rx = [re.compile(p) for p in spectral_param_patterns]
    return [p.register_hook(lambda g: g.float() if g is not None and g.dtype != torch.float32 else g)
            for name, p in model.named_parameters() if any(r.search(name) for r in rx)]


def get_distributed_sampler(dataset, shuffle: bool = True, seed: int = 42):
    """Reference-named sampler helper: a DistributedSampler with more than one rank, else None."""
    return build_distributed_sampler(dataset, shuffle=shuffle, seed=seed)


def build_distributed_sampler(dataset, shuffle: bool = True, seed: int = 0, drop_last: bool = False):
    from torch.utils.data.distributed import DistributedSampler

    if not is_distributed():
        return None
    return DistributedSampler(dataset, num_replicas=get_world_size(), rank=get_rank(), shuffle=shuffle, seed=seed,
                              drop_last=drop_last)


class GradientAllReducer:
    """Flat-buffer gradient averaging over the default process group.

    Parameters' ``.grad`` are views into one contiguous fp32 buffer, so the
    reduction is one collective (or one fused kernel) per bucket.  Ranks
    must call :meth:`reduce` at the same point (after backward).
    """

    def __init__(self, params: Sequence[torch.nn.Parameter], bucket_mb: float = 0.0, use_fused: bool = True,
                 average: bool = True):
        self.params = [p for p in params if p.requires_grad]
        dev = self.params[0].device
        sizes = [p.numel() for p in self.params]
        self.numel = sum(sizes)
        self.world = get_world_size()
        self.average = average
        self.bucket_elems = int(bucket_mb * 1e6 / 4) if bucket_mb > 0 else self.numel
        self.fused = None
        # The fused NVLink kernel is the reducer on CUDA with more than one rank.
        # It is turned off only on request (use_fused=False or
        # TGCM_FUSED_ALLREDUCE=0); when it was requested and cannot be set up the
        # constructor raises instead of silently running the NCCL path.
        want_fused = (use_fused and self.world > 1 and dev.type == "cuda"
                      and os.environ.get("TGCM_FUSED_ALLREDUCE", "1") != "0")
        if want_fused:
            from tornado_gcm_b200.parallel.transport import get_transport

            try:
                self.fused = get_transport("nvlink", device=dev).gradient_reducer(self.numel, dev)
            except Exception as exc:
                raise RuntimeError(f"fused gradient all-reduce requested but unavailable: {exc}; "
                                   "set TGCM_FUSED_ALLREDUCE=0 to use NCCL") from exc
        if self.world <= 1:
            self.backend = "none (one rank)"
        elif self.fused is not None:
            self.backend = "fused NVLink peer-memory kernel (csrc/comm.cu)"
        else:
            self.backend = "nccl" if dev.type == "cuda" else str(dist.get_backend())
        # the flat buffer is the reducer's symmetric allocation when fused
        self.flat = self.fused.flat if self.fused is not None else torch.zeros(self.numel, dtype=torch.float32,
                                                                               device=dev)
        self.views = []
        off = 0
        for p, n in zip(self.params, sizes):
            self.views.append(self.flat[off:off + n].view_as(p))
            off += n

    def attach(self) -> None:
        """Point each parameter's .grad at its view of the flat buffer."""
        for p, v in zip(self.params, self.views):
            p.grad = v

    def zero(self) -> None:
        self.flat.zero_()
        self.attach()

    def reduce(self) -> None:
        if self.world <= 1:
            return
        # grads may have been re-allocated by autograd if .grad was None
        for p, v in zip(self.params, self.views):
            if p.grad is not None and p.grad.data_ptr() != v.data_ptr():
                v.copy_(p.grad)
                p.grad = v
        if self.fused is not None:
            if self.average:
                self.fused.all_reduce_mean(self.flat)
            else:
                self.fused.all_reduce_sum(self.flat)
            return
        for s in range(0, self.numel, self.bucket_elems):
            chunk = self.flat[s:s + self.bucket_elems]
            dist.all_reduce(chunk, op=dist.ReduceOp.SUM)
        if self.average:
            self.flat.mul_(1.0 / self.world)

    def broadcast_parameters(self, src: int = 0) -> None:
        if self.world <= 1:
            return
        with torch.no_grad():
            for p in self.params:
                dist.broadcast(p.data, src=src)


def all_reduce_metrics(metrics: dict, op: str = "mean") -> dict:
    from tornado_gcm_b200.parallel.metrics import all_reduce_metrics as _arm

    return _arm(metrics, op)
