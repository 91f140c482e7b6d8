"""Data parallelism under the reference's module path (``distributed/ddp.py:47-475``).

The implementation lives in :mod:`tornado_gcm_b200.parallel.ddp`; this module
exposes it under the reference's names (``register_spectral_grad_hooks``,
``get_distributed_sampler``) so code written against
``tornado_gcm.distributed.ddp`` keeps working.
"""

from __future__ import annotations

from tornado_gcm_b200.parallel.ddp import (  # noqa: F401
    DISTRIBUTED_AVAILABLE,
    DDPConfig,
    FSDPConfig,
    GradientAllReducer,
    all_reduce_metrics,
    build_distributed_sampler,
    cleanup_distributed,
    get_distributed_sampler,
    get_local_rank,
    get_rank,
    get_world_size,
    is_distributed,
    is_main_process,
    register_fp32_spectral_grad_hooks,
    register_spectral_grad_hooks,
    setup_distributed,
    wrap_ddp,
    wrap_fsdp,
)

__all__ = [
    "DDPConfig", "FSDPConfig", "GradientAllReducer", "setup_distributed", "cleanup_distributed", "wrap_ddp",
    "wrap_fsdp", "all_reduce_metrics", "is_main_process", "is_distributed", "get_world_size", "get_rank",
    "get_local_rank", "register_spectral_grad_hooks", "register_fp32_spectral_grad_hooks",
    "get_distributed_sampler", "build_distributed_sampler",
]
