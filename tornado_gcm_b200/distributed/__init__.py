"""Distributed training: data parallelism, FSDP and DTensor sharding — reference ``distributed/__init__.py:11-74``."""

from tornado_gcm_b200.distributed.ddp import (  # noqa: F401
    DDPConfig,
    FSDPConfig,
    all_reduce_metrics,
    cleanup_distributed,
    get_distributed_sampler,
    get_rank,
    get_world_size,
    is_main_process,
    register_spectral_grad_hooks,
    setup_distributed,
    wrap_ddp,
    wrap_fsdp,
)
from tornado_gcm_b200.distributed.dtensor_sharding import (  # noqa: F401
    DTensorShardingSpec,
    LocalDeviceMesh,
    SpectralShardingContext,
    create_device_mesh,
    gather_state,
    gather_state_dict,
    gather_tensor,
    get_neuralgcm_field_specs,
    layout_to_sharding_spec,
    maybe_enable_dtensor_sharding,
    redistribute_tensor,
    shard_module_params,
    shard_state,
    shard_state_dict,
    shard_tensor,
    shard_tensor_from_local,
)
from tornado_gcm_b200.parallel.sharded_sht import LatitudeShardedSHT, latitude_partition  # noqa: F401

__all__ = [
    "DDPConfig", "FSDPConfig", "setup_distributed", "cleanup_distributed", "wrap_ddp", "wrap_fsdp",
    "all_reduce_metrics", "is_main_process", "get_world_size", "get_rank", "register_spectral_grad_hooks",
    "get_distributed_sampler", "DTensorShardingSpec", "SpectralShardingContext", "LocalDeviceMesh",
    "create_device_mesh", "shard_tensor", "shard_tensor_from_local", "gather_tensor", "redistribute_tensor",
    "shard_state_dict", "gather_state_dict", "shard_state", "gather_state", "shard_module_params",
    "get_neuralgcm_field_specs", "layout_to_sharding_spec", "maybe_enable_dtensor_sharding",
    "LatitudeShardedSHT", "latitude_partition",
]
