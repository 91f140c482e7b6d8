"""DTensor sharding of states and parameters — reference ``distributed/dtensor_sharding.py:54-846``.

The public surface matches the reference (mesh creation with a single-rank
``LocalDeviceMesh`` fallback, :class:`DTensorShardingSpec` factories, tensor /
state-dict / ``State`` shard and gather, ``maybe_enable_dtensor_sharding``,
``shard_module_params``, per-field specs and :class:`SpectralShardingContext`).

What differs is the transform path for latitude-sharded nodal data.  The
reference gathers every spatially sharded field to ``Replicate`` before each
transform.  Here a field sharded on the latitude axis (``Shard`` of the last
dimension of a ``(…, I, J)`` nodal tensor, i.e. ``spatial_lat``) is
transformed in place by :class:`~tornado_gcm_b200.parallel.sharded_sht.LatitudeShardedSHT`
with the ``"contiguous"`` partition (the same rows as ``torch.chunk``):
``to_modal`` all-reduces the partial quadrature sums (modal-sized, not
nodal-sized traffic) and ``to_nodal`` from replicated modal coefficients needs
no communication at all.  Longitude sharding still gathers (the Fourier sum
couples all longitudes of a row).

Field layout conventions follow the reference: ``level`` = ``Shard(0)``
(levels of ``(n, …)`` fields, or the batch), ``spatial_lon`` = ``Shard(1)``,
``spatial_lat`` = ``Shard(2)`` of ``(n, I, J)`` nodal fields.
"""

from __future__ import annotations

import dataclasses
import logging
from typing import Any, Optional

import torch
import torch.distributed as dist
import torch.nn as nn

from tornado_gcm_b200.core.primitive_equations import State

logger = logging.getLogger(__name__)

LAYOUTS = ("replicate", "none", "level", "batch", "spatial_lon", "spatial_lat")


@dataclasses.dataclass
class LocalDeviceMesh:
    """Single-rank stand-in for a ``DeviceMesh`` (no process group needed)."""

    mesh_shape: tuple
    mesh_dim_names: tuple
    device_type: str = "cpu"

    @property
    def ndim(self) -> int:
        return len(self.mesh_shape)

    @property
    def mesh(self) -> torch.Tensor:
        return torch.zeros(self.mesh_shape, dtype=torch.int64)

    def size(self, dim: Optional[int] = None) -> int:
        if dim is None:
            n = 1
            for s in self.mesh_shape:
                n *= s
            return n
        return self.mesh_shape[dim]


def dtensor_available() -> bool:
    try:
        from torch.distributed.device_mesh import DeviceMesh  # noqa: F401
        from torch.distributed.tensor import DTensor, Replicate, Shard  # noqa: F401
    except ImportError:
        return False
    return True


def _placements():
    from torch.distributed.tensor import Replicate, Shard

    return Shard, Replicate


def _parse_mesh_shape(mesh_shape) -> Optional[tuple]:
    if mesh_shape is None:
        return None
    if isinstance(mesh_shape, (tuple, list)):
        return tuple(int(s) for s in mesh_shape) or None
    text = str(mesh_shape).strip().lower()
    if text in ("", "auto", "none"):
        return None
    shape = tuple(int(t) for t in text.replace("x", ",").split(",") if t.strip())
    if not shape or min(shape) <= 0:
        raise ValueError(f"invalid mesh shape {mesh_shape!r}")
    return shape


def _parse_mesh_dim_names(names, ndim: int) -> Optional[tuple]:
    if names is None or names == "":
        return None
    parts = tuple(names) if isinstance(names, (tuple, list)) else tuple(
        t.strip() for t in str(names).split(",") if t.strip())
    if len(parts) != ndim:
        raise ValueError(f"mesh dim names {parts} do not match a {ndim}-D mesh")
    return parts


# ─────────────────────────────── mesh ───────────────────────────────


def create_device_mesh(mesh_shape=None, mesh_dim_names=None, device_type: str = "cuda"):
    """``DeviceMesh`` over the initialised process group (reference ``:133-222``).

    ``mesh_shape=None`` gives a 1-D ``("dp",)`` mesh over all ranks.  Without a
    process group, or with one rank when the mesh cannot be built, a
    :class:`LocalDeviceMesh` is returned.
    """
    shape = _parse_mesh_shape(mesh_shape)
    initialised = dist.is_available() and dist.is_initialized()
    world = dist.get_world_size() if initialised else 1
    if shape is None:
        shape = (world,)
        mesh_dim_names = mesh_dim_names or ("dp",)
    names = _parse_mesh_dim_names(mesh_dim_names, len(shape)) or tuple(f"dim{i}" for i in range(len(shape)))
    prod = 1
    for s in shape:
        prod *= s
    if prod != world:
        raise ValueError(f"mesh {shape} has {prod} ranks but the world has {world}")
    if not initialised:
        return LocalDeviceMesh(shape, names, device_type)
    from torch.distributed.device_mesh import init_device_mesh

    try:
        return init_device_mesh(device_type, shape, mesh_dim_names=names)
    except Exception as exc:  # noqa: BLE001
        if world == 1:
            logger.warning("using LocalDeviceMesh on a single rank (%s)", exc)
            return LocalDeviceMesh(shape, names, device_type)
        raise


# ─────────────────────────────── specs ──────────────────────────────


@dataclasses.dataclass
class DTensorShardingSpec:
    """Placements for one tensor on a mesh (one entry per mesh dimension)."""

    placements: tuple

    @staticmethod
    def level_shard(mesh_ndim: int = 1) -> "DTensorShardingSpec":
        Shard, Replicate = _placements()
        return DTensorShardingSpec(tuple([Shard(0)] + [Replicate()] * (mesh_ndim - 1)))

    @staticmethod
    def batch_shard(mesh_ndim: int = 1) -> "DTensorShardingSpec":
        return DTensorShardingSpec.level_shard(mesh_ndim)

    @staticmethod
    def replicate(mesh_ndim: int = 1) -> "DTensorShardingSpec":
        _, Replicate = _placements()
        return DTensorShardingSpec(tuple(Replicate() for _ in range(mesh_ndim)))

    @staticmethod
    def spatial_shard(dim: int = 1, mesh_ndim: int = 1) -> "DTensorShardingSpec":
        """Shard nodal ``(n, I, J)`` fields on longitude (``dim=1``) or latitude (``dim=2``)."""
        Shard, Replicate = _placements()
        return DTensorShardingSpec(tuple([Shard(dim)] + [Replicate()] * (mesh_ndim - 1)))

    def sharded_dim(self) -> Optional[int]:
        Shard, _ = _placements()
        for p in self.placements:
            if isinstance(p, Shard):
                return p.dim
        return None


def layout_to_sharding_spec(layout: Optional[str], mesh_ndim: int = 1) -> DTensorShardingSpec:
    name = (layout or "replicate").strip().lower()
    if name in ("replicate", "none"):
        return DTensorShardingSpec.replicate(mesh_ndim)
    if name in ("level", "batch"):
        return DTensorShardingSpec.level_shard(mesh_ndim)
    if name == "spatial_lon":
        return DTensorShardingSpec.spatial_shard(1, mesh_ndim)
    if name == "spatial_lat":
        return DTensorShardingSpec.spatial_shard(2, mesh_ndim)
    raise ValueError(f"unknown DTensor layout {layout!r}; expected one of {LAYOUTS}")


# ─────────────────────────── tensors ────────────────────────────────


def _is_dtensor(t) -> bool:
    try:
        from torch.distributed.tensor import DTensor
    except ImportError:
        return False
    return isinstance(t, DTensor)


def shard_tensor(tensor: torch.Tensor, spec: DTensorShardingSpec, mesh):
    """Distribute a full tensor (identity on a :class:`LocalDeviceMesh`)."""
    if isinstance(mesh, LocalDeviceMesh):
        return tensor
    from torch.distributed.tensor import distribute_tensor

    return distribute_tensor(tensor, device_mesh=mesh, placements=spec.placements)


def shard_tensor_from_local(local_tensor: torch.Tensor, spec: DTensorShardingSpec, mesh, global_shape=None):
    """Wrap this rank's shard without communication."""
    if isinstance(mesh, LocalDeviceMesh):
        return local_tensor
    from torch.distributed.tensor import DTensor

    kw = {} if global_shape is None else {"shape": torch.Size(global_shape),
                                          "stride": torch.empty(global_shape, device="meta").stride()}
    return DTensor.from_local(local_tensor, device_mesh=mesh, placements=spec.placements, run_check=False, **kw)


def gather_tensor(dtensor):
    """Full tensor of a DTensor (all-gather when sharded); plain tensors pass through."""
    return dtensor.full_tensor() if _is_dtensor(dtensor) else dtensor


def redistribute_tensor(dtensor, target_spec: DTensorShardingSpec, mesh=None):
    if not _is_dtensor(dtensor):
        return dtensor
    return dtensor.redistribute(device_mesh=mesh or dtensor.device_mesh, placements=target_spec.placements)


# ─────────────────────── state dicts and states ─────────────────────


def _map_tensors(fn, obj, prefix: str = ""):
    if isinstance(obj, torch.Tensor):
        return fn(prefix, obj)
    if isinstance(obj, dict):
        return {k: _map_tensors(fn, v, f"{prefix}.{k}" if prefix else str(k)) for k, v in obj.items()}
    return obj


def shard_state_dict(state: dict, mesh, field_specs: Optional[dict] = None,
                     default_spec: Optional[DTensorShardingSpec] = None) -> dict:
    """Shard every tensor of a (nested) dict; nested keys are ``"outer.inner"``."""
    default_spec = default_spec or DTensorShardingSpec.level_shard(mesh.ndim)
    field_specs = field_specs or {}

    def spec_for(key):
        if key in field_specs:
            return field_specs[key]
        head = key.split(".", 1)[0]
        return field_specs.get(head, default_spec)

    return _map_tensors(lambda k, t: shard_tensor(t, spec_for(k), mesh), state)


def gather_state_dict(state: dict) -> dict:
    return _map_tensors(lambda k, t: gather_tensor(t), state)


def shard_state(state: State, mesh, field_specs: Optional[dict] = None,
                default_spec: Optional[DTensorShardingSpec] = None) -> State:
    default_spec = default_spec or DTensorShardingSpec.level_shard(mesh.ndim)
    field_specs = field_specs or {}
    spec = lambda k: field_specs.get(k, default_spec)
    tracers = {k: shard_tensor(v, field_specs.get(f"tracers.{k}", field_specs.get("tracers", default_spec)), mesh)
               for k, v in state.tracers.items()}
    return State(shard_tensor(state.vorticity, spec("vorticity"), mesh),
                 shard_tensor(state.divergence, spec("divergence"), mesh),
                 shard_tensor(state.temperature_variation, spec("temperature_variation"), mesh),
                 shard_tensor(state.log_surface_pressure, spec("log_surface_pressure"), mesh),
                 tracers, state.sim_time)


def gather_state(state: State) -> State:
    g = gather_tensor
    return State(g(state.vorticity), g(state.divergence), g(state.temperature_variation),
                 g(state.log_surface_pressure), {k: g(v) for k, v in state.tracers.items()}, state.sim_time)


# ───────────────────────── parameters ───────────────────────────────


def shard_module_params(module: nn.Module, mesh, param_specs: Optional[dict] = None,
                        default_spec: Optional[DTensorShardingSpec] = None) -> None:
    """Replace each parameter by a DTensor-backed one (reference ``:670-719``)."""
    if isinstance(mesh, LocalDeviceMesh):
        return
    from torch.distributed.tensor import distribute_tensor

    default_spec = default_spec or DTensorShardingSpec.replicate(mesh.ndim)
    param_specs = param_specs or {}
    for name, p in list(module.named_parameters()):
        spec = param_specs.get(name, param_specs.get(name.rsplit(".", 1)[-1], default_spec))
        owner = module
        *path, leaf = name.split(".")
        for part in path:
            owner = getattr(owner, part)
        owner.register_parameter(leaf, nn.Parameter(distribute_tensor(p.data, mesh, spec.placements),
                                                    requires_grad=p.requires_grad))


def get_neuralgcm_field_specs(coords: Any, mesh_ndim: int = 1) -> dict:
    """Recommended specs: 3-D fields and tracers on levels, surface fields and bases replicated."""
    level = DTensorShardingSpec.level_shard(mesh_ndim)
    rep = DTensorShardingSpec.replicate(mesh_ndim)
    specs = {"vorticity": level, "divergence": level, "temperature_variation": level, "tracers": level,
             "log_surface_pressure": rep, "basis.f": rep, "basis.p": rep, "basis.w": rep}
    layers = getattr(getattr(coords, "vertical", None), "layers", None)
    if layers is not None and layers <= 1:
        for k in ("vorticity", "divergence", "temperature_variation", "tracers"):
            specs[k] = rep
    return specs


# ─────────────────────── spectral context ───────────────────────────


class SpectralShardingContext:
    """Transforms of sharded nodal / modal DTensors (reference ``:779-846``).

    * level (``Shard(0)``): each rank transforms its own levels, no traffic;
    * latitude (``Shard`` of the last nodal dim): partial sums + one
      all-reduce of the modal field (``to_modal``); ``to_nodal`` from
      replicated modal coefficients is local;
    * longitude: all-gather before the transform, as in the reference.
    """

    def __init__(self, mesh, spec: DTensorShardingSpec):
        self.mesh = mesh
        self.spec = spec
        self._dim = None if isinstance(mesh, LocalDeviceMesh) else spec.sharded_dim()
        self._sht = {}

    def _lat_sht(self, grid):
        from tornado_gcm_b200.parallel.sharded_sht import LatitudeShardedSHT

        key = id(grid)
        if key not in self._sht:
            group = self.mesh.get_group(0)
            self._sht[key] = LatitudeShardedSHT(grid, world=dist.get_world_size(group),
                                                rank=dist.get_rank(group), group=group, scheme="contiguous")
        return self._sht[key]

    def _replicated(self):
        return DTensorShardingSpec.replicate(self.mesh.ndim)

    def to_modal(self, grid, nodal_dt):
        """Nodal (DTensor or local) → modal DTensor (level-sharded or replicated)."""
        local = nodal_dt.to_local() if _is_dtensor(nodal_dt) else nodal_dt
        if self._dim is None:
            return grid.to_modal(local)
        if self._dim == 0:
            return shard_tensor_from_local(grid.to_modal(local), self.spec, self.mesh)
        if self._dim == local.ndim - 1:     # latitude: partial sums + all-reduce
            modal = self._lat_sht(grid).to_modal(local)
        else:                               # longitude: gather the rows first
            modal = grid.to_modal(gather_tensor(nodal_dt))
        return shard_tensor_from_local(modal, self._replicated(), self.mesh)

    def to_nodal(self, grid, modal_dt):
        """Modal → nodal DTensor with this context's spec."""
        if self._dim is None:
            return grid.to_nodal(modal_dt.to_local() if _is_dtensor(modal_dt) else modal_dt)
        if self._dim == 0:
            local = modal_dt.to_local() if _is_dtensor(modal_dt) else modal_dt
            return shard_tensor_from_local(grid.to_nodal(local), self.spec, self.mesh)
        full = gather_tensor(modal_dt)
        sh = grid.spherical_harmonics
        shape = tuple(full.shape[:-2]) + (sh.longitude_nodes, sh.latitude_nodes)
        if self._dim == full.ndim - 1:      # each rank evaluates its own latitude rows
            return shard_tensor_from_local(self._lat_sht(grid).to_nodal(full), self.spec, self.mesh,
                                           global_shape=shape)
        return shard_tensor(grid.to_nodal(full), self.spec, self.mesh)


# ─────────────────────────── model hook ─────────────────────────────

# State layouts that run the model step itself sharded (modal rows by zonal
# wavenumber, nodal columns by latitude block) instead of sharding the state
# between steps and gathering it before each one.
MODEL_SHARDED_LAYOUTS = ("spatial_lat", "wavenumber_latitude")


def _is_hybrid_gcm(model) -> bool:
    return all(hasattr(model, a) for a in ("model", "encoder", "decoder", "loss"))


def _shard_hybrid_model(model: nn.Module, config: Any) -> nn.Module:
    """Latitude layout on a hybrid GCM: the whole step runs sharded over the ranks.

    The reference shards the state by latitude and gathers it back before every
    step (its spectral context is never used by the step,
    ``distributed/dtensor_sharding.py:779-846``, ``training/trainer.py:184-206``).
    Here the layout selects :func:`~tornado_gcm_b200.parallel.spectral_shard.shard_hybrid_gcm`:
    every spectral field keeps the rows of this rank's wavenumbers, every nodal
    field this rank's latitude block, and the transforms move data between the
    two layouts (fused peer-memory epilogues on NVLink, ``torch.distributed``
    collectives elsewhere).  ``model.scatter_fields`` cuts a batch of nodal
    fields down to this rank's block; train it with
    ``GCMTrainer(data_parallel=True, grad_average=False)``.
    """
    from tornado_gcm_b200.parallel import spectral_shard as ss

    dev = next(model.parameters()).device
    engine = getattr(config, "dtensor_transform_engine", None) or ("auto" if dev.type == "cuda" else "collective")
    ss.shard_hybrid_gcm(model, None, engine)
    ctx = model.shard
    model._dtensor_runtime_mode = "model_sharded"
    model._dtensor_mesh = None
    model.scatter_fields = lambda fields: ss.scatter_fields(fields, ctx)
    return model


def maybe_enable_dtensor_sharding(model: nn.Module, config: Any, coords: Any = None) -> nn.Module:
    """Bind a mesh and state shard/gather helpers to ``model`` when ``config.dtensor_aware``.

    Reads ``dtensor_mesh_shape``, ``dtensor_mesh_dim_names``,
    ``dtensor_state_layout`` (default ``level``) and ``dtensor_param_layout``
    (default ``replicate``) from ``config``; parameters are sharded only for a
    non-replicated parameter layout.
    """
    if not getattr(config, "dtensor_aware", False):
        return model
    state_layout = getattr(config, "dtensor_state_layout", "level") or "level"
    if state_layout in MODEL_SHARDED_LAYOUTS and _is_hybrid_gcm(model):
        return _shard_hybrid_model(model, config)
    backend = dist.get_backend() if dist.is_available() and dist.is_initialized() else ""
    if backend == "nccl":
        device = "cuda"
    elif backend in ("gloo", "mpi"):
        device = "cpu"
    else:
        device = "cuda" if any(p.is_cuda for p in model.parameters()) else "cpu"
    shape = _parse_mesh_shape(getattr(config, "dtensor_mesh_shape", None))
    names = _parse_mesh_dim_names(getattr(config, "dtensor_mesh_dim_names", None), len(shape) if shape else 1)
    mesh = create_device_mesh(shape, names, device)
    if coords is None:
        for owner in (getattr(model, "model_config", None), getattr(model, "config", None), model):
            coords = getattr(owner, "coords", None)
            if coords is not None:
                break
    param_layout = getattr(config, "dtensor_param_layout", "replicate") or "replicate"
    state_spec = layout_to_sharding_spec(state_layout, mesh.ndim)
    param_spec = layout_to_sharding_spec(param_layout, mesh.ndim)
    field_specs = get_neuralgcm_field_specs(coords, mesh.ndim) if coords is not None else {}
    if state_layout != "level":
        for k in ("vorticity", "divergence", "temperature_variation", "tracers"):
            field_specs[k] = state_spec
    model._dtensor_mesh = mesh
    model._dtensor_runtime_mode = "local_fallback" if isinstance(mesh, LocalDeviceMesh) else "device_mesh"
    model._dtensor_field_specs = field_specs
    model._dtensor_state_default_spec = state_spec
    model._dtensor_param_default_spec = param_spec
    model._dtensor_spectral_context = SpectralShardingContext(mesh, state_spec)
    model.shard_state_with_dtensor = lambda s: shard_state(s, mesh, field_specs, state_spec)
    model.gather_state_from_dtensor = gather_state
    model._dtensor_parameterization_sharded = False
    if param_layout not in ("replicate", "none") and hasattr(model, "parameterization"):
        try:
            shard_module_params(model.parameterization, mesh, default_spec=param_spec)
            model._dtensor_parameterization_sharded = True
        except Exception as exc:  # noqa: BLE001
            logger.warning("parameter sharding not applied: %s", exc)
    return model


__all__ = [
    "LocalDeviceMesh", "DTensorShardingSpec", "SpectralShardingContext", "create_device_mesh", "shard_tensor",
    "shard_tensor_from_local", "gather_tensor", "redistribute_tensor", "shard_state_dict", "gather_state_dict",
    "shard_state", "gather_state", "shard_module_params", "get_neuralgcm_field_specs", "layout_to_sharding_spec",
    "maybe_enable_dtensor_sharding", "dtensor_available",
]
