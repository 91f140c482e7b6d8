"""Latitude-sharded transforms and DTensor sharding on CPU ranks (gloo).

The sharded transforms are checked against the single-process transform of
the full field (FP64): ``to_nodal`` on each rank's latitude rows and
``to_modal`` from the rows (partial sums + all-reduce), for the mirrored
(even/odd Legendre) and contiguous (``torch.chunk``) partitions.
"""

import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tornado_gcm_b200.core import spherical_harmonic as shm
from tornado_gcm_b200.parallel.sharded_sht import LatitudeShardedSHT, latitude_partition


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))


@pytest.mark.parametrize("scheme", ["mirrored", "contiguous"])
@pytest.mark.parametrize("world", [1, 2, 3, 5])
def test_latitude_partition_covers_grid(scheme, world):
    for J in (32, 64, 33):
        parts = [latitude_partition(J, world, r, scheme) for r in range(world)]
        allidx = np.sort(np.concatenate(parts))
        assert np.array_equal(allidx, np.arange(J))
        if scheme == "mirrored":
            for p in parts:
                s = set(p.tolist())
                assert all((J - 1 - j) in s for j in p)


@pytest.mark.parametrize("scheme", ["mirrored", "contiguous"])
def test_sharded_sht_single_process(scheme):
    g = shm.Grid.T21()
    torch.manual_seed(0)
    x = torch.randn(2, 3, *g.modal_shape, dtype=torch.float64) * torch.as_tensor(g.mask)
    nodal = g.to_nodal(x)
    for world in (2, 4):
        total = 0
        for r in range(world):
            s = LatitudeShardedSHT(g, world=world, rank=r, scheme=scheme)
            np.testing.assert_allclose(s.to_nodal(x).numpy(), s.scatter(nodal).numpy(), atol=1e-11)
            total = total + s.partial_to_modal(s.scatter(nodal))
        np.testing.assert_allclose(total.numpy(), g.to_modal(nodal).numpy(), atol=1e-11)


def test_sharded_sht_halves_legendre_work():
    g = shm.Grid.TL63()
    full = LatitudeShardedSHT(g, world=2, rank=0, scheme="contiguous")
    half = LatitudeShardedSHT(g, world=2, rank=0, scheme="mirrored")
    assert half.flops_legendre(1) <= 0.52 * full.flops_legendre(1)


def _worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from tornado_gcm_b200.core.primitive_equations import State
        from tornado_gcm_b200.distributed import dtensor_sharding as ds

        g = shm.Grid.T21()
        torch.manual_seed(0)  # same data on every rank
        x = torch.randn(4, *g.modal_shape, dtype=torch.float64) * torch.as_tensor(g.mask)
        nodal = g.to_nodal(x)
        res = {}
        # process-group sharded transforms (mirrored pairs)
        s = LatitudeShardedSHT(g, scheme="mirrored")
        res["nodal"] = float((s.to_nodal(x) - s.scatter(nodal)).abs().max())
        res["modal"] = float((s.to_modal(s.scatter(nodal)) - g.to_modal(nodal)).abs().max())
        res["gather"] = float((s.gather(s.scatter(nodal)) - nodal).abs().max())
        # DTensor layer
        mesh = ds.create_device_mesh(device_type="cpu")
        spec = ds.DTensorShardingSpec.spatial_shard(dim=2)
        nodal_dt = ds.shard_tensor(nodal, spec, mesh)
        ctx = ds.SpectralShardingContext(mesh, spec)
        modal_dt = ctx.to_modal(g, nodal_dt)
        res["ctx_modal"] = float((ds.gather_tensor(modal_dt) - g.to_modal(nodal)).abs().max())
        back = ctx.to_nodal(g, modal_dt)
        res["ctx_nodal"] = float((ds.gather_tensor(back) - nodal).abs().max())
        lev = ds.SpectralShardingContext(mesh, ds.DTensorShardingSpec.level_shard())
        res["lev_modal"] = float((ds.gather_tensor(lev.to_modal(g, ds.shard_tensor(nodal, lev.spec, mesh)))
                                  - g.to_modal(nodal)).abs().max())
        st = State(x, 2 * x, 3 * x, x[:1], {"q": 4 * x}, 0.0)
        sh = ds.shard_state(st, mesh, ds.get_neuralgcm_field_specs(None))
        res["local_levels"] = int(sh.vorticity.to_local().shape[0])
        back_state = ds.gather_state(sh)
        res["state"] = float(max((back_state.tracers["q"] - 4 * x).abs().max(),
                                 (back_state.divergence - 2 * x).abs().max()))
        sd = ds.gather_state_dict(ds.shard_state_dict({"a": x, "inner": {"b": 2 * x}}, mesh))
        res["sd"] = float((sd["inner"]["b"] - 2 * x).abs().max())

        class Cfg:
            dtensor_aware = True
            dtensor_state_layout = "level"
            dtensor_param_layout = "replicate"

        m = torch.nn.Linear(3, 3)
        ds.maybe_enable_dtensor_sharding(m, Cfg())
        res["mode"] = m._dtensor_runtime_mode
        q.put((rank, res))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        q.put((rank, traceback.format_exc()))


def test_sharded_transforms_gloo_world2():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, res in out:
        assert isinstance(res, dict), res
        for k in ("nodal", "modal", "gather", "ctx_modal", "ctx_nodal", "lev_modal", "state", "sd"):
            assert res[k] < 1e-10, (rank, k, res[k])
        assert res["local_levels"] == 2
        assert res["mode"] == "device_mesh"


def test_local_mesh_without_process_group():
    from tornado_gcm_b200.distributed import dtensor_sharding as ds

    mesh = ds.create_device_mesh(device_type="cpu")
    assert isinstance(mesh, ds.LocalDeviceMesh) and mesh.ndim == 1
    t = torch.randn(4, 3)
    assert ds.shard_tensor(t, ds.DTensorShardingSpec.level_shard(), mesh) is t
    with pytest.raises(ValueError):
        ds.layout_to_sharding_spec("diagonal")
    assert ds._parse_mesh_shape("2,2") == (2, 2) and ds._parse_mesh_shape("auto") is None
