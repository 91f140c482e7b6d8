"""The model step sharded over wavenumbers (modal) and latitude blocks (nodal), on gloo CPU ranks.

The sharded transforms, the sharded spectral operators and the whole 5.6°
hybrid model (encoder → packed SIL3 physics steps with the column tower and
the FP64 fixer → decoder → loss → backward) on 2 and 4 ranks are compared
with the same computation on the full grid in one process.
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

from tornado_gcm_b200.core import spherical_harmonic as sh
from tornado_gcm_b200.parallel import spectral_shard as ss


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))


def _spawn(fn, world):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for o in out:
        assert not isinstance(o[1], str), o[1]
    return sorted(out, key=lambda o: o[0])


def test_layout_covers_every_row_once_and_balances_work():
    g = sh.Grid.TL127()
    for world in (2, 4, 8):
        lays = [ss.ShardLayout(g, world, r) for r in range(world)]
        rows = np.concatenate([lay.rows[r][lay.rows[r] >= 0] for r, lay in enumerate(lays)])
        assert sorted(rows.tolist()) == list(range(lays[0].M2))
        L = lays[0].L
        work = [sum(L - m for m in lay.local_m) for lay in lays]
        assert max(work) / min(work) < 1.05
        lay = lays[0]
        assert all(lay.Jr * world == lay.J and lay.Jr % 4 == 0 for lay in lays)
        # (cos, sin) rows of one wavenumber stay adjacent at odd/even local positions
        for r in range(world):
            for gi, m in enumerate(lay.group_m[r]):
                if m > 0:
                    assert tuple(lay.rows[r][2 * gi - 1:2 * gi + 1]) == (2 * m - 1, 2 * m)


def _worker_transforms(rank, world, port, q):
    try:
        _init(rank, world, port)
        g = sh.Grid.T21(precision="float32")
        sg = ss.make_sharded_grid(g, None, "collective")
        lay = sg.layout
        torch.manual_seed(0)
        x = torch.randn(3, *g.modal_shape, dtype=torch.float64) * torch.as_tensor(g.mask)
        xl = lay.scatter_modal(x)
        e_syn = float((sg.to_nodal(xl) - lay.scatter_nodal(g.to_nodal(x))).abs().max())
        nod = g.to_nodal(x)
        e_ana = float((sg.to_modal(lay.scatter_nodal(nod)) - lay.scatter_modal(g.to_modal(nod))).abs().max())
        u, v = sh.get_cos_lat_vector(x[:2], x[1:], g)
        ul, vl = sh.get_cos_lat_vector(xl[:2], xl[1:], sg)
        e_op = float((ul - lay.scatter_modal(u)).abs().max() + (vl - lay.scatter_modal(v)).abs().max())
        # adjoints: <S x, y> = <x, S^T y> summed over ranks
        xr = torch.randn_like(xl).requires_grad_(True)
        yr = torch.randn(3, *sg.nodal_shape, dtype=torch.float64)
        (sg.to_nodal(xr) * yr).sum().backward()
        lhs = (sg.to_nodal(xr.detach()) * yr).sum()
        rhs = (xr.detach() * xr.grad).sum()
        t = torch.stack([lhs, rhs])
        dist.all_reduce(t)
        q.put((rank, e_syn, e_ana, e_op, float(abs(t[0] - t[1]) / abs(t[0]))))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_transforms_match_full_grid(world):
    for _, e_syn, e_ana, e_op, e_adj in _spawn(_worker_transforms, world):
        assert e_syn < 1e-10 and e_ana < 1e-10 and e_op < 1e-12 and e_adj < 1e-12


def _worker_model(rank, world, port, q):
    try:
        _init(rank, world, port)
        from tornado_gcm_b200.models.builders import build_hybrid_gcm

        def make():
            gcm, data = build_hybrid_gcm("5.6deg", "cpu", seed=0)
            gcm.model.packed_on_cpu = True
            gcm.physics_steps_per_output = 2
            return gcm, data

        ref, data = make()
        enc = ref.encoder
        norm = lambda d: {k: (v - getattr(enc, f"mean_{k}")) / getattr(enc, f"std_{k}") for k, v in d.items()}
        x0, tg, forc = norm(data.sample(2, 0)), [norm(data.sample(2, 1)), norm(data.sample(2, 2))], data.forcings(2)
        l_ref = ref.loss(x0, tg, forc)
        l_ref.backward()
        g_ref = {n: p.grad for n, p in ref.named_parameters() if p.grad is not None}
        shd, _ = make()
        ss.shard_hybrid_gcm(shd, None, "collective")
        c = shd.shard
        loss = shd.loss(ss.scatter_fields(x0, c), [ss.scatter_fields(t, c) for t in tg], ss.scatter_fields(forc, c))
        loss.backward()
        tot = loss.detach().clone()
        dist.all_reduce(tot)
        worst = 0.0
        for n, p in shd.named_parameters():
            if p.grad is None:
                continue
            gsum = p.grad.clone()
            dist.all_reduce(gsum)
            worst = max(worst, float((gsum - g_ref[n]).norm() / (g_ref[n].norm() + 1e-30)))
        q.put((rank, float(l_ref.detach()), float(tot), worst, len(g_ref)))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_model_loss_and_gradients_match_full_model(world):
    for _, l_ref, l_shd, worst, n_grads in _spawn(_worker_model, world):
        assert n_grads > 10
        assert abs(l_shd - l_ref) <= 1e-5 * abs(l_ref)
        assert worst < 1e-4


def _worker_dtensor_entry(rank, world, port, q):
    """The reference's DTensor entry point with the latitude layout runs the sharded step."""
    try:
        _init(rank, world, port)
        from tornado_gcm_b200.distributed.dtensor_sharding import maybe_enable_dtensor_sharding
        from tornado_gcm_b200.models.builders import build_hybrid_gcm

        def make():
            gcm, data = build_hybrid_gcm("5.6deg", "cpu", seed=0)
            gcm.model.packed_on_cpu = True
            gcm.physics_steps_per_output = 2
            return gcm, data

        ref, data = make()
        enc = ref.encoder
        norm = lambda d: {k: (v - getattr(enc, f"mean_{k}")) / getattr(enc, f"std_{k}") for k, v in d.items()}
        x0, tg, forc = norm(data.sample(2, 0)), [norm(data.sample(2, 1))], data.forcings(2)
        l_ref = float(ref.loss(x0, tg, forc).detach())

        class Cfg:
            dtensor_aware = True
            dtensor_state_layout = "spatial_lat"

        shd, _ = make()
        out = maybe_enable_dtensor_sharding(shd, Cfg())
        sc = out.scatter_fields
        loss = out.loss(sc(x0), [sc(t) for t in tg], sc(forc)).detach().clone()
        dist.all_reduce(loss)
        q.put((rank, l_ref, float(loss), out._dtensor_runtime_mode, out.shard.world))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))


def test_dtensor_latitude_layout_runs_the_sharded_step():
    for _, l_ref, l_shd, mode, w in _spawn(_worker_dtensor_entry, 2):
        assert mode == "model_sharded" and w == 2
        assert abs(l_shd - l_ref) <= 1e-5 * abs(l_ref)
