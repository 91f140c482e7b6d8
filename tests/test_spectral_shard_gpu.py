"""Wavenumber/latitude-sharded transforms and model step on B200s (fused engine).

* one GPU (a one-rank group): the routed Legendre epilogues (synthesis
  columns stored to the latitude owner, analysis groups reduced into the
  wavenumber owner) reproduce the regular transforms and are adjoint to each
  other;
* two GPUs (skipped with fewer): the fused sharded transforms against the
  full-grid transform, and the sharded 2.8° model's loss and weight gradients
  against the same model on one GPU.

Ranks are child processes with NCCL for bootstrap (NVLS off); the transforms
use plain peer stores / reductions and a bounded peer barrier.
"""

import datetime
import os
import socket
import traceback

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs CUDA")]


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import torch.distributed as dist

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    return dist


def _spawn(fn, world):
    import torch.multiprocessing as mp

    port = _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=900) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for o in out:
        assert not isinstance(o[1], str), o[1]
    return sorted(out, key=lambda o: o[0])


def _rel(a, b):
    return float((a.double() - b.double()).norm() / (b.double().norm() + 1e-30))


def _worker_transforms(rank, world, port, q):
    try:
        dist = _init(rank, world, port)
        from tornado_gcm_b200.core import spherical_harmonic as sh
        from tornado_gcm_b200.ops import _ext
        from tornado_gcm_b200.parallel import spectral_shard as ss

        _ext.require("sharded transform test")
        dev = torch.device("cuda", rank)
        res = {}
        for name in ("TL63", "TL127"):
            g = getattr(sh.Grid, name)(precision="float32")
            sg = ss.make_sharded_grid(g, None, "fused", dev)
            lay = sg.layout
            torch.manual_seed(0)
            m, l = g.modal_mesh
            amp = torch.as_tensor(g.mask * (1.0 + l) ** -1.5)
            x = torch.randn(7, *g.modal_shape, dtype=torch.float64) * amp
            nod = g.to_nodal(x)
            xl = lay.scatter_modal(x).float().to(dev)
            out = sg.to_nodal(xl)
            res[name + "_synth"] = _rel(out.cpu(), lay.scatter_nodal(nod))
            back = sg.to_modal(lay.scatter_nodal(nod).float().to(dev))
            res[name + "_anal"] = _rel(back.cpu(), lay.scatter_modal(g.to_modal(nod)))
            # adjoint pair: <S x, y> == <x, S^T y> over all ranks
            xr = xl.clone().requires_grad_(True)
            y = torch.randn(7, *sg.nodal_shape, device=dev)
            (sg.to_nodal(xr) * y).sum().backward()
            t = torch.stack([(sg.to_nodal(xl) * y).sum().double(), (xl * xr.grad).sum().double()])
            dist.all_reduce(t)
            res[name + "_adjoint"] = float(abs(t[0] - t[1]) / abs(t[0]))
        torch.cuda.synchronize(dev)
        res["flag"] = _ext.check_error_flag(dev)
        q.put((rank, res))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))


def _check_transforms(world):
    for _, res in _spawn(_worker_transforms, world):
        assert res["flag"] == 0
        for k, v in res.items():
            if k != "flag":
                # TF32 transforms; the adjoint check compares two inner products of random fields
                assert v < 3e-3 if k.endswith(("_synth", "_anal")) else v < 1e-2, (k, v)


def test_routed_transforms_one_rank():
    _check_transforms(1)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_sharded_transforms_two_gpus():
    _check_transforms(2)


def _worker_model(rank, world, port, q):
    try:
        dist = _init(rank, world, port)
        from tornado_gcm_b200.models.builders import build_hybrid_gcm
        from tornado_gcm_b200.ops import _ext
        from tornado_gcm_b200.parallel import spectral_shard as ss

        dev = torch.device("cuda", rank)

        def make():
            gcm, data = build_hybrid_gcm("2.8deg", dev, seed=0)
            gcm.physics_steps_per_output = 2
            return gcm, data

        ref, data = make()
        enc = ref.encoder
        norm = lambda d: {k: ((v.to(dev) - getattr(enc, f"mean_{k}")) / getattr(enc, f"std_{k}")) for k, v in d.items()}
        x0, tg = norm(data.sample(2, 0)), [norm(data.sample(2, 1))]
        forc = {k: v.to(dev) for k, v in data.forcings(2).items()}
        l_ref = ref.loss(x0, tg, forc)
        l_ref.backward()
        g_ref = {n: p.grad.detach().clone() for n, p in ref.named_parameters() if p.grad is not None}
        shd, _ = make()
        ss.shard_hybrid_gcm(shd, None, "fused")
        c = shd.shard
        loss = shd.loss(ss.scatter_fields(x0, c), [ss.scatter_fields(t, c) for t in tg], ss.scatter_fields(forc, c))
        loss.backward()
        tot = loss.detach().clone()
        dist.all_reduce(tot)
        worst = 0.0
        for n, p in shd.named_parameters():
            if p.grad is None:
                continue
            gs = p.grad.detach().clone()
            dist.all_reduce(gs)
            worst = max(worst, _rel(gs, g_ref[n]))
        torch.cuda.synchronize(dev)
        q.put((rank, float(l_ref.detach()), float(tot), worst, _ext.check_error_flag(dev)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_model_matches_one_gpu():
    for _, l_ref, l_shd, worst, flag in _spawn(_worker_model, 2):
        assert flag == 0
        assert abs(l_shd - l_ref) <= 2e-3 * abs(l_ref)   # TF32 transforms, different summation order
        assert worst < 3e-2


def _worker_fsdp(rank, world, port, q):
    try:
        dist = _init(rank, world, port)
        from tornado_gcm_b200.models.builders import build_hybrid_gcm
        from tornado_gcm_b200.ops import _ext
        from tornado_gcm_b200.parallel import spectral_shard as ss

        dev = torch.device("cuda", rank)
        gcm, data = build_hybrid_gcm("2.8deg", dev, seed=0)
        ss.shard_hybrid_gcm(gcm, None, "fused")
        enc = gcm.encoder
        norm = {k: ((v.to(dev) - getattr(enc, f"mean_{k}")) / getattr(enc, f"std_{k}"))
                for k, v in data.sample(3, 0).items()}
        forc = ss.scatter_fields({k: v.to(dev) for k, v in data.forcings(3).items()}, gcm.shard)
        with torch.no_grad():
            f = gcm.normalize_forcings(forc)
            s0 = gcm.encoder(ss.scatter_fields(norm, gcm.shard), f)
            outs = []
            for fsdp in (False, True):
                if fsdp:
                    gcm.model.parameterization.shard_tower_weights()
                s = s0
                for _ in range(3):
                    s = gcm.model.step(s, f)
                outs.append(gcm.decoder(s, f))
        err = max(_rel(outs[1][k], outs[0][k]) for k in outs[0])
        # sharded save of the tower: each rank's rows only; the all-gather restores the weights
        from tornado_gcm_b200.parallel.fsdp_gather import local_state_dict
        from tornado_gcm_b200.training import sharded_checkpoint as sc

        par = gcm.model.parameterization
        names = [f"layers.{i}" for i in range(len(par._fsdp_layers))]
        local, meta = local_state_dict(par._fsdp_layers, names)
        full = sc.all_gather_state_dict({k: v.to(dev) for k, v in local.items()}, meta)
        ref = par.tower.neural_net.state_dict()
        # weights live as BF16 shards, biases in fp32
        err_ckpt = max(_rel(full[k].float(), (ref[k].to(torch.bfloat16) if k.endswith("weight") else ref[k])
                            .float().to(dev)) for k in full)
        err = max(err, err_ckpt)
        torch.cuda.synchronize(dev)
        q.put((rank, err, _ext.check_error_flag(dev)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fsdp_tower_weights_match_replicated_weights():
    """Sharded model with the tower's weights FSDP-sharded (GEMMs read peer rows as they run)
    gives the decoded forecast of the replicated-weight run."""
    for _, err, flag in _spawn(_worker_fsdp, 2):
        assert flag == 0
        assert err < 1e-3
