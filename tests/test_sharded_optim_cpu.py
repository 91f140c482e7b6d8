"""Sharded data parallelism (gradients and AdamW state split over the ranks) on gloo CPU ranks.

The trainer with ``data_parallel="sharded"`` must follow the replicated data-parallel
trainer step for step: same losses, same weights on every rank (reduce-scatter of the
mean gradient, clipping by the global norm, AdamW on each rank's chunk, all-gather).
Two and three ranks; three leaves a padded tail in the flat buffers.
"""

import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


class _Toy(torch.nn.Module):
    """A stand-in for the hybrid GCM: the trainer needs ``loss(data0, targets, forcings)``."""

    def __init__(self):
        super().__init__()
        self.a = torch.nn.Linear(5, 7)
        self.b = torch.nn.Linear(7, 3)
        self.scale = torch.nn.Parameter(torch.ones(3))

    def loss(self, data0, targets, forcings):
        x = data0["x"]
        for t in targets:
            x = torch.tanh(self.b(torch.tanh(self.a(x))) * self.scale) @ forcings["w"]
            x = x + t["x"] * 0.1
        return (x * x).mean()


def _batch(rank, step):
    g = torch.Generator().manual_seed(1000 * step + rank)
    data0 = {"x": torch.randn(6, 5, generator=g)}
    targets = [{"x": torch.randn(6, 5, generator=g)} for _ in range(2)]
    forc = {"w": torch.randn(3, 5, generator=g) * 0.5}
    return data0, targets, forc


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        from tornado_gcm_b200.training.trainer import GCMTrainer

        torch.manual_seed(0)
        m_rep = _Toy()
        m_sh = _Toy()
        m_sh.load_state_dict(m_rep.state_dict())
        if rank > 0:  # the sharded path must start every rank from rank 0's weights
            with torch.no_grad():
                for p in m_sh.parameters():
                    p.add_(float(rank))
        # a clip threshold low enough to be active
        t_rep = GCMTrainer(m_rep, lr=1e-2, weight_decay=0.01, max_grad_norm=0.05, data_parallel=True)
        t_sh = GCMTrainer(m_sh, lr=1e-2, weight_decay=0.01, max_grad_norm=0.05, data_parallel="sharded")
        errs, losses = [], []
        for step in range(4):
            b = _batch(rank, step)
            l1 = float(t_rep.train_step(*b))
            l2 = float(t_sh.train_step(*b))
            losses.append(abs(l1 - l2))
            errs.append(max(float((p - s).abs().max()) for p, s in zip(m_rep.parameters(), m_sh.parameters())))
        # every rank holds the same gathered weights
        flat = torch.cat([p.detach().reshape(-1) for p in m_sh.parameters()])
        parts = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(parts, flat)
        spread = max(float((x - parts[0]).abs().max()) for x in parts)
        # the moments are 1/world of the model (one padded chunk per rank)
        st = t_sh.zero_opt.optimizer.state[t_sh.zero_opt.shard]
        q.put((rank, {"errs": errs, "loss": losses, "spread": spread, "chunk": t_sh.zero_opt.chunk,
                      "numel": t_sh.zero_opt.numel, "moment": int(st["exp_avg"].numel()),
                      "backend": t_sh.grad_reducer}))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_optimizer_matches_replicated_dp(world):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, r in res:
        assert isinstance(r, dict), r
        assert max(r["errs"]) < 2e-6, r["errs"]
        assert max(r["loss"]) < 1e-6
        assert r["spread"] == 0.0
        assert r["chunk"] * world >= r["numel"] and r["chunk"] % 4 == 0
        assert r["moment"] == r["chunk"]
        assert r["backend"].startswith("sharded optimizer: gloo")


def test_sharded_optimizer_single_rank_is_adamw_with_clipping():
    """One process without a process group: ShardedAdamW == clip_grad_norm_ + AdamW."""
    from tornado_gcm_b200.parallel.sharded_optim import ShardedAdamW

    torch.manual_seed(1)
    a, b = _Toy(), _Toy()
    b.load_state_dict(a.state_dict())
    ref = torch.optim.AdamW(a.parameters(), lr=1e-2, weight_decay=0.01, betas=(0.9, 0.95), eps=1e-6)
    opt = ShardedAdamW(list(b.parameters()), lr=1e-2, weight_decay=0.01, max_grad_norm=0.05)
    for step in range(3):
        data = _batch(0, step)
        ref.zero_grad()
        a.loss(*data).backward()
        torch.nn.utils.clip_grad_norm_(a.parameters(), 0.05)
        ref.step()
        opt.zero_grad()
        b.loss(*data).backward()
        opt.step()
        for p, s in zip(a.parameters(), b.parameters()):
            torch.testing.assert_close(p, s, atol=1e-6, rtol=1e-6)


def test_sharded_optimizer_state_round_trip():
    """The optimizer shard saves and loads its moments; a shard of another layout is refused."""
    from tornado_gcm_b200.parallel.sharded_optim import ShardedAdamW

    torch.manual_seed(2)
    m = _Toy()
    opt = ShardedAdamW(list(m.parameters()), lr=1e-2)
    opt.zero_grad()
    m.loss(*_batch(0, 0)).backward()
    opt.step()
    sd = opt.state_dict()
    assert sd["world"] == 1 and sd["chunk"] == opt.chunk and sd["numel"] == opt.numel
    m2 = _Toy()
    opt2 = ShardedAdamW(list(m2.parameters()), lr=1e-2)
    opt2.load_state_dict(sd)
    a = opt.optimizer.state[opt.shard]["exp_avg"]
    b = opt2.optimizer.state[opt2.shard]["exp_avg"]
    torch.testing.assert_close(a, b)
    bad = dict(sd, chunk=sd["chunk"] + 4)
    with pytest.raises(ValueError):
        opt2.load_state_dict(bad)


def _worker_full_state(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        from tornado_gcm_b200.parallel.sharded_optim import ShardedAdamW

        torch.manual_seed(0)
        m_sh, m_rep = _Toy(), _Toy()
        m_rep.load_state_dict(m_sh.state_dict())
        opt = ShardedAdamW(list(m_sh.parameters()), lr=1e-2, weight_decay=0.01, max_grad_norm=None)
        for step in range(2):
            opt.zero_grad()
            m_sh.loss(*_batch(0, step)).backward()    # same data on every rank: the mean is that gradient
            opt.step()
        full = opt.full_state_dict()
        # a replicated AdamW resumes from the gathered state and matches one more sharded step
        with torch.no_grad():
            for a, b in zip(m_rep.parameters(), m_sh.parameters()):
                a.copy_(b)
        ref_opt = torch.optim.AdamW(m_rep.parameters(), lr=1e-2, weight_decay=0.01, betas=(0.9, 0.95), eps=1e-6)
        ref_opt.load_state_dict(full)
        for o, model in ((opt, m_sh), (ref_opt, m_rep)):
            o.zero_grad()
            model.loss(*_batch(0, 2)).backward()
            o.step()
        err = max(float((a - b).abs().max()) for a, b in zip(m_rep.parameters(), m_sh.parameters()))
        # and the sharded optimizer takes the full state back
        opt2 = ShardedAdamW(list(_Toy().parameters()), lr=1e-2)
        opt2.load_full_state_dict(full)
        mom = opt2.optimizer.state[opt2.shard]["exp_avg"]
        q.put((rank, err, len(full["state"]), int(mom.numel() == opt2.chunk)))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        q.put((rank, traceback.format_exc()))


def test_sharded_optimizer_full_state_round_trip():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_full_state, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert not isinstance(r[1], str), r[1]
        _, err, n, ok = r
        assert err < 1e-6 and n == 5 and ok       # five parameters in the toy model


def _worker_sda_sharded(rank, world, port, path, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        from tornado_gcm_b200.models.builders import build_hybrid_gcm
        from tornado_gcm_b200.precision.sda import SDAConfig
        from tornado_gcm_b200.training.sda_trainer import SDATrainer

        cfg = SDAConfig()
        cfg.training.rollout_steps = 1
        cfg.training.batch_size = 1
        gcm, _ = build_hybrid_gcm("5.6deg", "cpu", seed=0)
        tr = SDATrainer(gcm, cfg, total_steps=2, data_parallel="sharded")
        hist = tr.fit(log_every=1)
        tr.save_checkpoint(path)                  # collective gather; rank 0 writes
        dist.barrier()
        tr.load_checkpoint(path)
        flat = torch.cat([p.detach().reshape(-1) for p in gcm.parameters()])
        parts = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(parts, flat)
        q.put((rank, float(hist[-1]["loss"]), float(max((x - parts[0]).abs().max() for x in parts)),
               tr._trainer.grad_reducer))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        q.put((rank, traceback.format_exc()))


def test_sda_trainer_sharded_checkpoint_round_trip(tmp_path):
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    path = str(tmp_path / "sda.pt")
    procs = [ctx.Process(target=_worker_sda_sharded, args=(r, world, port, path, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    losses = set()
    for r in res:
        assert not isinstance(r[1], str), r[1]
        _, loss, spread, backend = r
        losses.add(round(loss, 6))
        assert spread == 0.0 and backend.startswith("sharded optimizer")
    assert len(losses) == 2                         # each rank trained on its own samples
    ck = torch.load(path, weights_only=False)
    assert len(ck["optimizer_state_dict"]["state"]) > 0
