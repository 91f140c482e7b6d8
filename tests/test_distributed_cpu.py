"""Multi-process host logic on CPU ranks (gloo): gradient averaging, the packed
metric all-reduce, and failure detection by host-side injection (a rank that
raises before a collective; the survivors' collective ends with an error
instead of hanging)."""

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


def _free_port_pair() -> int:
    """A port p with p and p + 1 both free (the recovery test re-forms its group on p + 1)."""
    for _ in range(200):
        p = _free_port()
        try:
            with socket.socket() as a, socket.socket() as b:
                a.bind(("127.0.0.1", p))
                b.bind(("127.0.0.1", p + 1))
            return p
        except OSError:
            continue
    raise RuntimeError("no pair of adjacent free ports")


def _init(rank, world, port, timeout_s=30.0):
    """Gloo group whose collectives time out after ``timeout_s``.  The ranks first meet on the
    store with a generous limit (spawned ranks can take many seconds to import torch on a busy
    machine), so that a short collective timeout does not also cut the rendezvous short."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=120))
    store.set(f"up{rank}", "1")
    store.wait([f"up{r}" for r in range(world)])
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _worker_reduce(rank, world, port, q):
    try:
        _init(rank, world, port)
        from tornado_gcm_b200.parallel.ddp import GradientAllReducer
        from tornado_gcm_b200.parallel.metrics import all_reduce_metrics

        torch.manual_seed(0)
        model = torch.nn.Sequential(torch.nn.Linear(5, 7), torch.nn.Linear(7, 3))
        red = GradientAllReducer(list(model.parameters()), bucket_mb=0.0001)
        red.broadcast_parameters()
        red.zero()
        x = torch.full((4, 5), float(rank + 1))
        model(x).sum().backward()
        local = [p.grad.clone() for p in model.parameters()]
        red.reduce()
        gathered = [torch.zeros_like(t) for t in local for _ in range(1)]
        sums = []
        for t in local:
            tt = t.clone()
            dist.all_reduce(tt)
            sums.append(tt / world)
        ok_grads = all(torch.allclose(p.grad, s, atol=1e-6) for p, s in zip(model.parameters(), sums))
        m = all_reduce_metrics({"loss": torch.tensor(float(rank)), "n": 2.0})
        q.put((rank, ok_grads, m["loss"], m["n"], len(gathered)))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))


def test_gradient_allreducer_and_metrics_gloo():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_reduce, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert len(r) == 5, r[1]
        _, ok, loss, n, _ = r
        assert ok
        assert loss == pytest.approx(0.5)
        assert n == pytest.approx(2.0)


def _worker_failure(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5.0)
        t = torch.ones(3)
        dist.all_reduce(t)  # both ranks healthy here
        if rank == 1:
            raise RuntimeError("injected failure on rank 1")
        try:
            dist.all_reduce(t)  # rank 1 never joins: must end with an error, not hang
            q.put((rank, "completed"))
        except Exception as exc:
            q.put((rank, "error:" + type(exc).__name__))
    except RuntimeError as exc:
        q.put((rank, "raised:" + str(exc)))


def test_peer_failure_surfaces_as_error_not_hang():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_failure, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():  # pragma: no cover
            p.kill()
    assert res[1].startswith("raised:")
    assert res[0].startswith("error:")


def _worker_elastic(rank, world, port, ckpt_dir, q):
    try:
        import torch.distributed as dist

        from tornado_gcm_b200.parallel.elastic import maybe_inject_fault, run_with_recovery

        def train(hb, r, w, attempt):
            path = os.path.join(ckpt_dir, "state.pt")
            start, acc = 0, torch.zeros(1)
            if os.path.exists(path):
                ck = torch.load(path)
                start, acc = ck["step"] + 1, ck["acc"]
            for step in range(start, 6):
                if attempt == 0:
                    maybe_inject_fault(rank, step, "2:3:exit")   # original rank 2 dies before step 3
                hb.beat(step)
                hb.check(step)                                   # host-side detection before the collective
                t = torch.ones(1)
                dist.all_reduce(t)
                acc = acc + t
                if r == 0:
                    torch.save({"step": step, "acc": acc}, path + ".tmp")
                    os.replace(path + ".tmp", path)
                dist.barrier()
            return float(acc)

        out = run_with_recovery(train, rank, world, "127.0.0.1", port, heartbeat_timeout_s=3.0)
        q.put((rank, out))
    except Exception:  # pragma: no cover
        q.put((rank, traceback.format_exc()))


def test_rank_failure_detected_and_survivors_resume(tmp_path):
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port_pair()
    procs = [ctx.Process(target=_worker_elastic, args=(r, world, port, str(tmp_path), q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world - 1)]
    for p in procs:
        p.join(timeout=60)
    assert procs[2].exitcode == 17
    for rank, out in res:
        assert isinstance(out, dict), out
        assert out["attempts"] == 2 and out["world"] == 2
        # steps 0-2 summed over 3 ranks, steps 3-5 over the 2 survivors
        assert out["result"] == 3 * 3 + 3 * 2


def test_transport_selection_on_cpu():
    from tornado_gcm_b200.parallel.transport import GlooTransport, NVLinkTransport, get_transport

    assert isinstance(get_transport("auto", device="cpu"), GlooTransport)
    assert isinstance(get_transport("nvlink"), NVLinkTransport)
    with pytest.raises(ValueError):
        get_transport("carrier-pigeon")
    t = get_transport("gloo")
    red = t.gradient_reducer(10, "cpu")
    red.flat.fill_(3.0)
    red.all_reduce_mean(red.flat)  # one process: unchanged
    assert float(red.flat.sum()) == 30.0
