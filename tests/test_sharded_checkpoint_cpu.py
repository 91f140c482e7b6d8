"""Sharded (row-sharded, FSDP-style) checkpoints on gloo ranks: every rank saves only its
rows, the files gather back into the full state dict, the online all-gather gives the
same dict on every rank, and a full checkpoint loads back into the ranks' shards."""

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


def _model_sd():
    torch.manual_seed(3)
    m = torch.nn.Sequential(torch.nn.Linear(21, 37), torch.nn.GELU(), torch.nn.Linear(37, 5),
                            torch.nn.Linear(5, 70))
    sd = dict(m.state_dict())
    sd["stats.mean"] = torch.randn(7)
    return sd


def _worker(rank, world, port, directory, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
        from tornado_gcm_b200.training import sharded_checkpoint as sc

        full = _model_sd()
        local, meta = sc.shard_state_dict(full, rank, world)
        held = sum(v.numel() for k, v in local.items() if meta[k]["sharded"])
        sc.save_sharded(directory, local, meta, rank, world, extra={"step": 12})
        dist.barrier()
        online = sc.all_gather_state_dict(local, meta)
        ok_online = all(torch.equal(online[k], full[k]) for k in full)
        back = sc.load_full_into_shards(full, meta, rank)
        ok_back = all(torch.equal(back[k], local[k]) for k in local)
        q.put((rank, ok_online, ok_back, held))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover - reported to the parent
        q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_save_and_gather(world, tmp_path):
    from tornado_gcm_b200.training import sharded_checkpoint as sc

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path), q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert len(r) == 4, r[1]
        assert r[1] and r[2], r
    full = _model_sd()
    n_weights = sum(v.numel() for k, v in full.items() if v.dim() >= 2)
    assert sum(r[3] for r in res) == n_weights  # every weight row is held by exactly one rank
    gathered = sc.gather_sharded(tmp_path)
    assert set(gathered) == set(full)
    for k in full:
        assert torch.equal(gathered[k], full[k]), k


def test_row_rule_matches_the_gathered_linear_layout():
    from tornado_gcm_b200.training import sharded_checkpoint as sc

    # 193 output rows over 8 ranks: 25 -> 32 rows per rank, ranks 6 and 7 hold 1 and 0 rows
    per = sc.shard_rows(193, 8)
    assert per == 32
    assert sc.row_range(193, 6, per) == (192, 193)
    assert sc.row_range(193, 7, per) == (193, 193)
