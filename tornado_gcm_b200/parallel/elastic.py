"""Rank-failure detection, host-side fault injection and restart from checkpoint.

The reference has no rank-failure detection (its recovery is limited to NaN
roll-back).  Here:

* :class:`Heartbeat` — every rank writes ``(step, wall time)`` into the
  process group's key-value store between steps; before the next collective
  each rank checks every peer's entry.  A peer that has not advanced within
  ``timeout_s`` (or that wrote a ``left`` marker) raises
  :class:`RankFailureError` on the host, BEFORE any kernel or collective of
  that step is launched, so no GPU ever waits on a dead peer.  The process
  group's own (short) timeout is the second line of defence for a rank that
  dies inside a collective.
* :func:`maybe_inject_fault` — host-side fault injection driven by the
  ``TGCM_FAULT_INJECT`` environment variable (``"<rank>:<step>:<kind>"``,
  kind ``raise`` | ``exit`` | ``hang_host``): the chosen rank raises, exits
  without finishing, or stops beating (sleeps on the host).  Nothing is
  injected on the device.
* :func:`run_with_recovery` — runs a training function; on a rank failure
  the survivors tear down the process group, rendezvous again without the
  failed rank and resume from the last checkpoint.

All of it works over gloo on CPU ranks, which is how it is tested.
"""

from __future__ import annotations

import datetime
import json
import logging
import os
import time
from typing import Callable, Optional

import torch.distributed as dist

logger = logging.getLogger(__name__)

FAULT_ENV = "TGCM_FAULT_INJECT"


class RankFailureError(RuntimeError):
    def __init__(self, dead_ranks, step=None):
        self.dead_ranks = sorted(dead_ranks)
        self.step = step
        super().__init__(f"ranks {self.dead_ranks} stopped responding (step {step})")


class InjectedFault(RuntimeError):
    pass


def parse_fault_spec(spec: Optional[str]) -> Optional[tuple]:
    if not spec:
        return None
    rank, step, kind = spec.split(":")
    if kind not in ("raise", "exit", "hang_host"):
        raise ValueError(f"unknown fault kind {kind!r}")
    return int(rank), int(step), kind


def maybe_inject_fault(rank: int, step: int, spec: Optional[str] = None) -> None:
    """Inject the configured host-side fault when ``(rank, step)`` matches."""
    f = parse_fault_spec(spec if spec is not None else os.environ.get(FAULT_ENV))
    if f is None or f[0] != rank or f[1] != step:
        return
    kind = f[2]
    logger.warning("injecting fault %s on rank %d at step %d", kind, rank, step)
    if kind == "raise":
        raise InjectedFault(f"injected failure on rank {rank} at step {step}")
    if kind == "exit":
        os._exit(17)
    time.sleep(3600.0)  # hang_host: stop beating; peers detect it through the heartbeat


class Heartbeat:
    """Store-based liveness check between steps."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0, prefix: str = "tgcm_hb"):
        self.store = store
        self.rank = rank
        self.world = world
        self.timeout_s = float(timeout_s)
        self.prefix = prefix
        self._seen: dict = {}

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self, step: int) -> None:
        self.store.set(self._key(self.rank), json.dumps({"step": int(step), "t": time.time()}))

    def leave(self) -> None:
        """Announce an orderly exit (peers treat it as a failure at once)."""
        self.store.set(self._key(self.rank), json.dumps({"step": -1, "t": time.time(), "left": True}))

    def _read(self, r: int):
        try:
            if not self.store.check([self._key(r)]):
                return None
            return json.loads(self.store.get(self._key(r)).decode())
        except Exception:  # noqa: BLE001 - a store error is a failure signal too
            return {"left": True}

    def check(self, step: int, wait: bool = True) -> None:
        """Raise :class:`RankFailureError` if a peer has not reached ``step``.

        With ``wait`` the call polls until every peer has reached ``step`` or
        ``timeout_s`` passes (peers that are merely slower are waited for).
        """
        t0 = time.time()
        while True:
            late, dead = [], []
            for r in range(self.world):
                if r == self.rank:
                    continue
                rec = self._read(r)
                if rec is not None and rec.get("left"):
                    dead.append(r)
                elif rec is None or rec["step"] < step:
                    late.append(r)
            if dead:
                raise RankFailureError(dead, step)
            if not late:
                return
            if not wait or time.time() - t0 > self.timeout_s:
                raise RankFailureError(late, step)
            time.sleep(0.01)


def init_group(rank: int, world: int, addr: str, port: int, backend: str = "gloo", timeout_s: float = 30.0,
               store=None):
    """Process group with a short collective timeout and a TCP store for heartbeats."""
    if store is None:
        store = dist.TCPStore(addr, port, world, rank == 0, timeout=datetime.timedelta(seconds=timeout_s))
    dist.init_process_group(backend, store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return store


def run_with_recovery(train_fn: Callable, rank: int, world: int, addr: str, base_port: int,
                      max_restarts: int = 2, backend: str = "gloo", heartbeat_timeout_s: float = 10.0,
                      survivors_fn: Optional[Callable] = None) -> dict:
    """Run ``train_fn(heartbeat, rank, world, attempt)``; on :class:`RankFailureError`, re-form the
    group from the survivors on ``base_port + attempt`` and call it again (it resumes from its checkpoint).

    Survivor ranks are renumbered densely in their old order.  ``survivors_fn(dead)`` may
    override which old ranks continue.  Returns ``{"attempts", "rank", "world", "result"}``.
    """
    attempt, cur_rank, cur_world = 0, rank, world
    while True:
        store = init_group(cur_rank, cur_world, addr, base_port + attempt, backend)
        hb = Heartbeat(store, cur_rank, cur_world, heartbeat_timeout_s, prefix=f"tgcm_hb{attempt}")
        try:
            result = train_fn(hb, cur_rank, cur_world, attempt)
            dist.barrier()
            dist.destroy_process_group()
            return {"attempts": attempt + 1, "rank": cur_rank, "world": cur_world, "result": result}
        except RankFailureError as exc:
            logger.warning("rank %d: %s; re-forming the group", cur_rank, exc)
            try:
                dist.destroy_process_group()
            except Exception:  # noqa: BLE001
                pass
            if attempt >= max_restarts:
                raise
            alive = [r for r in range(cur_world) if r not in exc.dead_ranks]
            if survivors_fn is not None:
                alive = survivors_fn(exc.dead_ranks)
            cur_rank, cur_world = alive.index(cur_rank), len(alive)
            attempt += 1
