"""Whole-step CUDA graphs for inference — the role of reference
``precision/accelerator/fused_zone_cast.py:33-147`` (``FusedAdvanceKernel``).

The reference hands ``model.step`` to ``torch.compile``.  Here the step is
already made of a fixed sequence of sm_100a kernels, so the B200 way to
remove its launch and host overhead is to capture one outer step into a
CUDA graph and replay it:

* inputs are copied into static buffers, the graph is replayed, and the
  outputs are cloned out of the graph's private pool;
* one graph per (shapes, dtypes, tracer keys, fixer phase); the fixer
  cadence (a Python-side counter in the model) is honoured by capturing one
  graph per phase ``step_count % cadence``;
* parameters are watched through their version counters; a change (load,
  hot-swap, optimizer step) drops the graphs;
* grad-enabled calls, CPU tensors and capture failures run eagerly.
"""

from __future__ import annotations

import logging
from typing import Any, Optional

import torch
import torch.nn as nn

logger = logging.getLogger(__name__)


def _flatten(obj, out: list):
    if torch.is_tensor(obj):
        out.append(obj)
    elif hasattr(obj, "tensors") and hasattr(obj, "tracers"):
        out.extend(obj.tensors())
    elif isinstance(obj, dict):
        for k in sorted(obj):
            _flatten(obj[k], out)
    elif isinstance(obj, (list, tuple)):
        for v in obj:
            _flatten(v, out)
    return out


def _signature(state, forcings) -> tuple:
    ts = _flatten(state, []) + _flatten(forcings, [])
    keys = tuple(sorted(state.tracers)) if hasattr(state, "tracers") else ()
    fkeys = tuple(sorted(forcings)) if isinstance(forcings, dict) else ()
    return keys, fkeys, tuple((tuple(t.shape), t.dtype, str(t.device)) for t in ts)


class FusedAdvanceKernel:
    """Callable ``(state, forcings) → next state`` backed by CUDA graphs."""

    def __init__(self, model: nn.Module, policy: Any = None, compile_mode: str = "cuda_graph",
                 dynamic: bool = False, fallback_on_error: bool = True, warmup_steps: int = 2):
        self._model = model
        self._policy = policy
        self._compile_mode = compile_mode
        self._fallback = fallback_on_error
        self._warmup = max(1, int(warmup_steps))
        self._graphs: dict = {}
        self._param_versions: Optional[tuple] = None
        self._using_eager = False
        self._call_count = 0
        self._replays = 0
        self._pool = None

    # ── helpers ──
    def _versions(self) -> tuple:
        return tuple(p._version for p in self._model.parameters())

    def _cadence(self) -> int:
        return max(1, int(getattr(self._model, "_fixer_cadence", 1)))

    def _capture(self, state, forcings, phase: int):
        model = self._model
        static_state = state.tree_map(lambda t: t.clone())
        static_forc = None if forcings is None else {k: (v.clone() if torch.is_tensor(v) else v)
                                                     for k, v in forcings.items()}
        saved_count = model._step_count
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(self._warmup):  # allocator and lazy caches warm up outside the graph
                model._step_count = phase
                model.step(static_state, static_forc)
        torch.cuda.current_stream().wait_stream(side)
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        graph = torch.cuda.CUDAGraph()
        model._step_count = phase
        with torch.cuda.graph(graph, pool=self._pool):
            static_out = model.step(static_state, static_forc)
        model._step_count = saved_count
        return graph, static_state, static_forc, static_out

    # ── API ──
    def __call__(self, state: Any, forcings: Any = None) -> Any:
        self._call_count += 1
        model = self._model
        if (self._using_eager or torch.is_grad_enabled() or not hasattr(state, "vorticity")
                or not state.vorticity.is_cuda):
            return model.step(state, forcings)
        ver = self._versions()
        if ver != self._param_versions:
            self._graphs.clear()
            self._param_versions = ver
        phase = model._step_count % self._cadence()
        key = (_signature(state, forcings), phase)
        ent = self._graphs.get(key)
        if ent is None:
            try:
                ent = self._capture(state, forcings, phase)
            except Exception as exc:
                if not self._fallback:
                    raise
                logger.warning("FusedAdvanceKernel: capture failed (%s); running eagerly", exc)
                self._using_eager = True
                return model.step(state, forcings)
            self._graphs[key] = ent
        graph, s_in, f_in, s_out = ent
        for dst, src in zip(s_in.tensors(), state.tensors()):
            dst.copy_(src)
        if f_in is not None:
            for k, v in f_in.items():
                if torch.is_tensor(v):
                    v.copy_(forcings[k])
        graph.replay()
        self._replays += 1
        model._step_count += 1
        out = s_out.tree_map(lambda t: t.clone())
        sim = None if state.sim_time is None else state.sim_time + model.config.dt
        return type(out)(out.vorticity, out.divergence, out.temperature_variation, out.log_surface_pressure,
                         out.tracers, sim)

    def reset(self) -> None:
        self._graphs.clear()
        self._param_versions = None
        self._using_eager = False
        self._call_count = 0
        self._replays = 0

    @property
    def is_compiled(self) -> bool:
        return bool(self._graphs) and not self._using_eager

    @property
    def is_eager(self) -> bool:
        return self._using_eager

    def stats(self) -> dict:
        return {"call_count": self._call_count, "is_compiled": self.is_compiled, "is_eager": self.is_eager,
                "compile_mode": self._compile_mode, "graphs": len(self._graphs), "replays": self._replays}
