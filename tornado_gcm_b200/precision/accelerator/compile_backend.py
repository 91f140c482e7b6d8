"""Execution-backend plumbing — reference ``precision/accelerator/compile_backend.py:34-207``.

The reference registers ``State`` as a pytree for dynamo, sets dynamo
options and benchmarks compiled against eager steps.  This framework runs
no tracing compiler: its equivalents are the pytree registration (useful
for ``torch.utils._pytree`` tooling), the matmul-precision switches that
PyTorch's own GEMMs obey, and a graph-versus-eager step benchmark timed
with CUDA events.
"""

from __future__ import annotations

import time
from typing import Any

import torch

_PYTREE_REGISTERED = False


def register_state_pytree() -> None:
    global _PYTREE_REGISTERED
    if _PYTREE_REGISTERED:
        return
    import torch.utils._pytree as pytree

    from tornado_gcm_b200.core.primitive_equations import State

    def flatten(s):
        keys = tuple(sorted(s.tracers))
        children = [s.vorticity, s.divergence, s.temperature_variation, s.log_surface_pressure]
        children += [s.tracers[k] for k in keys]
        return children, (keys, s.sim_time)

    def unflatten(children, ctx):
        keys, sim = ctx
        return State(children[0], children[1], children[2], children[3], dict(zip(keys, children[4:])), sim)

    try:
        pytree.register_pytree_node(State, flatten, unflatten)
    except ValueError:  # already registered by another import path
        pass
    _PYTREE_REGISTERED = True


def configure_matmul_precision(allow_tf32: bool = True, allow_fp16_accumulation: bool = False,
                               deterministic: bool = False) -> None:
    """TF32 and reduced-precision-reduction switches for PyTorch's own matmuls and convolutions
    (the sm_100a kernels choose their precision per zone)."""
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = allow_fp16_accumulation
    torch.backends.cuda.matmul.allow_tf32 = allow_tf32
    torch.backends.cudnn.allow_tf32 = allow_tf32
    torch.set_float32_matmul_precision("high" if allow_tf32 else "highest")
    if deterministic:
        torch.use_deterministic_algorithms(True, warn_only=True)


def configure_dynamo(*_args, **_kwargs) -> dict:
    """No tracing compiler is used; returns the (empty) option set for API parity."""
    return {}


def benchmark_graph(model, state, forcings=None, steps: int = 10, warmup: int = 3) -> dict[str, Any]:
    """Mean ms per outer step, eager versus CUDA-graph replay (CUDA events)."""
    from tornado_gcm_b200.precision.accelerator.graphed_step import FusedAdvanceKernel

    if not state.vorticity.is_cuda:
        t0 = time.perf_counter()
        with torch.no_grad():
            s = state
            for _ in range(steps):
                s = model.step(s, forcings)
        return {"eager_ms": 1000.0 * (time.perf_counter() - t0) / steps, "graph_ms": None, "speedup": None}

    def timed(fn):
        with torch.no_grad():
            s = state
            for _ in range(warmup):
                s = fn(s, forcings)
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(steps):
                s = fn(s, forcings)
            b.record()
            torch.cuda.synchronize()
        return a.elapsed_time(b) / steps

    eager = timed(model.step)
    graph = timed(FusedAdvanceKernel(model))
    return {"eager_ms": eager, "graph_ms": graph, "speedup": eager / graph if graph else None}


benchmark_compile = benchmark_graph
