"""Benchmark utilities — reference ``precision/benchmarks.py:41-231``.

* :class:`TimingBenchmark` — CUDA-event (or wall-clock on CPU) timing with
  warm-up, mean/std/min/max report;
* :class:`MemoryBenchmark` — peak-allocation measurement;
* :class:`StorageBenchmark` — write/read throughput of the storage manager;
* :class:`PrecisionBenchmark` — the class the reference CLI's ``benchmark``
  command calls (``cli.py:140``) but never defines: one outer model step per
  precision policy (PZHA-B200, FP32 Z1, full FP64 fixer), timed, with the
  state drift against the highest-precision run.

Kernel micro-benchmarks (used for profiler captures on small cases)::

    python -m tornado_gcm_b200.precision.benchmarks mlp --tokens 32768 --width 384
    python -m tornado_gcm_b200.precision.benchmarks sht --grid TL63 --slices 1292
    python -m tornado_gcm_b200.precision.benchmarks stage --grid TL63 --batch 4
    python -m tornado_gcm_b200.precision.benchmarks linear --mode dgrad --tokens 32768 --width 384 --cycles
    python -m tornado_gcm_b200.precision.benchmarks bgemm --groups 1292 --m 128 --n 64 --k 128 --cycles
"""

from __future__ import annotations

import argparse
import dataclasses
import gc
import json
import statistics
import time
from typing import Any, Callable, Optional

import torch


@dataclasses.dataclass
class BenchmarkResult:
    name: str
    mean_ms: float
    std_ms: float
    min_ms: float
    max_ms: float
    iterations: int
    extra: dict = dataclasses.field(default_factory=dict)


class TimingBenchmark:
    def __init__(self, warmup: int = 3, iterations: int = 10, use_cuda_events: bool = True) -> None:
        self._warmup = warmup
        self._iterations = iterations
        self._use_cuda = use_cuda_events and torch.cuda.is_available()
        self._results: list[BenchmarkResult] = []

    def time_fn(self, name: str, fn: Callable, *args: Any, **kwargs: Any) -> BenchmarkResult:
        for _ in range(self._warmup):
            fn(*args, **kwargs)
        if self._use_cuda:
            torch.cuda.synchronize()
        times = []
        for _ in range(self._iterations):
            if self._use_cuda:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                fn(*args, **kwargs)
                b.record()
                torch.cuda.synchronize()
                times.append(a.elapsed_time(b))
            else:
                t0 = time.perf_counter()
                fn(*args, **kwargs)
                times.append(1000.0 * (time.perf_counter() - t0))
        r = BenchmarkResult(name, round(statistics.mean(times), 4),
                            round(statistics.stdev(times), 4) if len(times) > 1 else 0.0,
                            round(min(times), 4), round(max(times), 4), self._iterations)
        self._results.append(r)
        return r

    def report(self) -> str:
        lines = ["=" * 70, "Performance Benchmark Report", "=" * 70]
        for r in self._results:
            lines.append(f"  {r.name:<30s}  mean={r.mean_ms:8.3f}ms  std={r.std_ms:7.3f}ms  "
                         f"min={r.min_ms:8.3f}ms  max={r.max_ms:8.3f}ms  (n={r.iterations})")
        lines.append("=" * 70)
        return "\n".join(lines)

    @property
    def results(self) -> list[BenchmarkResult]:
        return list(self._results)


class MemoryBenchmark:
    @staticmethod
    def measure(fn: Callable, *args: Any, device: str = "cuda", **kwargs: Any) -> dict:
        if device == "cuda" and torch.cuda.is_available():
            gc.collect()
            torch.cuda.empty_cache()
            torch.cuda.reset_peak_memory_stats()
            before = torch.cuda.memory_allocated() / 2 ** 20
            fn(*args, **kwargs)
            torch.cuda.synchronize()
            after = torch.cuda.memory_allocated() / 2 ** 20
            peak = torch.cuda.max_memory_allocated() / 2 ** 20
            return {"before_mb": round(before, 2), "after_mb": round(after, 2), "peak_mb": round(peak, 2),
                    "delta_mb": round(after - before, 2)}
        import tracemalloc

        tracemalloc.start()
        fn(*args, **kwargs)
        cur, peak = tracemalloc.get_traced_memory()
        tracemalloc.stop()
        return {"current_mb": round(cur / 2 ** 20, 2), "peak_mb": round(peak / 2 ** 20, 2)}


class StorageBenchmark:
    @staticmethod
    def measure_write_throughput(manager: Any, variables: dict, output_dir: str, iterations: int = 5) -> dict:
        total = sum(t.numel() * t.element_size() for t in manager._flatten(variables).values())
        times, written = [], 0
        for i in range(iterations):
            t0 = time.perf_counter()
            summ = manager.write(variables, output_dir, step=i)
            times.append(time.perf_counter() - t0)
            written = sum(v["size_bytes"] for v in summ.values())
        mean = statistics.mean(times)
        return {"mean_s": round(mean, 5), "throughput_mb_s": round(total / 2 ** 20 / mean, 2),
                "compression_ratio": round(written / max(total, 1), 4)}

    @staticmethod
    def measure_read_throughput(manager: Any, input_dir: str, iterations: int = 5, step: int = 0) -> dict:
        times = []
        for _ in range(iterations):
            t0 = time.perf_counter()
            manager.read(input_dir, step=step)
            times.append(time.perf_counter() - t0)
        return {"mean_s": round(statistics.mean(times), 5)}


@dataclasses.dataclass
class PrecisionBenchmarkResult:
    rows: list

    def report(self) -> str:
        lines = ["=" * 78, "Precision benchmark (one outer step per policy)", "=" * 78,
                 f"  {'policy':<22s} {'ms/step':>10s} {'rel. drift vs FP64 ref':>24s}"]
        for r in self.rows:
            d = "-" if r["drift"] is None else f"{r['drift']:.3e}"
            lines.append(f"  {r['policy']:<22s} {r['ms']:10.3f} {d:>24s}")
        lines.append("=" * 78)
        return "\n".join(lines)

    def to_dict(self) -> dict:
        return {"rows": self.rows}


class PrecisionBenchmark:
    """Time one outer step of the hybrid model under several precision policies.

    The highest-precision policy (FP64 transforms) is the drift reference; each
    other policy's state after ``n_steps`` outer steps is compared with it.
    """

    def __init__(self, sda_config=None, device: str = "cuda", n_steps: int = 2, resolution: Optional[str] = None,
                 batch: int = 1):
        self.sda_config = sda_config
        self.device = torch.device(device if (device != "cuda" or torch.cuda.is_available()) else "cpu")
        self.n_steps = int(n_steps)
        res = resolution
        if res is None and sda_config is not None and getattr(sda_config, "model", None) is not None:
            res = getattr(sda_config.model, "resolution", None)
        self.resolution = res or "2.8deg"
        self.batch = batch

    def _policies(self):
        from tornado_gcm_b200.precision.policy import PrecisionPolicy

        base = self.sda_config.policy if self.sda_config is not None else PrecisionPolicy.pzha_b200()
        return [("fp64-transforms", PrecisionPolicy.pzha_b200(), "highest"),
                ("configured", base, None),
                ("pzha-b200", PrecisionPolicy.pzha_b200(), None)]

    def run(self) -> PrecisionBenchmarkResult:
        from tornado_gcm_b200.models.builders import build_hybrid_gcm

        rows, ref = [], None
        for name, policy, sht in self._policies():
            gcm, data = build_hybrid_gcm(self.resolution, self.device, policy=policy, sht_precision=sht)
            enc = gcm.encoder
            x0 = {k: ((v.to(self.device) - getattr(enc, f"mean_{k}")) / getattr(enc, f"std_{k}"))
                  for k, v in data.sample(self.batch, 0).items()}
            f = gcm.normalize_forcings({k: v.to(self.device) for k, v in data.forcings(self.batch).items()})
            with torch.no_grad():
                s0 = gcm.encoder(x0, f)

                def run():
                    s = s0
                    for _ in range(self.n_steps * gcm.physics_steps_per_output):
                        s = gcm.model.step(s, f)
                    return s

                tb = TimingBenchmark(warmup=1, iterations=2)
                r = tb.time_fn(name, run)
                out = run()
            vec = torch.cat([t.reshape(-1).double().cpu() for t in out.tensors()])
            drift = None
            if ref is None:
                ref = vec
            else:
                drift = float((vec - ref).norm() / ref.norm())
            rows.append({"policy": name, "ms": r.mean_ms / self.n_steps, "drift": drift})
        return PrecisionBenchmarkResult(rows)


# ── kernel micro-benchmarks ─────────────────────────────────────────────────
def _mlp_case(args):
    from tornado_gcm_b200.ops import linear as lops

    dev = torch.device("cuda")
    torch.manual_seed(0)
    dims = [args.width_in] + [args.width] * args.layers + [args.width_out]
    layers = [torch.nn.Linear(a, b).to(dev) for a, b in zip(dims[:-1], dims[1:])]
    acts = ["gelu_tanh"] * (len(layers) - 1) + ["none"]
    x = torch.randn(args.tokens, args.width_in, device=dev, requires_grad=True)

    def step():
        y = lops.mlp_forward(x, layers, acts)
        torch.autograd.grad(y.sum(), [x] + [p for lyr in layers for p in lyr.parameters()])

    flops = 6.0 * args.tokens * sum(a * b for a, b in zip(dims[:-1], dims[1:]))
    return step, flops


def _sht_case(args):
    from tornado_gcm_b200.core import spherical_harmonic as sh
    from tornado_gcm_b200.ops import sht as sht_ops

    g = getattr(sh.Grid, args.grid)(precision="tf32")
    x = torch.randn(args.slices, *g.modal_shape, device="cuda")
    b = sht_ops.bases(g.spherical_harmonics, x.device)

    nod = sht_ops.to_nodal_lat_major(x, g.spherical_harmonics)

    def step():
        if args.mode in ("fwd", "both"):
            n = sht_ops.to_nodal_lat_major(x, g.spherical_harmonics)
        if args.mode in ("dgrad", "both", "wgrad"):
            sht_ops.to_modal_lat_major(nod, g.spherical_harmonics)

    M2, L = g.modal_shape
    I, J = g.nodal_shape
    leg = sum(2 * J * (L - m) for m in range((M2 + 1) // 2)) * 2
    flops = 2.0 * args.slices * (leg + 2 * I * M2 * J)
    del b
    return step, flops


def _stage_case(args):
    import numpy as np

    from tornado_gcm_b200.core import coordinate_systems as cs, primitive_equations as pe
    from tornado_gcm_b200.core import sigma_coordinates as sc, spherical_harmonic as sh
    from tornado_gcm_b200.ops import dycore as dyops, spectral
    from tornado_gcm_b200.utils.units import SimUnits

    g = getattr(sh.Grid, args.grid)(precision="tf32")
    n = 32
    coords = cs.CoordinateSystem(g, sc.SigmaCoordinates.equidistant(n))
    keys = ("specific_cloud_ice_water_content", "specific_cloud_liquid_water_content", "specific_humidity")
    eq = pe.PrimitiveEquationsSigma(np.linspace(210, 290, n), torch.zeros(g.modal_shape), coords,
                                    SimUnits.from_si(), humidity_key="specific_humidity", cloud_keys=keys[:2])
    st = dyops.PackedSIL3(eq, 0.1, np.ones(g.modal_shape[-1]), keys)
    C = spectral.packed_channels(n, keys)["C"]
    y = 1e-3 * torch.randn(args.batch, C, *g.modal_shape, device="cuda", requires_grad=True)
    P = torch.zeros_like(y)

    def step():
        out = st.step_packed(y, P)
        torch.autograd.grad(out.sum(), [y])

    return step, 0.0


def _recipe_case(args):
    import numpy as np

    from tornado_gcm_b200.core import coordinate_systems as cs, primitive_equations as pe
    from tornado_gcm_b200.core import sigma_coordinates as sc, spherical_harmonic as sh
    from tornado_gcm_b200.ops import spectral
    from tornado_gcm_b200.utils.units import SimUnits

    g = getattr(sh.Grid, args.grid)(precision="tf32")
    n = 32
    coords = cs.CoordinateSystem(g, sc.SigmaCoordinates.equidistant(n))
    keys = ("specific_cloud_ice_water_content", "specific_cloud_liquid_water_content", "specific_humidity")
    eq = pe.PrimitiveEquationsSigma(np.linspace(210, 290, n), torch.zeros(g.modal_shape), coords,
                                    SimUnits.from_si(), humidity_key="specific_humidity", cloud_keys=keys[:2])
    rec = {"pre": spectral.explicit_pre_recipe(eq, keys), "post": spectral.explicit_post_recipe(eq, keys)}[args.recipe]
    if args.transpose:
        rec = rec.transpose()
    L = g.modal_shape[-1]
    x = torch.randn(args.batch, rec.c_in, *g.modal_shape, device="cuda")
    lp = (L + 3) // 4 * 4
    return (lambda: rec.apply(x, lp)), 0.0


def _linear_case(args):
    from tornado_gcm_b200.ops import _ext

    ops = _ext.require("linear micro-benchmark")
    dev = torch.device("cuda")
    T, K, O = args.tokens, args.width, args.width
    X = torch.randn(T, K, device=dev).bfloat16()
    W = torch.randn(O, K, device=dev).bfloat16() * 0.05
    bias = torch.zeros(O, device=dev)
    out = torch.empty(T, O, device=dev, dtype=torch.bfloat16)
    aux = torch.empty(T, O, device=dev, dtype=torch.bfloat16)
    dY = torch.randn(T, O, device=dev).bfloat16()
    dX = torch.empty(T, K, device=dev, dtype=torch.bfloat16)
    dW = torch.zeros(O, K, device=dev)
    err = _ext.error_flag(dev)
    if args.mode == "fwd":
        fn = lambda: ops.linear_fwd(X, W, bias, 3, out, aux, err)
    elif args.mode == "dgrad":
        fn = lambda: ops.linear_dgrad(dY, W, dX, X, 3, err)
    else:
        fn = lambda: ops.linear_wgrad(dY, X, dW, 0, err)
    return fn, 2.0 * T * K * O


def _bgemm_case(args):
    from tornado_gcm_b200.ops import _ext

    ops = _ext.require("batched GEMM micro-benchmark")
    dev = torch.device("cuda")
    A = torch.randn(args.groups, args.m, args.k, device=dev)
    B = torch.randn(args.groups, args.n, args.k, device=dev)
    C = torch.empty(args.groups, args.m, args.n, device=dev)
    err = _ext.error_flag(dev)
    return (lambda: ops.bgemm_tf32(A, B, C, 1.0, err)), 2.0 * args.groups * args.m * args.n * args.k


def _single_rank_group() -> None:
    """A one-rank NCCL group so the peer-memory paths run on one GPU (kernel captures)."""
    import datetime
    import os

    import torch.distributed as dist

    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", torch.cuda.current_device()))


def _fused_sht_case(args):
    """Latitude-sharded analysis with the cross-GPU sum in the Legendre GEMM epilogue (one rank:
    the same kernels, the peer list holds this GPU's own buffer)."""
    from tornado_gcm_b200.core import spherical_harmonic as sh
    from tornado_gcm_b200.parallel.sharded_sht import LatitudeShardedSHT

    _single_rank_group()
    g = getattr(sh.Grid, args.grid)(precision="tf32")
    M2, L = g.modal_shape
    I, J = g.nodal_shape
    sht = LatitudeShardedSHT(g, scheme="mirrored")
    sht.enable_fused(args.slices, torch.device("cuda"))
    nodal = torch.randn(args.slices, I, J, device="cuda")

    def step():
        with torch.no_grad():
            sht.to_modal_fused(nodal)

    return step, 2.0 * args.slices * (M2 * I * J + M2 * J * L)


def _gathered_linear_case(args):
    """Linear layer whose weight is read from the ranks' shards by the GEMM producer (one rank)."""
    from tornado_gcm_b200.parallel.fsdp_gather import GatheredLinear

    _single_rank_group()
    w = torch.randn(args.width, args.width, device="cuda") / args.width ** 0.5
    lin = GatheredLinear(w, torch.zeros(args.width, device="cuda"), "gelu_tanh")
    x = torch.randn(args.tokens, args.width, device="cuda").to(torch.bfloat16)

    def step():
        lin(x)

    return step, 2.0 * args.tokens * args.width * args.width


def gemm_cycle_breakdown(fn, launch_index: int = -1) -> list:
    """Run ``fn`` once per GEMM launch recorded and return per-CTA-averaged cycle counters.

    Counters (cycles, averaged over the CTAs of the last GEMM launch in ``fn``):
    producer waiting for a free ring stage, MMA waiting for a free accumulator,
    MMA waiting for operands, epilogue waiting for an accumulator, epilogue work.
    """
    from tornado_gcm_b200.ops import _ext

    ops = _ext.require("GEMM profile")
    buf = torch.zeros(1024, 8, dtype=torch.int64, device="cuda")
    ops.gemm_profile_buffer(buf, launch_index)
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        ops.gemm_profile_buffer(None)
    b = buf[buf[:, 7] > 0].double()
    if b.numel() == 0:
        return []
    m = b.mean(0).tolist()
    return [{"producer_wait": m[0], "mma_wait_acc": m[2], "mma_wait_full": m[3], "epi_wait": m[5],
             "epi_work": m[6], "tiles_per_cta": m[7], "ctas": int(b.shape[0])}]


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="kernel micro-benchmarks (CUDA events)")
    ap.add_argument("case", choices=["mlp", "sht", "stage", "linear", "bgemm", "recipe", "fused_sht",
                                     "gathered_linear"])
    ap.add_argument("--recipe", default="pre", choices=["pre", "post"])
    ap.add_argument("--transpose", action="store_true")
    ap.add_argument("--mode", default="fwd", choices=["fwd", "dgrad", "wgrad", "both"],
                    help="linear: which GEMM; sht: fwd = synthesis, dgrad = analysis, both")
    ap.add_argument("--groups", type=int, default=1292)
    ap.add_argument("--m", type=int, default=128)
    ap.add_argument("--n", type=int, default=64)
    ap.add_argument("--k", type=int, default=128)
    ap.add_argument("--tokens", type=int, default=32768)
    ap.add_argument("--width", type=int, default=384)
    ap.add_argument("--width-in", type=int, default=197)
    ap.add_argument("--width-out", type=int, default=193)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--grid", default="TL63")
    ap.add_argument("--slices", type=int, default=1292)
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--cycles", action="store_true", help="print the GEMM cycle breakdown of one call")
    ap.add_argument("--launch", type=int, default=-1, help="which GEMM launch of the call to break down (-1: last)")
    args = ap.parse_args(argv)
    fn, flops = {"mlp": _mlp_case, "sht": _sht_case, "stage": _stage_case, "linear": _linear_case,
                 "bgemm": _bgemm_case, "recipe": _recipe_case, "fused_sht": _fused_sht_case,
                 "gathered_linear": _gathered_linear_case}[args.case](args)
    tb = TimingBenchmark(warmup=args.warmup, iterations=args.iters)
    r = tb.time_fn(args.case, fn)
    out = {"case": args.case, "mean_ms": r.mean_ms, "min_ms": r.min_ms}
    if flops:
        out["tflops"] = round(flops / (r.min_ms * 1e-3) / 1e12, 2)
    if args.cycles:
        out["gemm_cycles"] = gemm_cycle_breakdown(fn, args.launch)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
