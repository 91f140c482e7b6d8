#!/usr/bin/env python
"""Training-throughput benchmark of the hybrid GCM (6-h model steps per second).

Workload (per GPU): 2.8° model (TL63, 128×64 Gaussian grid, 32 σ levels),
batch 4, backpropagation through a 4 × 6-h rollout (72 physics steps of
20 min, neural tendency every physics step), column encoder 3×256 from 7
fields × 37 pressure levels, column tower 5×384, column decoder 3×256, Z2
fixer every step, MSE loss on the decoded fields, AdamW (lr 1e-4), grad
clipping and EMA.  Synthetic reanalysis-shaped data, random-init weights.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

For N > 1 launch one process per GPU with torch.distributed.run; data
parallel over ranks (weak scaling, batch 4 per GPU).  Device time of the K
timed steps is taken with CUDA events between barrier + synchronize and
reduced as the max over ranks.  Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

PUBLISHED = {"2.8deg": 4.1, "1.4deg": 1.3, "0.7deg": 0.35}  # reference README, steps/s on 1× A100
METRIC = "model steps/s (train & 6h-forecast) at 2.8°/1.4°/0.7°, 1/2/4/8 B200, vs ref NCCL"
DTYPE_ZONES = "bf16 (Z3 towers) + tf32 (Z1 transforms/dycore) + fp64-accumulated (Z2 fixer)"
E2E_UNIT = "6h model-steps/s (samples x 6-h steps, all GPUs), end to end"
# What still differs between the reference arm and this framework's arm of the training benchmark.
REFERENCE_DIFFERENCES = [
    "tower: the reference's ModalNeuralDivCurlParameterization feeds 3n+1 modal-derived nodal features "
    "(+4 forcings) and returns 3n+1 tendencies (no tracers); this framework's column tower maps 6n+1+4 -> 6n+1 "
    "(tracers included), i.e. more tower work per column",
    "transforms: FP64 einsum (the reference selects FP64 above total wavenumber 42) vs TF32 tcgen05 GEMMs (Z1)",
    "towers: BF16 autocast over eager nn.Linear (the reference trainer's Z3 path) vs BF16 tcgen05 GEMMs (Z3)",
    "fixer: F64ConservationFixer (full FP64 upcast) vs FP64-accumulated packed fixer kernel",
    "batching: the reference modules take one sample at a time, so the arm loops over the 4 samples "
    "(one backward each); this framework runs the batch as one tensor",
    "step capture: eager PyTorch vs one CUDA graph for the whole training step",
]
# this framework's kernels live in the tgcm namespace (device-side names "tgcm::…")
MY_KERNELS = ("tgcm::",)


# ── helpers ─────────────────────────────────────────────────────────────────
def measured_peaks() -> dict:
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            d = json.load(fh)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def step_roofline(acc: dict, ms_per_step: float) -> dict:
    """Roofline of one training step from the op accounting of an eager step: the
    algorithmic bytes of every native op at the measured HBM bandwidth against its
    FLOPs at the measured BF16 rate (TF32 at half of it), and the timed step."""
    from tornado_gcm_b200.ops import accounting

    pk = measured_peaks()
    sm = accounting.summary(acc, pk["hbm_gbs"], pk["bf16_tflops"])
    sm = {k: (round(v, 4) if isinstance(v, float) else v) for k, v in sm.items()}
    sm["tflop"] = {k: round(v, 4) for k, v in sm["tflop"].items()}
    sm["peaks"] = pk["source"]
    sm["frac_of_roofline"] = round(sm["roofline_ms"] / ms_per_step, 4) if ms_per_step > 0 else None
    return sm


def write_kernel_table(prof, path: str, acc: dict | None = None) -> None:
    """Per-kernel count and summed device time of one profiled step, largest first;
    with ``acc`` (op accounting of the same step) the per-op traffic table follows."""
    agg: dict = {}
    for ev in prof.events():
        if ev.device_type != torch.autograd.DeviceType.CUDA:
            continue
        name = ev.name if len(ev.name) < 110 else ev.name[:107] + "..."
        c, t = agg.get(name, (0, 0.0))
        agg[name] = (c + 1, t + ev.device_time_total)
    total = sum(t for _, t in agg.values()) or 1.0
    rows = sorted(agg.items(), key=lambda kv: -kv[1][1])
    with open(path, "w") as fh:
        fh.write(f"# one eager training step; total device time {total / 1000.0:.2f} ms\n")
        fh.write("share%  time_ms  count  kernel\n")
        for name, (c, t) in rows:
            fh.write(f"{100.0 * t / total:6.2f} {t / 1000.0:8.3f} {c:6d}  {name}\n")
        if acc:
            from tornado_gcm_b200.ops import accounting

            pk = measured_peaks()
            sm = accounting.summary(acc, pk["hbm_gbs"], pk["bf16_tflops"])
            fh.write(f"\n# native-op accounting of the same step ({pk['source']} peaks: "
                     f"{pk['hbm_gbs']} GB/s, {pk['bf16_tflops']} TFLOP/s BF16)\n")
            fh.write(f"# total {sm['alg_bytes_gb']:.2f} GB -> {sm['t_hbm_ms']:.1f} ms at HBM; "
                     f"TFLOP {sm['tflop']} -> {sm['t_flop_ms']:.1f} ms\n")
            for line in accounting.table_lines(acc, pk["hbm_gbs"]):
                fh.write(line + "\n")


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--resolution", default="2.8deg")
    p.add_argument("--mode", choices=["train", "forecast"], default="train",
                   help="train: backprop through the rollout (default); forecast: ensemble 6-h forecast")
    p.add_argument("--members", type=int, default=16, help="forecast: ensemble members per GPU")
    p.add_argument("--fsdp", action="store_true",
                   help="forecast: shard the column tower's weights over the GPUs; every GEMM reads the other "
                        "ranks' rows from their memory as it runs (all-gather fused into the GEMM)")
    p.add_argument("--save-forecast", default=None,
                   help="forecast: write the last 6-h output of rank 0 to this .pt file (for comparisons)")
    p.add_argument("--checkpoint", choices=["auto", "on", "off"], default="auto",
                   help="train: recompute each 6-h block in backward (auto: on above 2.8 degrees)")
    p.add_argument("--checkpoint-segment", type=int, default=-1,
                   help="physics steps per recomputed segment (0: whole 6-h block; default 8 at 0.7 degrees)")
    p.add_argument("--batch", type=int, default=4, help="per-GPU batch")
    p.add_argument("--parallel", choices=["dp", "lat", "sharded"], default="dp",
                   help="train: dp = data parallel (replicated model, batch per GPU); lat = the model sharded "
                        "over the GPUs (modal rows by zonal wavenumber, nodal columns by latitude block), all "
                        "GPUs on one global batch of batch x GPUs samples; sharded = data parallel with the "
                        "gradients and AdamW state split over the GPUs (reduce-scatter, sharded AdamW, "
                        "all-gather of the weights)")
    p.add_argument("--rollout", type=int, default=4, help="6-h steps per training example")
    p.add_argument("--no-graph", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--reference-e2e-steps", type=int, default=3,
                   help="reference arm: steps of its end-to-end timed region (each takes tens of seconds)")
    p.add_argument("--kernel-table", default=None,
                   help="write a per-kernel device-time table of one eager step (torch profiler, "
                        "outside the timed region) to this path")
    return p.parse_args()


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.lines: list[str] = []
        self._thr = None

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if self.uuid:
            cmd += ["-i", self.uuid]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self._thr = threading.Thread(target=self._read, daemon=True)
        self._thr.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self._thr is not None:
            self._thr.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 10:
                continue
            try:
                sm.append(float(parts[2]))
                smax.append(float(parts[3]))
            except ValueError:
                continue
            for nm, flag in zip(names, parts[6:10]):
                if flag.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(gpus: int, need_group: bool = False):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 or need_group:
        os.environ.setdefault("MASTER_PORT", "29533")
        os.environ.setdefault("WORLD_SIZE", str(world))
        os.environ.setdefault("RANK", str(rank))
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world <= 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def device_uuid() -> str | None:
    try:
        u = torch.cuda.get_device_properties(torch.cuda.current_device()).uuid
        s = str(u)
        return s if s.startswith("GPU-") else "GPU-" + s
    except Exception:
        return None


def timed_region(step_fn, steps: int, world: int, sampler: ClockSampler | None):
    barrier(world)
    torch.cuda.synchronize()
    if sampler is not None:
        sampler.start()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        step_fn(i)
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop() if sampler is not None else None
    ms = start.elapsed_time(end)
    return max_over_ranks(ms, world), clocks


# ── this framework ──────────────────────────────────────────────────────────
def run_b200(args, rank, world):
    if args.mode == "forecast":
        return run_b200_forecast(args, rank, world)
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from tornado_gcm_b200.models.builders import RESOLUTIONS, build_hybrid_gcm
    from tornado_gcm_b200.ops import _ext
    from tornado_gcm_b200.training.trainer import GCMTrainer

    _ext.require("benchmark")
    dev = torch.device("cuda", torch.cuda.current_device())
    gcm, data = build_hybrid_gcm(args.resolution, dev, seed=0)
    spec = RESOLUTIONS[args.resolution]
    gcm.checkpoint_outer_steps = (args.checkpoint == "on" or
                                  (args.checkpoint == "auto" and args.resolution not in ("2.8deg", "5.6deg")))
    gcm.checkpoint_segment = args.checkpoint_segment if args.checkpoint_segment >= 0 else (
        8 if args.resolution == "0.7deg" else 0)
    lat = args.parallel == "lat"
    shard = None
    if lat:
        from tornado_gcm_b200.parallel import spectral_shard as ss

        ss.shard_hybrid_gcm(gcm, None, "fused")
        shard = gcm.shard
    dp_mode = "sharded" if (args.parallel == "sharded" and world > 1) else world > 1
    trainer = GCMTrainer(gcm, lr=1e-4, graph=not args.no_graph, data_parallel=dp_mode, grad_average=not lat)
    # lat: every rank holds 1/W of each of the batch x W samples (same per-GPU work as dp)
    B, K = (args.batch * world if lat else args.batch), args.rollout
    enc = gcm.encoder
    local = (lambda d: ss.scatter_fields(d, shard)) if lat else (lambda d: d)

    def norm(d):
        return local({k: ((v.to(dev) - getattr(enc, f"mean_{k}")) / getattr(enc, f"std_{k}")).cpu()
                      for k, v in d.items()})

    # pinned host pool of a few batches (cycled); distinct per rank (dp) or shared (lat)
    pool = []
    for j in range(2):
        s = (0 if lat else 100 * rank) + 10 * j
        x0 = norm(data.sample(B, s))
        tg = [norm(data.sample(B, s + i + 1)) for i in range(K)]
        pool.append(({k: v.pin_memory() for k, v in x0.items()},
                     [{k: v.pin_memory() for k, v in t.items()} for t in tg]))
    forc_host = {k: v.contiguous().pin_memory() for k, v in local(data.forcings(B)).items()}
    to_dev = lambda d: {k: v.to(dev, non_blocking=True) for k, v in d.items()}
    dev_pool = [(to_dev(a), [to_dev(t) for t in b]) for a, b in pool]
    forc_dev = to_dev(forc_host)
    h2d_bytes = sum(v.numel() * v.element_size() for v in pool[0][0].values())
    h2d_bytes += sum(v.numel() * v.element_size() for t in pool[0][1] for v in t.values())
    h2d_bytes += sum(v.numel() * v.element_size() for v in forc_host.values())

    losses = []

    def step_dev(i):
        x0, tg = dev_pool[i % len(dev_pool)]
        losses.append(trainer.train_step(x0, tg, forc_dev))

    for i in range(args.warmup):
        step_dev(i)
    torch.cuda.synchronize()
    _ext.check_error_flag(dev)
    sampler = ClockSampler(device_uuid()) if rank == 0 else None
    ms, clocks = timed_region(step_dev, args.steps, world, sampler)
    _ext.check_error_flag(dev)
    ms_per_step = ms / args.steps
    loss_last = float(losses[-1].item()) if losses else float("nan")
    if lat and world > 1:  # each rank's loss is its share of the global loss
        import torch.distributed as dist

        t = torch.tensor([loss_last], dtype=torch.float64, device=dev)
        dist.all_reduce(t)
        loss_last = float(t.item())

    samples_per_step = B if lat else world * B
    e2e = None
    if not args.no_e2e:
        host_loss = []

        def step_e2e(i):
            x0h, tgh = pool[i % len(pool)]
            x0 = to_dev(x0h)
            tg = [to_dev(t) for t in tgh]
            f = to_dev(forc_host)
            loss = trainer.train_step(x0, tg, f)
            host_loss.append(float(loss.item()))  # D2H read of the step's result

        ms_e2e, _ = timed_region(step_e2e, args.steps, world, None)
        e2e = {"value": samples_per_step * K / (ms_e2e / args.steps / 1000.0), "unit": E2E_UNIT,
               "h2d_bytes_per_step": int(h2d_bytes), "d2h_bytes_per_step": 4,
               "ms_per_step": ms_e2e / args.steps}

    # count this framework's kernels in one (eager) step, outside the timed region
    launches = None
    roofline = None
    try:
        from torch.profiler import ProfilerActivity, profile

        x0, tg = dev_pool[0]
        use_graph = trainer.use_graph
        trainer.use_graph = False
        try:
            from tornado_gcm_b200.ops import accounting

            with accounting.counting() as acc, profile(activities=[ProfilerActivity.CUDA]) as prof:
                trainer._zero()
                trainer._step_body(x0, tg, forc_dev)
                torch.cuda.synchronize()
        finally:
            trainer.use_graph = use_graph
        n_mine = 0
        n_all = 0
        for ev in prof.events():
            if ev.device_type == torch.autograd.DeviceType.CUDA:
                n_all += 1
                if any(k in ev.name for k in MY_KERNELS):
                    n_mine += 1
        launches = {"per_step_mine": n_mine, "per_step_all": n_all}
        roofline = step_roofline(acc, ms_per_step)
        if args.kernel_table and rank == 0:
            write_kernel_table(prof, args.kernel_table, acc)
    except Exception as exc:  # pragma: no cover
        launches = {"error": str(exc)}

    value = samples_per_step * K / (ms_per_step / 1000.0)
    if rank == 0:
        out = {
            "metric": METRIC,
            "value": value,
            "unit": "6h model-steps/s (samples x 6-h steps, all GPUs)",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": value / PUBLISHED.get(args.resolution, float("nan")),
            "dtype": DTYPE_ZONES,
            "data": "synthetic reanalysis-shaped fields, random-init weights",
            "config": {
                "model": f"{args.resolution} {spec.grid} L{spec.layers} hybrid GCM (encoder 3x256, tower 5x"
                         f"{spec.tower_width}, decoder 3x256, IMEX-SIL3 dt={spec.dt_minutes:g} min, "
                         f"{spec.physics_steps_per_output} physics steps per 6 h)",
                "global_batch": samples_per_step,
                "seq_len": K,
                "seq_len_meaning": "6-h rollout steps per example (backprop through the whole rollout)",
                "parallelism": (f"lat{world} (modal rows by zonal wavenumber, nodal columns by latitude block; "
                                f"transposes fused into the Legendre GEMMs)") if lat else (
                    f"dp{world} (gradients and AdamW state sharded)" if dp_mode == "sharded" else f"dp{world}"),
                "zones": "Z1 TF32 tcgen05 transforms, Z3 BF16 tcgen05 towers, Z2 FP64-accumulated fixer",
                "grad_reducer": trainer.grad_reducer,
                "cuda_graph": trainer.use_graph,
                "activation_checkpointing": ("none" if not gcm.checkpoint_outer_steps else
                                             f"segments of {gcm.checkpoint_segment} physics steps"
                                             if gcm.checkpoint_segment else "per 6-h block"),
                "l2": f"working set per step (activations of {K * spec.physics_steps_per_output} physics steps) "
                      "far exceeds the 126 MB L2",
                "loss": loss_last,
                "peak_mem_gb": torch.cuda.max_memory_allocated() / 1e9,
                "roofline": roofline,
            },
            "clocks": clocks,
            "e2e": e2e,
            "gpu_launches": (launches or {}).get("per_step_mine", 0) * args.steps,
            "launch_detail": launches,
            "impl": "b200",
        }
        print(json.dumps(out), flush=True)
    trainer.release_graph()


def run_b200_forecast(args, rank, world):
    """Ensemble forecast through the public inference API (``MPInference.rollout``).

    Members (``--members`` per GPU) share one analysis; each adds a Gaussian
    random field (σ = 1 in normalised data units, correlation length 1000 km)
    to every input field and level, and all members advance as ONE batch.  A
    timed "step" is one 6-h forecast step of the whole ensemble (physics steps
    replayed from a CUDA graph, outputs decoded every 6 h).
    """
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from tornado_gcm_b200.inference.runner import MPInference
    from tornado_gcm_b200.models.builders import RESOLUTIONS, build_hybrid_gcm
    from tornado_gcm_b200.neural.stochastic import GaussianRandomField
    from tornado_gcm_b200.ops import _ext

    _ext.require("benchmark")
    dev = torch.device("cuda", torch.cuda.current_device())
    gcm, data = build_hybrid_gcm(args.resolution, dev, seed=0)
    spec = RESOLUTIONS[args.resolution]
    lat = args.parallel == "lat"
    M, K = (args.members * world if lat else args.members), args.steps
    enc = gcm.encoder
    grid = gcm.model.config.coords.horizontal
    grf = GaussianRandomField(grid, correlation_length_km=1000.0, variance=1.0).to(dev)
    # lat: one ensemble of members x GPUs shared by all ranks (each holds its latitude block)
    gen = torch.Generator(device=dev).manual_seed(1234 + (0 if lat else rank))
    with torch.no_grad():
        ens = {}
        for k, v in data.sample(1, 0 if lat else 100 * rank).items():
            x = (v.to(dev) - getattr(enc, f"mean_{k}")) / getattr(enc, f"std_{k}")
            noise = grid.to_nodal(grf.sample_modal((M,) + tuple(x.shape[1:-2]), generator=gen, device=dev))
            ens[k] = (x + noise).contiguous()
    forc_full = data.forcings(M)
    if lat:
        from tornado_gcm_b200.parallel import spectral_shard as ss

        ss.shard_hybrid_gcm(gcm, None, "fused")
        ens = ss.scatter_fields(ens, gcm.shard)
        forc_full = ss.scatter_fields(forc_full, gcm.shard)
    if args.fsdp:
        gcm.model.parameterization.shard_tower_weights()
    engine = MPInference(gcm)
    ens_host = {k: v.cpu().pin_memory() for k, v in ens.items()}
    forc_host = {k: v.contiguous().pin_memory() for k, v in forc_full.items()}
    forc_dev = {k: v.to(dev) for k, v in forc_host.items()}

    members_total = M if lat else world * M
    warm = engine.rollout(ens, max(1, args.warmup), forcings=forc_dev)  # graph capture + warm-up
    finite = all(bool(torch.isfinite(v).all()) for v in warm[-1].values())
    if args.save_forecast and rank == 0:
        torch.save({k: v.detach().cpu() for k, v in warm[-1].items()}, args.save_forecast)
    torch.cuda.synchronize()
    _ext.check_error_flag(dev)
    sampler = ClockSampler(device_uuid()) if rank == 0 else None
    ms, clocks = timed_region(lambda i: engine.rollout(ens, K, forcings=forc_dev), 1, world, sampler)
    _ext.check_error_flag(dev)

    e2e = None
    d2h = 0
    if not args.no_e2e:
        def e2e_run(i):
            nonlocal d2h
            x = {k: v.to(dev, non_blocking=True) for k, v in ens_host.items()}
            f = {k: v.to(dev, non_blocking=True) for k, v in forc_host.items()}
            traj = engine.rollout(x, K, forcings=f, offload=True)  # every 6-h output copied to the host
            d2h = sum(t.numel() * t.element_size() for t in traj[0].values())

        ms_e2e, _ = timed_region(e2e_run, 1, world, None)
        h2d = sum(v.numel() * v.element_size() for v in ens_host.values())
        h2d += sum(v.numel() * v.element_size() for v in forc_host.values())
        e2e = {"value": members_total * K / (ms_e2e / 1000.0),
               "unit": "6h model-steps/s (ensemble members x 6-h steps, all GPUs), end to end",
               "h2d_bytes_per_step": int(h2d / K), "d2h_bytes_per_step": int(d2h),
               "h2d_note": "initial ensemble + forcings copied once per forecast, amortised over its steps",
               "ms_per_step": ms_e2e / K}

    # this framework's kernels per 6-h step: one eager physics step and one decode, profiled
    launches = None
    try:
        from torch.profiler import ProfilerActivity, profile

        def count(fn):
            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                fn()
                torch.cuda.synchronize()
            return sum(1 for ev in prof.events() if ev.device_type == torch.autograd.DeviceType.CUDA
                       and any(k in ev.name for k in MY_KERNELS))

        with torch.no_grad():
            f_n = gcm.normalize_forcings(forc_dev)
            s0 = gcm.encoder(ens, f_n)
            n_phys = count(lambda: gcm.model.step(s0, f_n))
            n_dec = count(lambda: gcm.decoder(s0, f_n))
        launches = {"per_physics_step": n_phys, "per_decode": n_dec,
                    "per_6h_step": n_phys * spec.physics_steps_per_output + n_dec}
    except Exception as exc:  # pragma: no cover
        launches = {"error": str(exc)}

    value = members_total * K / (ms / 1000.0)
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "mode": "forecast", "value": value,
            "unit": "6h model-steps/s (ensemble members x 6-h forecast steps, all GPUs)",
            "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": ms / K,
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": value / PUBLISHED.get(args.resolution, float("nan")),
            "dtype": DTYPE_ZONES, "data": "synthetic reanalysis-shaped analysis + GRF member perturbations, random-init weights",
            "config": {
                "model": f"{args.resolution} {spec.grid} L{spec.layers} hybrid GCM (tower 5x{spec.tower_width}, "
                         f"IMEX-SIL3 dt={spec.dt_minutes:g} min, {spec.physics_steps_per_output} physics steps per 6 h)",
                "global_batch": members_total, "seq_len": K,
                "seq_len_meaning": "6-h forecast steps (one timed rollout)",
                "parallelism": ((f"lat{world} (model sharded over GPUs: modal rows by wavenumber, nodal columns "
                                 f"by latitude block)" if lat else f"dp{world} (ensemble members over GPUs)")
                                + (", tower weights FSDP-sharded (all-gather fused into the GEMM)"
                                   if args.fsdp else "")),
                "members_per_gpu": args.members, "perturbation": "GRF sigma=1 (normalised units), 1000 km",
                "outputs_finite_after_warmup": finite,
                "zones": "Z1 TF32 tcgen05 transforms, Z3 BF16 tcgen05 towers, Z2 FP64-accumulated fixer",
                "cuda_graph": True,
                "l2": "ensemble state and decoded outputs exceed the 126 MB L2",
                "peak_mem_gb": torch.cuda.max_memory_allocated() / 1e9,
            },
            "clocks": clocks, "e2e": e2e,
            "gpu_launches": (launches or {}).get("per_6h_step", 0) * K, "launch_detail": launches,
            "impl": "b200",
        }), flush=True)


# ── reference arm (unmodified reference from baseline/_ref) ─────────────────
def _reference_setup(args, rank):
    """The 2.8° hybrid model assembled from the reference's own modules (or None if not installed)."""
    here = os.path.dirname(os.path.abspath(__file__))
    ref_root = os.path.join(here, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "tornado_gcm")):
        return None
    sys.path.insert(0, ref_root)
    from types import SimpleNamespace

    import numpy as np
    import torch.nn.functional as F

    from tornado_gcm.core import coordinate_systems, sigma_coordinates, spherical_harmonic
    from tornado_gcm.model.api import ModelConfig, NeuralGCMModel
    from tornado_gcm.neural.fixers import F64ConservationFixer
    from tornado_gcm.neural.parameterizations import ModalNeuralDivCurlParameterization
    from tornado_gcm.neural.standard_layers import Mlp
    from tornado_gcm.neural.towers import ForwardTower
    from tornado_gcm.precision.policy import PrecisionPolicy

    if args.resolution != "2.8deg":
        raise SystemExit("reference arm implemented for the 2.8deg configuration")
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(0)
    # physical constants in the reference's non-dimensional units (pint is not installed)
    L0, T0 = 6.37122e6, 1.0 / (2 * 7.292e-5)
    nd = lambda si, e_len, e_time: si * (T0 ** (-e_time)) / (L0 ** e_len)
    R = nd(1004.0 * 2 / 7, 2, -2)
    specs = SimpleNamespace(R=R, R_vapor=nd(461.0, 2, -2), g=nd(9.80616, 1, -2), Cp=R / (2 / 7),
                            Cp_vapor=nd(1859.0, 2, -2), kappa=2 / 7, angular_velocity=7.292e-5 * T0, radius=1.0)
    grid = spherical_harmonic.Grid.TL63()
    vertical = sigma_coordinates.SigmaCoordinates.equidistant(32)
    coords = coordinate_systems.CoordinateSystem(grid, vertical)
    n = 32
    t_ref = np.maximum(200.0, 288.0 * vertical.centers ** 0.19)
    dt = 20 * 60 / T0
    cfg = ModelConfig(coords=coords, dt=dt, inner_steps=18, dycore_substeps=1, physics_specs=specs,
                      reference_temperature=t_ref, orography=torch.zeros(grid.modal_shape),
                      precision_policy=PrecisionPolicy(), filter_attenuation=dt / (120 * 60 / T0), filter_order=3,
                      filter_cutoff=0.0, stability_filter_attenuation=dt / (4 * 60 / T0),
                      stability_filter_order=10, stability_filter_cutoff=0.4, humidity_key="specific_humidity",
                      cloud_keys=("specific_cloud_ice_water_content", "specific_cloud_liquid_water_content"))
    tower = ForwardTower(Mlp.uniform(3 * n + 1 + 4, 3 * n + 1, hidden_size=384, hidden_layers=5,
                                     activation=F.gelu))
    param = ModalNeuralDivCurlParameterization(grid, tower, n)
    # Z2 fixer in FP64, as the benchmark configuration asks for (the reference's full-upcast fixer)
    model = NeuralGCMModel(cfg, parameterization=param, conservation_fixer=F64ConservationFixer()).to(dev)
    encoder = ForwardTower(Mlp.uniform(7 * 37 + 4, 6 * n + 1, hidden_size=256, hidden_layers=3,
                                       activation=F.gelu)).to(dev)
    decoder = ForwardTower(Mlp.uniform(6 * n + 1, 7 * 37, hidden_size=256, hidden_layers=3,
                                       activation=F.gelu)).to(dev)
    params = list(model.parameters()) + list(encoder.parameters()) + list(decoder.parameters())
    with torch.no_grad():
        for m in (tower, encoder, decoder):
            m.neural_net.layers[-1].weight.mul_(0.01)
    I, J = grid.nodal_shape
    g = torch.Generator(device="cpu").manual_seed(rank)
    forc = torch.randn(4, I, J, generator=g).to(dev)
    t_ref_t = torch.tensor(t_ref, dtype=torch.float32, device=dev).reshape(-1, 1, 1)
    tr_keys = ("specific_humidity", "specific_cloud_liquid_water_content", "specific_cloud_ice_water_content")

    def encode(x):  # x: (7*37, I, J) → reference State
        h = encoder(torch.cat([x, forc], 0))
        u, v, T = h[:n] * 1e-3, h[n:2 * n] * 1e-3, h[2 * n:3 * n] + t_ref_t
        trs = [h[3 * n + i * n:3 * n + (i + 1) * n] * 1e-6 for i in range(3)]
        lnps = h[6 * n:] * 1e-3
        vort, div = spherical_harmonic.uv_nodal_to_vor_div_modal(grid, u, v)
        temp = grid.to_modal(T - t_ref_t)
        from tornado_gcm.core.primitive_equations import State

        return State(vort, div, temp, grid.to_modal(lnps),
                     {k: grid.to_modal(t) for k, t in zip(tr_keys, trs)}, sim_time=0.0)

    def decode(s):
        u, v = spherical_harmonic.vor_div_to_uv_nodal(grid, s.vorticity, s.divergence)
        parts = [u * 1e3, v * 1e3, grid.to_nodal(s.temperature_variation)]
        parts += [grid.to_nodal(s.tracers[k]) * 1e6 for k in tr_keys] + [grid.to_nodal(s.log_surface_pressure)]
        return decoder(torch.cat(parts, 0))

    return SimpleNamespace(model=model, params=params, cfg=cfg, grid=grid, forc=forc, encode=encode,
                           decode=decode, gen=g, dev=dev, I=I, J=J)


def _reference_unavailable(rank):
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref/tornado_gcm not installed"}))


def run_reference(args, rank, world):
    if args.mode == "forecast":
        return run_reference_forecast(args, rank, world)
    ref = _reference_setup(args, rank)
    if ref is None:
        return _reference_unavailable(rank)
    model, params, cfg, dev, forc = ref.model, ref.params, ref.cfg, ref.dev, ref.forc
    encode, decode = ref.encode, ref.decode
    opt = torch.optim.AdamW(params, lr=1e-4, betas=(0.9, 0.95), eps=1e-6)
    ema = [p.detach().clone() for p in params]
    B, K = args.batch, args.rollout
    I, J = ref.I, ref.J
    mk = lambda *s: torch.randn(*s, generator=ref.gen)
    pool = [(mk(B, 7 * 37, I, J).pin_memory(), mk(B, K, 7 * 37, I, J).pin_memory()) for _ in range(2)]

    # the reference trainer's own precision handling (training/trainer.py:219-309): the policy's
    # TF32 setting, and the forward under BF16 autocast when Z3 computes in BF16 (its default)
    cfg.precision_policy.apply_tf32_setting()
    autocast_bf16 = cfg.precision_policy.z3_compute_dtype == torch.bfloat16

    def step_fn(i, read_loss=False):
        xh, th = pool[i % 2]
        x = xh.to(dev, non_blocking=True)
        tgt = th.to(dev, non_blocking=True)
        opt.zero_grad(set_to_none=True)
        total = torch.zeros((), device=dev)
        for b in range(B):
            with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast_bf16):
                state = encode(x[b])
                loss = 0.0
                for k in range(K):
                    for _ in range(cfg.inner_steps):
                        state = model.step(state, forcings={"f": forc})
                    loss = loss + ((decode(state).float() - tgt[b, k]) ** 2).mean()
            (loss / (K * B)).backward()
            total = total + loss.detach() / (K * B)
        if world > 1:
            import torch.distributed as dist

            flat = torch.cat([p.grad.reshape(-1) for p in params if p.grad is not None])
            dist.all_reduce(flat)
            flat /= world
            off = 0
            for p in params:
                if p.grad is not None:
                    nn_ = p.grad.numel()
                    p.grad.copy_(flat[off:off + nn_].view_as(p.grad))
                    off += nn_
        torch.nn.utils.clip_grad_norm_(params, 1.0)
        opt.step()
        with torch.no_grad():
            for e, p in zip(ema, params):
                e.lerp_(p, 2.0 / 2000)
        if read_loss:
            host_loss.append(float(total.item()))  # D2H read of the step's loss

    host_loss = []
    for i in range(args.warmup):
        step_fn(i)
    sampler = ClockSampler(device_uuid()) if rank == 0 else None
    ms, clocks = timed_region(step_fn, args.steps, world, sampler)
    ms_per_step = ms / args.steps
    value = world * B * K / (ms_per_step / 1000.0)
    e2e = None
    if not args.no_e2e:
        # End to end as in this framework's arm: pinned-host inputs copied every step and the
        # step's loss read back to the host.  A few steps only: one step takes tens of seconds.
        n_e2e = max(1, min(args.steps, args.reference_e2e_steps))
        ms_e2e, _ = timed_region(lambda i: step_fn(i, read_loss=True), n_e2e, world, None)
        e2e = {"value": world * B * K / (ms_e2e / n_e2e / 1000.0), "unit": E2E_UNIT,
               "h2d_bytes_per_step": int(pool[0][0].numel() * 4 + pool[0][1].numel() * 4),
               "d2h_bytes_per_step": 4, "ms_per_step": ms_e2e / n_e2e, "steps": n_e2e}
    if rank == 0:
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": value,
            "unit": "6h model-steps/s (samples x 6-h steps, all GPUs)", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": value / PUBLISHED[args.resolution],
            "dtype": "bf16 autocast (Z3 towers) + tf32 matmul setting + FP64 transforms (the reference's stock "
                     "TL63 path) + FP64 fixer",
            "data": "synthetic, random-init weights",
            "config": {"model": "2.8deg TL63 L32 (reference NeuralGCMModel + ModalNeuralDivCurlParameterization "
                                "tower 5x384, encoder/decoder 3x256, F64ConservationFixer, built from reference "
                                "modules)",
                       "global_batch": world * B, "seq_len": K, "parallelism": f"dp{world}",
                       "batching": "per-sample loop (reference modules are single-sample)",
                       "config_differences": REFERENCE_DIFFERENCES,
                       "l2": "working set far exceeds L2"},
            "clocks": clocks, "e2e": e2e,
            "gpu_launches": 0,
        }), flush=True)


def run_reference_forecast(args, rank, world):
    """Ensemble forecast through the reference's EnsembleRunner → InferenceRunner → MPInference."""
    ref = _reference_setup(args, rank)
    if ref is None:
        return _reference_unavailable(rank)
    from tornado_gcm.inference.production import EnsembleRunner, InferenceConfig, InferenceRunner
    from tornado_gcm.inference.runner import MPInference

    M = args.members
    x0 = torch.randn(7 * 37, ref.I, ref.J, generator=ref.gen).pin_memory()
    engine = MPInference(ref.model)
    f = {"f": ref.forc}

    def forecast(steps):
        with torch.no_grad():
            s0 = ref.encode(x0.to(ref.dev, non_blocking=True))
            cfg = InferenceConfig(outer_steps=steps, inner_steps=ref.cfg.inner_steps, chunk_size=steps,
                                  nan_guard=False)
            runner = InferenceRunner(engine, cfg, forcing_fn=lambda t: f, post_process_fn=ref.decode)
            return EnsembleRunner(runner, n_members=M).run(s0)

    forecast(max(1, args.warmup))
    sampler = ClockSampler(device_uuid()) if rank == 0 else None
    ms, clocks = timed_region(lambda i: forecast(args.steps), 1, world, sampler)
    value = world * M * args.steps / (ms / 1000.0)
    if rank == 0:
        print(json.dumps({
            "impl": "reference", "mode": "forecast", "metric": METRIC, "value": value,
            "unit": "6h model-steps/s (ensemble members x 6-h forecast steps, all GPUs)", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": value / PUBLISHED[args.resolution],
            "dtype": "fp32 (reference default path: FP64 SHT at TL63)", "data": "synthetic, random-init weights",
            "config": {"model": "2.8deg TL63 L32 reference model (as in the training arm), decoded every 6 h",
                       "global_batch": world * M, "seq_len": args.steps, "parallelism": f"dp{world} (members)",
                       "members": "reference EnsembleRunner: one member after another"},
            "clocks": clocks, "gpu_launches": 0,
        }), flush=True)


def main():
    args = parse_args()
    rank, world, local = dist_setup(args.gpus, need_group=args.parallel == "lat" and args.impl == "b200")
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_b200(args, rank, world)
    finally:
        import torch.distributed as dist

        if dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
