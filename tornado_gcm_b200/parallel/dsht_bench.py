"""Distributed spherical-harmonic transform micro-benchmark.

Forward (nodal → modal) plus inverse (modal → nodal) transforms of ``F``
stacked fields with the sphere sharded over ``W`` GPUs the way the model
step shards it (modal rows by zonal wavenumber, nodal columns by latitude
block; :mod:`tornado_gcm_b200.parallel.spectral_shard`), at TL63 … TL511,
TF32 and FP64.  One process per GPU (``torchrun``).  Arms:

* ``fused`` (TF32) — tcgen05 Legendre GEMMs whose epilogues do the
  grid ↔ spectral transpose (peer stores / peer reductions over NVLink)
  plus one peer barrier per transform;
* ``nccl`` (TF32) — the same local tcgen05 transforms with the transpose done
  by NCCL (all-gather of the modal rows before synthesis, all-reduce of the
  partial Legendre sums after analysis): the baseline a NCCL build runs;
* ``fp64`` — FP64 tensor-core (DMMA) transforms with the NCCL transpose;
* on one GPU: the full-grid transforms (TF32 tcgen05 and FP64 DMMA).

Times are CUDA-event device times per forward+inverse pair, max over ranks.
Per arm: ms, TFLOP/s (this rank's GEMM flops), GB/s (nodal + modal bytes of
this rank through both transforms) and the fraction of the roofline, the
slower of compute at the measured peak (TF32: half the measured BF16 GEMM
rate; FP64: the nominal 40 TFLOP/s) and this rank's NVLink bytes at the
measured 770 GB/s per direction.

    torchrun --nproc-per-node 2 -m tornado_gcm_b200.parallel.dsht_bench --grids TL63 TL127 --fields 32 128
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0          # measured peer copy per direction per GPU
FP64_TFLOPS = 40.0          # nominal B200 FP64 (tensor core) rate


def _peaks() -> dict:
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            d = json.load(fh)
        return {"tf32": float(d["bf16_tflops"]) / 2.0, "fp64": FP64_TFLOPS}
    except Exception:
        return {"tf32": 1590.0 / 2.0, "fp64": FP64_TFLOPS}


def _time(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / iters
    if dist.is_initialized():
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


class _NcclTransforms:
    """Local transforms with the transpose done by NCCL collectives (TF32 tcgen05 or FP64 DMMA)."""

    def __init__(self, lay, precision: str, device):
        from tornado_gcm_b200.ops import sht as sht_ops

        self.lay = lay
        self.precision = precision
        sh = lay.grid.spherical_harmonics
        sl = lay.lat_slice()
        if precision == "tf32":
            full = sht_ops.bases(sh, device)
            idx = torch.arange(sl.start, sl.stop, device=device)
            from tornado_gcm_b200.parallel.sharded_sht import _LocalBases

            self.lb = _LocalBases(full, idx)
        else:
            self.p = sh.device_basis("p", device, torch.float64)[:, sl, :].contiguous()
            self.f = sh.device_basis("f", device, torch.float64)
            self.w = sh.device_basis("w", device, torch.float64)[sl].contiguous()
        self.rows = torch.as_tensor(lay.rows, device=device)

    def _gather(self, x_loc):
        lay = self.lay
        parts = [torch.empty_like(x_loc) for _ in range(lay.world)]
        dist.all_gather(parts, x_loc.contiguous())
        full = x_loc.new_zeros(x_loc.shape[:-2] + (lay.M2, x_loc.shape[-1]))
        for r, p in enumerate(parts):
            ok = self.rows[r] >= 0
            full[..., self.rows[r][ok], :] = p[..., ok, :]
        return full

    def _local_rows(self, full):
        dist.all_reduce(full)
        ok = self.rows[self.lay.rank] >= 0
        out = full.new_zeros(full.shape[:-2] + (self.lay.M2_loc, full.shape[-1]))
        out[..., ok, :] = full[..., self.rows[self.lay.rank][ok], :]
        return out

    def synth(self, x_loc):
        from tornado_gcm_b200.ops import _ext

        ops = _ext.require("benchmark")
        full = self._gather(x_loc)
        if self.precision == "tf32":
            lb = self.lb
            x3 = torch.nn.functional.pad(full, (0, lb.Lp - lb.L))[..., :lb.L]
            ws = _ext.empty(x3.shape[0] * lb.J * lb.M2p, dtype=torch.float32, device=x3.device)
            return ops.sht_synth(x3, lb.L, lb.P, lb.F, ws, None, _ext.error_flag(x3.device), True)
        S, M2, L = full.shape
        J = self.p.shape[1]
        I = self.f.shape[0]
        W = torch.empty(M2, S, J, dtype=torch.float64, device=full.device)
        ops.dgemm_strided(full, self.p, W, S, J, L, M2, [M2 * L, 1, L], [L, 1, J * L], [J, 1, S * J], 1.0, 0.0, None)
        out = torch.empty(S, I, J, dtype=torch.float64, device=full.device)
        ops.dgemm_strided(self.f, W, out, I, J, M2, S, [M2, 1, 0], [1, S * J, J], [J, 1, I * J], 1.0, 0.0, None)
        return out

    def anal(self, nodal):
        from tornado_gcm_b200.ops import _ext

        ops = _ext.require("benchmark")
        if self.precision == "tf32":
            lb = self.lb
            ws = _ext.empty(nodal.shape[0] * lb.M2 * lb.J, dtype=torch.float32, device=nodal.device)
            part = ops.sht_anal(nodal, lb.Ft, lb.Ptw, lb.L, ws, None, _ext.error_flag(nodal.device), True, None)
            return self._local_rows(part.contiguous())
        S, I, J = nodal.shape
        M2, L = self.p.shape[0], self.p.shape[2]
        Z = torch.empty(M2, S, J, dtype=torch.float64, device=nodal.device)
        ops.dgemm_strided(self.f, nodal.contiguous(), Z, M2, J, I, S, [1, M2, 0], [1, J, I * J], [S * J, 1, J], 1.0,
                          0.0, self.w)
        out = torch.empty(S, M2, L, dtype=torch.float64, device=nodal.device)
        ops.dgemm_strided(Z, self.p, out, S, L, J, M2, [J, 1, S * J], [1, L, J * L], [M2 * L, 1, L], 1.0, 0.0, None)
        return self._local_rows(out)


def run(grids, fields, iters: int, warmup: int) -> list:
    from tornado_gcm_b200.core import spherical_harmonic as shm
    from tornado_gcm_b200.parallel import spectral_shard as ss

    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    dev = torch.device("cuda", torch.cuda.current_device())
    peaks = _peaks()
    rows = []
    for gname in grids:
        g = getattr(shm.Grid, gname)(precision="tf32")
        M2, L = g.modal_shape
        I, J = g.nodal_shape
        for F in fields:
            gen = torch.Generator(device="cpu").manual_seed(0)
            l = torch.arange(L, dtype=torch.float64)
            modal = (torch.randn(F, M2, L, generator=gen, dtype=torch.float64) * torch.as_tensor(g.mask)
                     * (1.0 + l) ** -1.5)
            res = {"grid": gname, "fields": F, "gpus": world}
            jl = J // world
            flops = {}
            if world == 1:
                m32 = modal.float().to(dev)
                g64 = getattr(shm.Grid, gname)(precision="highest")
                m64 = modal.to(dev)
                res["tf32_ms"] = _time(lambda: g.to_modal(g.to_nodal(m32)), iters, warmup)
                res["fp64_ms"] = _time(lambda: g64.to_modal(g64.to_nodal(m64)), max(2, iters // 2), 1)
                arms = {"tf32": "tf32", "fp64": "fp64"}
                nv = 0.0
            else:
                sg = ss.make_sharded_grid(g, None, "fused", dev)
                lay = sg.layout
                x_loc = lay.scatter_modal(modal).float().to(dev)
                with torch.no_grad():
                    res["fused_ms"] = _time(lambda: sg.to_modal_lat_major(sg.to_nodal_lat_major(x_loc)), iters,
                                            warmup)
                    nccl = _NcclTransforms(lay, "tf32", dev)
                    res["nccl_ms"] = _time(lambda: nccl.anal(nccl.synth(x_loc)), iters, warmup)
                    f64 = _NcclTransforms(lay, "fp64", dev)
                    x64 = lay.scatter_modal(modal).to(dev)
                    res["fp64_ms"] = _time(lambda: f64.anal(f64.synth(x64)), max(2, iters // 2), 1)
                    out = sg.to_modal_lat_major(sg.to_nodal_lat_major(x_loc))
                    ref = lay.scatter_modal(g.with_precision("highest").to_modal(
                        g.with_precision("highest").to_nodal(modal)))
                    res["fused_rel_err"] = float((out.double().cpu() - ref).norm() / ref.norm())
                arms = {"fused": "tf32", "nccl": "tf32", "fp64": "fp64"}
                # bytes leaving this rank: synthesis rows (own m, other latitudes) + analysis partial sums
                nv = 4.0 * F * ((M2 / world) * J + M2 * L) * (world - 1) / world
            # GEMM flops of this rank: Fourier over its latitudes + Legendre (half-triangle synthesis)
            flops_rank = 2.0 * F * (M2 * I * jl * 2 + M2 * jl * L * 1.5)
            bytes_rank = 4.0 * F * (I * jl + M2 * L / world) * 2
            for arm, prec in arms.items():
                ms = res[arm + "_ms"]
                eb = 8.0 if prec == "fp64" else 4.0
                res[arm + "_tflops"] = flops_rank / (ms * 1e-3) / 1e12
                res[arm + "_gbs"] = bytes_rank * eb / 4.0 / (ms * 1e-3) / 1e9
                t_roof = max(flops_rank / (peaks[prec] * 1e12), nv * (eb / 4.0 if arm == "fp64" else 1.0)
                             / (NVLINK_GBS * 1e9))
                res[arm + "_roofline_frac"] = t_roof / (ms * 1e-3)
            res["nvlink_bytes_per_rank"] = nv
            rows.append(res)
            if rank == 0:
                print(json.dumps(res), flush=True)
    return rows


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--grids", nargs="+", default=["TL63", "TL127", "TL255", "TL511"])
    ap.add_argument("--fields", nargs="+", type=int, default=[32, 128])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    args = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    try:
        run(args.grids, args.fields, args.iters, args.warmup)
    finally:
        if dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
