"""Distributed spherical-harmonic transform micro-benchmark.

Forward (nodal → modal) plus inverse transforms of ``F`` stacked fields on
latitude-sharded grids (TL63 / TL127 / TL255 / TL511), TF32 and FP64, on
``W`` GPUs (one process per GPU, ``torchrun``).  Arms:

* ``fused`` — tcgen05 local transforms; the Legendre analysis GEMM adds its
  output into every rank's symmetric buffer over NVLink (cross-GPU sum fused
  into the GEMM epilogue) plus one peer barrier kernel;
* ``nccl`` — the same partial transforms followed by
  ``torch.distributed.all_reduce`` (the baseline a NCCL build would run);
* ``fp64`` — torch FP64 partial sums + NCCL (the precision oracle path);
* on one GPU: the full transform.

Times are CUDA-event device times per forward+inverse pair, max over ranks.
Reported per arm: milliseconds, effective GB/s (nodal + modal bytes moved
through the transform), TFLOP/s (Fourier + Legendre GEMM flops of this rank)
and the modal bytes that crossed NVLink per rank.

    torchrun --nproc-per-node 2 -m tornado_gcm_b200.parallel.dsht_bench --grids TL63 TL127 --fields 32 128
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist


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


def run(grids, fields, iters: int, warmup: int) -> list:
    from tornado_gcm_b200.core import spherical_harmonic as shm
    from tornado_gcm_b200.parallel.sharded_sht import LatitudeShardedSHT

    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    dev = torch.device("cuda", torch.cuda.current_device())
    rows = []
    for gname in grids:
        g = getattr(shm.Grid, gname)(precision="tf32")
        M2, L = g.modal_shape
        I, J = g.nodal_shape
        for F in fields:
            gen = torch.Generator(device="cpu").manual_seed(0)
            l = torch.arange(L, dtype=torch.float64)
            modal = (torch.randn(F, M2, L, generator=gen, dtype=torch.float64) * torch.as_tensor(g.mask)
                     * (1.0 + l) ** -1.5).float().to(dev)
            res = {"grid": gname, "fields": F, "gpus": world}
            if world == 1:
                def full():
                    g.to_modal(g.to_nodal(modal))
                ms = _time(full, iters, warmup)
                res["single_ms"] = ms
            else:
                sht = LatitudeShardedSHT(g, scheme="mirrored")
                sht.enable_fused(F, dev)
                nodal_local = sht.to_nodal_gpu(modal)

                def fused():
                    with torch.no_grad():
                        sht.to_modal_fused(sht.to_nodal_gpu(modal))

                def nccl():
                    part = sht.partial_to_modal(sht.to_nodal_gpu(modal)).contiguous()
                    dist.all_reduce(part)

                res["fused_ms"] = _time(fused, iters, warmup)
                res["nccl_ms"] = _time(nccl, iters, warmup)
                g64 = getattr(shm.Grid, gname)(precision="highest")
                s64 = LatitudeShardedSHT(g64, scheme="mirrored")
                m64 = modal.double()

                def fp64():
                    part = s64.partial_to_modal(s64.to_nodal(m64)).contiguous()
                    dist.all_reduce(part)

                if F <= 32:
                    res["fp64_nccl_ms"] = _time(fp64, max(2, iters // 4), 1)
                # accuracy of the fused path against the FP64 round trip
                with torch.no_grad():
                    out = sht.to_modal_fused(sht.to_nodal_gpu(modal))
                    ref = g64.to_modal(g64.to_nodal(m64))
                res["fused_rel_err"] = float((out.double() - ref).norm() / ref.norm())
                del nodal_local
            jl = J // world
            flops = 2.0 * F * (M2 * I * jl + M2 * jl * L) * 2  # Fourier + Legendre, forward + inverse
            bytes_moved = 4.0 * F * (I * jl + M2 * L) * 2
            for key in ("single_ms", "fused_ms", "nccl_ms"):
                if key in res:
                    res[key.replace("_ms", "_tflops")] = flops / (res[key] * 1e-3) / 1e12
                    res[key.replace("_ms", "_gbs")] = bytes_moved / (res[key] * 1e-3) / 1e9
            res["nvlink_bytes_per_rank"] = 4.0 * F * M2 * L * world if world > 1 else 0.0
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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    try:
        run(args.grids, args.fields, args.iters, args.warmup)
    finally:
        if dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
