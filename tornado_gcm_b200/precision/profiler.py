"""SDA profiler: precision audits + gradient/spectral statistics + zone timing
(reference ``precision/profiler.py:33-281``).

Gradient statistics are reduced on the device for all parameters at once
and fetched with a single host copy (the reference syncs per parameter);
zone timers use CUDA events when tensors live on a GPU, so GPU zone times
are device times rather than host wall time.
"""

from __future__ import annotations

import dataclasses
import json
import time
from collections import defaultdict, deque
from dataclasses import field
from typing import Any, Optional

import torch

from tornado_gcm_b200.precision.monitor import PrecisionMonitor
from tornado_gcm_b200.precision.policy import PrecisionZone


@dataclasses.dataclass
class GradientStats:
    mean: float = 0.0
    std: float = 0.0
    max_abs: float = 0.0
    min_abs: float = 0.0
    nan_count: int = 0
    numel: int = 0


@dataclasses.dataclass
class ProfilerMetrics:
    step: int = 0
    zone_timing: dict = field(default_factory=dict)
    zone_memory: dict = field(default_factory=dict)
    conservation_drift_ppm: dict = field(default_factory=dict)
    gradient_stats: dict = field(default_factory=dict)
    spectral_energy_tail: float = 0.0
    transfer_max_error: dict = field(default_factory=dict)
    warnings: list = field(default_factory=list)
    recent_losses: list = field(default_factory=list)
    nan_count: int = 0


class SDAProfiler(PrecisionMonitor):
    def __init__(self, config) -> None:
        super().__init__(enabled=config.enabled)
        self.config = config
        self._gradient_stats: dict = {}
        self._spectral_tail = 0.0
        self._zone_timers: dict = defaultdict(float)
        self._active: Optional[tuple] = None
        self._loss_history: deque = deque(maxlen=1000)
        self._nan_counter = 0

    def should_sample(self) -> bool:
        return self.enabled and self._step % max(self.config.sample_rate, 1) == 0

    @torch.no_grad()
    def audit_gradient_stats(self, named_parameters: Any) -> None:
        if not self.enabled or not self.config.gradient_audit:
            return
        self._gradient_stats.clear()
        names, rows = [], []
        for name, p in named_parameters:
            if p.grad is None:
                continue
            g = p.grad.detach().float().reshape(-1)
            nan = torch.isnan(g).sum().float()
            gc = torch.nan_to_num(g, 0.0)
            a = gc.abs()
            pos_min = torch.where(a > 0, a, torch.full_like(a, float("inf"))).min()
            rows.append(torch.stack([gc.mean(), gc.std() if gc.numel() > 1 else torch.zeros((), device=g.device),
                                     a.max(), torch.where(torch.isinf(pos_min), torch.zeros_like(pos_min), pos_min),
                                     nan, torch.tensor(float(g.numel()), device=g.device)]))
            names.append(name)
        if not rows:
            return
        vals = torch.stack(rows).cpu().tolist()
        for n, v in zip(names, vals):
            gs = GradientStats(v[0], v[1], v[2], v[3], int(v[4]), int(v[5]))
            self._gradient_stats[n] = gs
            self._nan_counter += gs.nan_count

    @torch.no_grad()
    def audit_spectral_energy(self, modal_tensor: torch.Tensor, cutoff_fraction: float = 0.5) -> None:
        if not self.enabled or not self.config.spectral_audit:
            return
        t = modal_tensor.detach().float()
        L = t.shape[-1]
        c = int(L * cutoff_fraction)
        tot, high = torch.stack([(t * t).sum(), (t[..., c:] ** 2).sum()]).cpu().tolist()
        self._spectral_tail = 0.0 if tot < 1e-30 else high / tot

    def start_zone_timer(self, zone: PrecisionZone) -> None:
        if not self.enabled or not self.config.performance_counters:
            return
        if self._active is not None:
            self._stop_active()
        if torch.cuda.is_available():
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._active = (zone.value, ev)
        else:
            self._active = (zone.value, time.perf_counter())

    def stop_zone_timer(self) -> None:
        if self._active is not None:
            self._stop_active()

    def _stop_active(self):
        name, start = self._active
        if isinstance(start, float):
            self._zone_timers[name] += time.perf_counter() - start
        else:
            end = torch.cuda.Event(enable_timing=True)
            end.record()
            end.synchronize()
            self._zone_timers[name] += start.elapsed_time(end) / 1000.0
        self._active = None

    def record_loss(self, loss_value: float) -> None:
        self._loss_history.append(float(loss_value))
        if loss_value != loss_value:
            self._nan_counter += 1

    def collect(self) -> ProfilerMetrics:
        transfer = {k: v[-1] for k, v in self._metrics.items() if k.endswith("/max_rel_error") and v}
        cons = {k: self._metrics[k][-1] for k in ("conservation/energy_drift_ppm", "conservation/mass_drift_ppm")
                if self._metrics.get(k)}
        warnings = []
        if self._nan_counter:
            warnings.append(f"NaN detected: {self._nan_counter} occurrences")
        if self.config.spectral_audit and self._spectral_tail > 0.1:
            warnings.append(f"High spectral tail energy: {self._spectral_tail:.4f}")
        for n, gs in self._gradient_stats.items():
            if gs.nan_count:
                warnings.append(f"NaN gradients in {n}: {gs.nan_count}")
            if gs.max_abs > 1e6:
                warnings.append(f"Gradient explosion in {n}: max={gs.max_abs:.2e}")
        mem = {}
        if torch.cuda.is_available():
            mem["allocated"] = int(torch.cuda.memory_allocated())
            mem["peak"] = int(torch.cuda.max_memory_allocated())
        return ProfilerMetrics(self._step, dict(self._zone_timers), mem, cons, dict(self._gradient_stats),
                               self._spectral_tail, transfer, warnings, list(self._loss_history)[-20:],
                               self._nan_counter)

    def summary(self, last_n: int = 10) -> dict:
        base = super().summary(last_n)
        for z, t in self._zone_timers.items():
            base[f"zone_time/{z}"] = t
        if self._spectral_tail > 0:
            base["spectral/energy_tail"] = self._spectral_tail
        if self._gradient_stats:
            base["gradient/max_abs"] = max(g.max_abs for g in self._gradient_stats.values())
            base["gradient/total_nans"] = float(sum(g.nan_count for g in self._gradient_stats.values()))
        return base

    def export_json(self, path: str) -> None:
        with open(path, "w", encoding="utf-8") as fh:
            json.dump(dataclasses.asdict(self.collect()), fh, indent=2, default=str)

    def log_to_tensorboard(self, writer: Any, global_step: int) -> None:
        for k, v in self.summary().items():
            writer.add_scalar(f"sda/{k}", v, global_step)

    def reset(self) -> None:
        super().reset()
        self._gradient_stats.clear()
        self._spectral_tail = 0.0
        self._zone_timers.clear()
        self._active = None
        self._loss_history.clear()
        self._nan_counter = 0
