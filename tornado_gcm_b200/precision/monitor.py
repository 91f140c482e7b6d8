"""Precision diagnostics at zone boundaries (reference ``precision/monitor.py:20-118``).

Statistics are reduced on the device and fetched in one host sync per audit
(the reference issues one ``.item()`` per metric).
"""

from __future__ import annotations

import logging
from collections import defaultdict

import torch

logger = logging.getLogger(__name__)


class PrecisionMonitor:
    def __init__(self, enabled: bool = True):
        self.enabled = enabled
        self._metrics: dict[str, list[float]] = defaultdict(list)
        self._step = 0

    def step(self) -> None:
        self._step += 1

    @torch.no_grad()
    def audit_zone_transfer(self, name: str, x_high: torch.Tensor, x_low: torch.Tensor) -> None:
        if not self.enabled:
            return
        hi = x_high.detach()
        rt = x_low.detach().to(hi.dtype)
        ah = hi.abs()
        rel = ((hi - rt).abs() / (ah + 1e-30)).max()
        nan_rate = x_low.detach().isnan().float().mean()
        pos = ah > 0
        big = ah.max()
        small = torch.where(pos, ah, torch.full_like(ah, float("inf"))).min()
        dyn = torch.where(pos.any(), torch.log2(big + 1e-30) - torch.log2(small + 1e-30), torch.zeros_like(big))
        vals = torch.stack([rel.double(), nan_rate.double(), dyn.double()]).cpu().tolist()
        self._metrics[f"{name}/max_rel_error"].append(vals[0])
        self._metrics[f"{name}/nan_rate"].append(vals[1])
        self._metrics[f"{name}/dynamic_range_bits"].append(vals[2])

    @torch.no_grad()
    def audit_conservation(self, energy_before, energy_after, mass_before, mass_after) -> None:
        if not self.enabled:
            return
        e = 1e6 * (energy_after - energy_before).abs() / (energy_before.abs() + 1e-30)
        m = 1e6 * (mass_after - mass_before).abs() / (mass_before.abs() + 1e-30)
        v = torch.stack([e.double().max(), m.double().max()]).cpu().tolist()
        self._metrics["conservation/energy_drift_ppm"].append(v[0])
        self._metrics["conservation/mass_drift_ppm"].append(v[1])

    def summary(self, last_n: int = 10) -> dict[str, float]:
        return {k: sum(v[-last_n:]) / len(v[-last_n:]) for k, v in self._metrics.items() if v}

    def log_summary(self, last_n: int = 10) -> None:
        s = self.summary(last_n)
        if s:
            logger.info("\n".join([f"[PrecisionMonitor step={self._step}]"] +
                                  [f"  {k}: {v:.6g}" for k, v in sorted(s.items())]))

    def reset(self) -> None:
        self._metrics.clear()
        self._step = 0
