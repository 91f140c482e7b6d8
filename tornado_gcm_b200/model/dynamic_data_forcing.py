"""Time-varying forcing lookup — reference ``model/dynamic_data_forcing.py:34-89``.

``build_dynamic_data_forcing_torch`` returns ``forcing_fn(forcings, sim_time)``
selecting the row of a forcing time series whose ``sim_time`` is nearest (by
interpolating the index and rounding, the rule of the JAX original); rows
farther than ``dt_tolerance`` from the requested time come back as NaN.  The
whole series is moved to the device once, so a lookup is an index on the
device instead of a host→device copy per step.
"""

from __future__ import annotations

from typing import Any, Callable, Mapping

import numpy as np
import torch

ForcingFn = Callable[[dict, float], dict]


def build_dynamic_data_forcing_torch(forcing_data_nondim: Mapping[str, Any], *, dt_tolerance: float,
                                     device: torch.device | str) -> ForcingFn:
    data = {k: np.asarray(v) for k, v in forcing_data_nondim.items()}
    if "sim_time" not in data:
        raise KeyError("forcing_data must contain 'sim_time'")
    times = np.asarray(data["sim_time"], dtype=np.float64).reshape(-1)
    T = times.shape[0]
    for k, v in data.items():
        if k != "sim_time" and v.shape[0] != T:
            raise ValueError(f"Leading time length mismatch for {k}: expected {T}, got {v.shape[0]}")
    dev = torch.device(device)
    series = {k: torch.as_tensor(v, dtype=torch.float32, device=dev) for k, v in data.items()}

    def forcing_fn(_forcing_in: dict, sim_time) -> dict:
        st = float(sim_time.item()) if torch.is_tensor(sim_time) else float(sim_time)
        idx = 0 if T == 1 else int(np.clip(np.round(np.interp(st, times, np.arange(T, dtype=np.float64))), 0, T - 1))
        valid = abs(float(times[idx]) - st) <= float(dt_tolerance)
        out = {}
        for k, v in series.items():
            row = v[idx]
            out[k] = row if valid else torch.full_like(row, float("nan"))
        return out

    return forcing_fn
