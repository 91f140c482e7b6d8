"""WeatherBench-style (u, v, t, z) state container (reference ``core/weatherbench_utils.py``)."""

from __future__ import annotations

import dataclasses
from typing import Optional

import torch


@dataclasses.dataclass
class State:
    u: torch.Tensor
    v: torch.Tensor
    t: torch.Tensor
    z: torch.Tensor
    sim_time: Optional[float] = None
    tracers: dict = dataclasses.field(default_factory=dict)
    diagnostics: dict = dataclasses.field(default_factory=dict)

    def _map(self, fn, other=None):
        if other is None:
            return State(fn(self.u), fn(self.v), fn(self.t), fn(self.z), self.sim_time,
                         {k: fn(x) for k, x in self.tracers.items()},
                         {k: fn(x) for k, x in self.diagnostics.items()})
        return State(fn(self.u, other.u), fn(self.v, other.v), fn(self.t, other.t), fn(self.z, other.z),
                     self.sim_time, {k: fn(x, other.tracers[k]) for k, x in self.tracers.items()},
                     {k: fn(x, other.diagnostics[k]) for k, x in self.diagnostics.items()})

    def __add__(self, other):
        return self._map(torch.add, other)

    def __mul__(self, s):
        return self._map(lambda x: x * s)

    __rmul__ = __mul__

    def tree_map(self, fn):
        return self._map(fn)
