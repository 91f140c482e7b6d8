"""Dict ↔ tensor mappings around towers — reference ``neural/mappings.py:16-111``.

Inputs are packed in sorted-key order along the channel axis (``-3``), the
tower runs once on the packed tensor, and its output is split by the
declared output sizes (views, no copies).
"""

from __future__ import annotations

from typing import Dict, Sequence

import torch
import torch.nn as nn


class NodalMapping(nn.Module):
    def __init__(self, tower: nn.Module, output_keys: Sequence[str], output_sizes: Sequence[int]):
        super().__init__()
        if len(output_keys) != len(output_sizes):
            raise ValueError("output_keys and output_sizes differ in length")
        self.tower = tower
        self.output_keys = list(output_keys)
        self.output_sizes = [int(s) for s in output_sizes]

    @staticmethod
    def _pack(inputs: Dict[str, torch.Tensor]) -> torch.Tensor:
        return torch.cat([v.unsqueeze(0) if v.ndim == 2 else v for _, v in sorted(inputs.items())], dim=-3)

    def _unpack(self, y: torch.Tensor) -> Dict[str, torch.Tensor]:
        return dict(zip(self.output_keys, torch.split(y, self.output_sizes, dim=-3)))

    def forward(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        return self._unpack(self.tower(self._pack(inputs)))


class NodalVolumeMapping(nn.Module):
    """Stack ``(levels, lon, lat)`` inputs as channels, keep the level axis."""

    def __init__(self, tower: nn.Module, output_keys: Sequence[str]):
        super().__init__()
        self.tower = tower
        self.output_keys = list(output_keys)

    def forward(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        y = self.tower(torch.stack([inputs[k] for k in sorted(inputs)], dim=0))
        return {k: y[i] for i, k in enumerate(self.output_keys)}


class ParallelMapping(nn.Module):
    """Sum of several mappings' outputs (keys of the first mapping)."""

    def __init__(self, mappings: Sequence[nn.Module]):
        super().__init__()
        self.mappings = nn.ModuleList(mappings)

    def forward(self, inputs: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        results = [m(inputs) for m in self.mappings]
        out = dict(results[0])
        for r in results[1:]:
            for k in out:
                if k in r:
                    out[k] = out[k] + r[k]
        return out
