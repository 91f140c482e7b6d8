"""Layer coordinates for shallow-water style models (reference ``core/layer_coordinates.py``)."""

from __future__ import annotations

import dataclasses

import numpy as np


@dataclasses.dataclass(frozen=True)
class LayerCoordinates:
    layers: int

    @property
    def centers(self) -> np.ndarray:
        return np.arange(self.layers, dtype=np.float64)

    def asdict(self):
        return {"layers": self.layers}
