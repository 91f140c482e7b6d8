"""Transform wrappers for neural pipelines — reference ``neural/spherical_harmonics.py:16-69``."""

from __future__ import annotations

import torch
import torch.nn as nn

from tornado_gcm_b200.core import spherical_harmonic


class FixedYlmMapping(nn.Module):
    """Non-learnable modal ↔ nodal mapping of a grid."""

    def __init__(self, grid):
        super().__init__()
        self.grid = grid

    def to_nodal(self, x: torch.Tensor) -> torch.Tensor:
        return self.grid.to_nodal(x)

    def to_modal(self, x: torch.Tensor) -> torch.Tensor:
        return self.grid.to_modal(x)

    def forward(self, x: torch.Tensor, direction: str = "to_nodal") -> torch.Tensor:
        if direction == "to_nodal":
            return self.to_nodal(x)
        if direction == "to_modal":
            return self.to_modal(x)
        raise ValueError(f"Unknown direction: {direction}")

    @property
    def nodal_shape(self):
        return self.grid.nodal_shape

    @property
    def modal_shape(self):
        return self.grid.modal_shape


class DivCurlTransform(nn.Module):
    """Nodal ``(u, v)`` → modal ``(vorticity, divergence)``."""

    def __init__(self, grid):
        super().__init__()
        self.grid = grid

    def forward(self, u_nodal: torch.Tensor, v_nodal: torch.Tensor):
        return spherical_harmonic.uv_nodal_to_vor_div_modal(self.grid, u_nodal, v_nodal)
