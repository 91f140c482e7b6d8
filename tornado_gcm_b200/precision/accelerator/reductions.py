"""FP64 reductions of the conservation path — reference
``precision/accelerator/triton_fixers.py:34-272`` (kernels K3/K4).

* :func:`sphere_integrate` — ``out[...] = Σ_{x,y} w[y] · z[..., x, y]``;
* :func:`spectral_norm` — ``out[...] = Σ_{m,l} x[..., m, l]²``;
* :func:`conservation_fix` — the lite mass + energy fixer.

The sm100 versions are one deterministic kernel launch each (one block per
output row, fixed reduction order, FP64 accumulation); the torch versions
are the FP64 oracle.
"""

from __future__ import annotations

from typing import Optional

import torch

from tornado_gcm_b200.ops import _ext


class KahanAccumulator:
    """Compensated FP64 running sum of tensors of a fixed shape."""

    def __init__(self, shape: tuple = (), device: torch.device | str = "cpu"):
        self.sum = torch.zeros(shape, dtype=torch.float64, device=device)
        self.comp = torch.zeros_like(self.sum)

    def add(self, x: torch.Tensor) -> None:
        y = x.to(torch.float64) - self.comp
        t = self.sum + y
        self.comp = (t - self.sum) - y
        self.sum = t

    def value(self) -> torch.Tensor:
        return self.sum

    def reset(self) -> None:
        self.sum.zero_()
        self.comp.zero_()


def sphere_integrate_torch(z: torch.Tensor, weights) -> torch.Tensor:
    w = torch.as_tensor(weights, dtype=torch.float64, device=z.device)
    return torch.einsum("y,...xy->...", w, z.to(torch.float64))


def spectral_norm_torch(x: torch.Tensor) -> torch.Tensor:
    return (x.to(torch.float64) ** 2).sum(dim=(-2, -1))


def sphere_integrate_sm100(z: torch.Tensor, weights) -> torch.Tensor:
    ops = _ext.require("sphere integral")
    w = torch.as_tensor(weights, dtype=torch.float64, device=z.device)
    return ops.sphere_integrate(z if z.dtype in (torch.float32, torch.float64) else z.float(), w)


def spectral_norm_sm100(x: torch.Tensor) -> torch.Tensor:
    ops = _ext.require("spectral norm")
    return ops.sum_squares(x if x.dtype in (torch.float32, torch.float64) else x.float(), 2)


def conservation_fix_sm100(state, state_before, fix_mass: bool = True, fix_energy: bool = True):
    from tornado_gcm_b200.ops import fixers as fixer_ops

    return fixer_ops.lite_fix(state, state_before, fix_mass, fix_energy)


def conservation_fix_torch(state, state_before, fix_mass: bool = True, fix_energy: bool = True):
    from tornado_gcm_b200.neural import fixers

    if fix_mass:
        state = fixers._mass_fix(state, state_before)
    if fix_energy:
        deficit = fixers.compute_total_energy_lite(state_before) - fixers.compute_total_energy_lite(state)
        state = fixers._energy_fix(state, deficit)
    return state


def _use_sm100(t: torch.Tensor, backend: Optional[str]) -> bool:
    return backend == "sm100" or (backend is None and t.is_cuda and _ext.available())


def sphere_integrate(z: torch.Tensor, weights, backend: Optional[str] = None) -> torch.Tensor:
    return sphere_integrate_sm100(z, weights) if _use_sm100(z, backend) else sphere_integrate_torch(z, weights)


def spectral_norm(x: torch.Tensor, backend: Optional[str] = None) -> torch.Tensor:
    return spectral_norm_sm100(x) if _use_sm100(x, backend) else spectral_norm_torch(x)


def has_sm100() -> bool:
    return torch.cuda.is_available() and _ext.available()
