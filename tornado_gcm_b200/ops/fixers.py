"""FP64-accumulating conservation fixer kernels (``csrc/fixers.cu``).

:func:`packed_fix` applies the dry-air-mass and energy fixes of reference
``neural/fixers.py:228-326`` (``LiteConservationFixer``) to a packed state
``(B, C, 2M-1, L)`` in two launches (FP64 partial sums, then the corrected
copy), with a one-launch adjoint; :func:`lite_fix` is the same on
:class:`~tornado_gcm_b200.core.primitive_equations.State` objects.

Batch semantics: the reference sums its energy proxy over every dimension;
here each sample has its own deficit (the reference's behaviour for one
sample), so batched training matches per-sample runs.
"""

from __future__ import annotations

import torch

from tornado_gcm_b200.ops import _ext


def available() -> bool:
    return _ext.available()


class PackedFixFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, y_before, n: int, fix_mass: bool, fix_energy: int):
        ops = _ext.require("conservation fixer")
        y = y.contiguous()
        y_before = y_before.contiguous()
        out, part = ops.packed_fix(y, y_before, n, fix_mass, fix_energy)
        ctx.save_for_backward(y, y_before, part)
        ctx.cfg = (n, fix_mass, fix_energy)
        return out

    @staticmethod
    def backward(ctx, gout):
        y, yb, part = ctx.saved_tensors
        n, fm, fe = ctx.cfg
        ops = _ext.require("conservation fixer adjoint")
        need_b = ctx.needs_input_grad[1]
        res = ops.packed_fix_adjoint(gout.contiguous(), y, yb, part, n, fm, fe, need_b)
        return res[0], (res[1] if need_b else None), None, None, None


ENERGY_SPLIT = {"levels": 2, "reference": 1}


def packed_fix(y: torch.Tensor, y_before: torch.Tensor, n: int, fix_mass: bool = True,
               fix_energy: bool = True, energy_split: str = "levels") -> torch.Tensor:
    """Packed ``[ζ | δ | T' | ln ps | …]`` state with mass and energy restored to ``y_before``'s.

    ``energy_split="levels"`` adds 1/n of the energy deficit to each level's
    T'(0,0)², which restores the energy proxy exactly; ``"reference"`` adds the
    whole deficit at every level, as reference ``neural/fixers.py:309-321``
    does (n times the deficit in total).
    """
    if not (fix_mass or fix_energy):
        return y
    mode = ENERGY_SPLIT[energy_split] if fix_energy else 0
    return PackedFixFn.apply(y, y_before, int(n), bool(fix_mass), mode)


def lite_fix(state, state_before, fix_mass: bool = True, fix_energy: bool = True, energy_split: str = "levels"):
    """:class:`State` version of :func:`packed_fix` (tracers pass through)."""
    from tornado_gcm_b200.core.primitive_equations import State

    n = state.vorticity.shape[-3]
    lead = state.vorticity.shape[:-3]

    def pack(s):
        parts = [s.vorticity, s.divergence, s.temperature_variation, s.log_surface_pressure]
        x = torch.cat([p.float() for p in parts], dim=-3)
        return x.reshape(-1, *x.shape[-3:])

    out = packed_fix(pack(state), pack(state_before), n, fix_mass, fix_energy, energy_split)
    out = out.reshape(*lead, *out.shape[-3:]).to(state.vorticity.dtype)
    return State(out[..., :n, :, :], out[..., n:2 * n, :, :], out[..., 2 * n:3 * n, :, :],
                 out[..., 3 * n:3 * n + 1, :, :], state.tracers, state.sim_time)
