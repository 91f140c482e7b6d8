"""Nodal fields ↔ token rows of the column networks (``csrc/tokens.cu``).

The column tower of the physics parameterization is pointwise over the
sphere: it sees one row of ``C`` input channels per grid column.  The
spectral transforms produce and consume latitude-major, channel-major nodal
fields ``(B, C, J, I)``.  :func:`nodal_to_tokens` turns such a field into
BF16 token rows ``(B·J·I, ld)`` — per-(channel, latitude) input factor
applied, forcing columns appended, zero padding to the 16-byte row the
tcgen05 linear layers read — and :func:`tokens_to_nodal` turns the tower's
output rows back into a nodal field with the output factor applied.  Each is
one tiled-transpose kernel, and each is the adjoint of the other, so the
backward pass uses the same two kernels.

This replaces the chain the reference's ``ForwardTower`` runs on every call
(``neural/towers.py:22-71``: move the feature axis last, flatten, cast, run
the network, move the axis back) plus the scale, concatenation and cast
around it.
"""

from __future__ import annotations

from typing import Optional

import torch

from tornado_gcm_b200.ops import _ext


class NodalToTokensFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, nod, scale, extra, ld: int):
        ops = _ext.require("nodal to tokens")
        ctx.scale, ctx.shape = scale, nod.shape
        tok = ops.nodal_to_tokens(nod.contiguous(), scale, extra, ld)
        return tok

    @staticmethod
    def backward(ctx, g):
        ops = _ext.require("nodal to tokens (adjoint)")
        B, C, J, I = ctx.shape
        return ops.tokens_to_nodal(g if g.stride(-1) == 1 else g.contiguous(), C, ctx.scale, B, J, I), None, None, None


class TokensToNodalFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tok, scale, B: int, J: int, I: int, ld_grad: int):
        ops = _ext.require("tokens to nodal")
        C = tok.shape[1]
        ctx.scale, ctx.C, ctx.ld_grad = scale, C, ld_grad
        return ops.tokens_to_nodal(tok, C, scale, B, J, I)

    @staticmethod
    def backward(ctx, g):
        ops = _ext.require("tokens to nodal (adjoint)")
        # BF16 rows padded with zeros to ld_grad: the network's backward reads them in place
        full = ops.nodal_to_tokens(g.contiguous(), ctx.scale, None, ctx.ld_grad)
        out = full[:, : ctx.C]
        out._tgcm_zero_padded = full  # marks the zero padding for the MLP backward
        return out, None, None, None, None, None


def nodal_to_tokens(nod: torch.Tensor, scale: torch.Tensor, extra: Optional[torch.Tensor], ld: int) -> torch.Tensor:
    """(B, C, J, I) fp32 → (B·J·I, ld) BF16; channel c scaled by ``scale[c, j]``; ``extra`` columns after C."""
    return NodalToTokensFn.apply(nod, scale.contiguous(), extra, int(ld))


def tokens_to_nodal(tok: torch.Tensor, scale: torch.Tensor, B: int, J: int, I: int, ld_grad: int) -> torch.Tensor:
    """(B·J·I, C) token rows (unit column stride) → (B, C, J, I) fp32 scaled by ``scale[c, j]``."""
    return TokensToNodalFn.apply(tok, scale.contiguous(), int(B), int(J), int(I), int(ld_grad))
