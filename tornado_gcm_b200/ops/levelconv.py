"""Vertical (level-axis) convolution towers on the tcgen05 BF16 GEMMs.

A ``ConvLevel`` layer with kernel k and 'same' padding is lowered onto the
token rows (column, level): ``csrc/levelconv.cu`` builds the BF16 operand
whose row holds the k level-neighbours of a token side by side, and the
layer is then one tcgen05 linear GEMM with the bias and ReLU fused into its
epilogue (``csrc/gemm.cu``).  Backward: weight gradient = the split-K wgrad
GEMM on the re-lowered input, bias gradient = a column sum, input gradient =
the dgrad GEMM folded back onto the levels by ``level_col2im`` with the
previous layer's ReLU derivative applied in the same pass.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from tornado_gcm_b200.ops import _ext


def _pad8(n: int) -> int:
    return (n + 7) // 8 * 8


def supports(tower, x: torch.Tensor) -> bool:
    """The tower's layers map onto the lowered GEMMs (odd kernels, 'same' padding, ReLU, no dilation)."""
    if not (x.is_cuda and _ext.available() and tower.activation is F.relu):
        return False
    for lyr in tower.layers:
        c = getattr(lyr, "conv", None)
        if not isinstance(c, nn.Conv1d) or c.kernel_size[0] % 2 == 0 or c.dilation[0] != 1 or c.stride[0] != 1 \
                or c.groups != 1 or c.padding not in ("same", (c.kernel_size[0] // 2,)):
            return False
    return True


def _lowered_weight(conv: nn.Conv1d, ld: int) -> torch.Tensor:
    """(Cout, Cin, k) → BF16 (pad8(Cout), ld) with column t*Cin + ci holding W[co, ci, t]."""
    co, ci, k = conv.weight.shape
    w2 = torch.zeros(_pad8(co), ld, dtype=torch.bfloat16, device=conv.weight.device)
    w2[:co, : k * ci] = conv.weight.detach().permute(0, 2, 1).reshape(co, k * ci)
    return w2


def _padded_bias(conv: nn.Conv1d) -> torch.Tensor | None:
    if conv.bias is None:
        return None
    b = torch.zeros(_pad8(conv.out_channels), dtype=torch.float32, device=conv.bias.device)
    b[: conv.out_channels] = conv.bias.detach()
    return b


class _LevelLowering:
    """(column, level) token rows; taps along the level axis."""

    def __init__(self, L: int):
        self.L = L

    def taps(self, conv) -> int:
        return conv.kernel_size[0]

    def weight(self, conv, ld: int) -> torch.Tensor:
        return _lowered_weight(conv, ld)

    def lower(self, ops, h, ci, conv, ld):
        return ops.level_im2col(h, self.L, ci, conv.kernel_size[0], ld)

    def fold(self, ops, dA, ci, conv, pre):
        return ops.level_col2im(dA, self.L, ci, conv.kernel_size[0], pre, 1 if pre is not None else 0)

    def grad_weight(self, dw2, conv):
        co, ci, k = conv.weight.shape
        return dw2[:co, : k * ci].reshape(co, k, ci).permute(0, 2, 1).contiguous()


class _LonLatLowering:
    """(batch, lon, lat) token rows; taps over (lon, lat), circular in longitude, zero-padded in latitude."""

    def __init__(self, I: int, J: int, dilation: int):
        self.I, self.J, self.dil = I, J, dilation

    def taps(self, conv) -> int:
        return conv.kernel_size[0] * conv.kernel_size[1]

    def weight(self, conv, ld: int) -> torch.Tensor:
        co, ci, kl, kt = conv.weight.shape
        w2 = torch.zeros(_pad8(co), ld, dtype=torch.bfloat16, device=conv.weight.device)
        w2[:co, : kl * kt * ci] = conv.weight.detach().permute(0, 2, 3, 1).reshape(co, kl * kt * ci)
        return w2

    def lower(self, ops, h, ci, conv, ld):
        kl, kt = conv.kernel_size
        return ops.lonlat_im2col(h, self.I, self.J, ci, kl, kt, self.dil, ld)

    def fold(self, ops, dA, ci, conv, pre):
        kl, kt = conv.kernel_size
        return ops.lonlat_col2im(dA, self.I, self.J, ci, kl, kt, self.dil, pre, 1 if pre is not None else 0)

    def grad_weight(self, dw2, conv):
        co, ci, kl, kt = conv.weight.shape
        return dw2[:co, : kl * kt * ci].reshape(co, kl, kt, ci).permute(0, 3, 1, 2).contiguous()


class LevelConvTowerFn(torch.autograd.Function):
    """A stack of convolutions, each one lowered GEMM (ReLU between layers, optionally after the last)."""

    @staticmethod
    def forward(ctx, x2d, lowering, convs, act_final: bool, *params):
        ops = _ext.require("convolution tower")
        err = _ext.error_flag(x2d.device)
        n = len(convs)
        h = x2d
        hs, pres, ws = [], [], []
        for i, conv in enumerate(convs):
            co, ci = conv.weight.shape[:2]
            ld = _pad8(lowering.taps(conv) * ci)
            A = lowering.lower(ops, h, ci, conv, ld)
            w2 = lowering.weight(conv, ld)
            relu = i < n - 1 or act_final
            last = i == n - 1
            out = torch.empty(A.shape[0], w2.shape[0], dtype=torch.float32 if last else torch.bfloat16,
                              device=x2d.device)
            aux = torch.empty(A.shape[0], w2.shape[0], dtype=torch.bfloat16, device=x2d.device) if relu else None
            ops.linear_fwd(A, w2, _padded_bias(conv), 1 if relu else 0, out, aux, err)
            hs.append(h)
            pres.append(aux)
            ws.append(w2)
            h = out
        ctx.lowering, ctx.convs, ctx.act_final = lowering, convs, act_final
        ctx.save_for_backward(*(hs + [p if p is not None else torch.empty(0) for p in pres] + ws))
        return h[:, : convs[-1].out_channels]

    @staticmethod
    def backward(ctx, g):
        ops = _ext.require("convolution tower backward")
        convs, low = ctx.convs, ctx.lowering
        n = len(convs)
        saved = ctx.saved_tensors
        hs, pres, ws = saved[:n], saved[n:2 * n], saved[2 * n:]
        err = _ext.error_flag(g.device)
        co_last = convs[-1].out_channels
        dy = torch.zeros(g.shape[0], ws[-1].shape[0], dtype=torch.bfloat16, device=g.device)
        dy[:, :co_last] = g
        if ctx.act_final and pres[-1].numel():
            dy = dy * (pres[-1] > 0)
        grads = [None] * n
        dx = None
        for i in range(n - 1, -1, -1):
            conv = convs[i]
            co, ci = conv.weight.shape[:2]
            ld = ws[i].shape[1]
            A = low.lower(ops, hs[i], ci, conv, ld)
            dw2 = torch.zeros(ws[i].shape, dtype=torch.float32, device=g.device)
            ops.linear_wgrad(dy, A, dw2, 0, err)
            gw = low.grad_weight(dw2, conv).to(conv.weight.dtype)
            gb = ops.colsum_bf16(dy, co).to(conv.bias.dtype) if conv.bias is not None else None
            grads[i] = (gw, gb)
            dA = torch.empty(dy.shape[0], ld, dtype=torch.bfloat16, device=g.device)
            ops.linear_dgrad(dy, ws[i], dA, None, 0, err)
            pre = pres[i - 1] if i > 0 and pres[i - 1].numel() else None
            dxi = low.fold(ops, dA, ci, conv, pre)
            if i > 0:
                dy = torch.zeros(dxi.shape[0], ws[i - 1].shape[0], dtype=torch.bfloat16, device=g.device)
                dy[:, :ci] = dxi
            else:
                dx = dxi
        flat = []
        for conv, (gw, gb) in zip(convs, grads):
            flat.append(gw)
            if conv.bias is not None:
                flat.append(gb)
        return (dx.to(ctx.saved_tensors[0].dtype) if dx is not None else None, None, None, None) + tuple(flat)


def level_conv_tower(tower, x: torch.Tensor) -> torch.Tensor:
    """``(..., channels, levels, lon, lat)`` through the tower on the lowered GEMMs."""
    *batch, c, levels, lon, lat = x.shape
    nb = len(batch)
    lead = tuple(range(nb))
    tok = x.permute(*lead, nb + 2, nb + 3, nb + 1, nb)          # (..., lon, lat, levels, c)
    x2d = tok.reshape(-1, c).float().contiguous()
    convs = tuple(lyr.conv for lyr in tower.layers)
    params = []
    for cv in convs:
        params.append(cv.weight)
        if cv.bias is not None:
            params.append(cv.bias)
    out = LevelConvTowerFn.apply(x2d, _LevelLowering(int(levels)), convs, bool(tower.activate_final), *params)
    oc = out.shape[-1]
    out = out.reshape(*batch, lon, lat, levels, oc)
    return out.permute(*lead, nb + 3, nb + 2, nb, nb + 1).to(x.dtype)  # (..., oc, levels, lon, lat)


def supports_lonlat(tower, x: torch.Tensor) -> bool:
    """Conv2DTower of ConvLonLat layers with odd kernels, one dilation, ReLU."""
    if not (x.is_cuda and _ext.available() and tower.activation is F.relu):
        return False
    dil = {getattr(lyr, "dilation", None) for lyr in tower.layers}
    if len(dil) != 1 or None in dil:
        return False
    for lyr in tower.layers:
        c = getattr(lyr, "conv", None)
        d = lyr.dilation
        if not isinstance(c, nn.Conv2d) or c.kernel_size[0] % 2 == 0 or c.kernel_size[1] % 2 == 0 \
                or c.stride != (1, 1) or c.groups != 1 or c.padding not in ((0, 0), "valid") \
                or c.dilation != (d, d):
            return False
    return True


def lonlat_conv_tower(tower, x: torch.Tensor) -> torch.Tensor:
    """``(..., channels, lon, lat)`` through a Conv2DTower on the lowered GEMMs."""
    *batch, c, lon, lat = x.shape
    nb = len(batch)
    lead = tuple(range(nb))
    x2d = x.permute(*lead, nb + 1, nb + 2, nb).reshape(-1, c).float().contiguous()   # (..., lon, lat, c) rows
    convs = tuple(lyr.conv for lyr in tower.layers)
    params = []
    for cv in convs:
        params.append(cv.weight)
        if cv.bias is not None:
            params.append(cv.bias)
    low = _LonLatLowering(int(lon), int(lat), int(tower.layers[0].dilation))
    out = LevelConvTowerFn.apply(x2d, low, convs, bool(tower.activate_final), *params)
    oc = out.shape[-1]
    return out.reshape(*batch, lon, lat, oc).permute(*lead, nb + 2, nb, nb + 1).to(x.dtype)
