"""Column MLPs on sm_100a: BF16 tcgen05 GEMMs with fused epilogues.

Forward per layer: ``H = act(X Wᵀ + b)`` in one GEMM (bias, activation and
the saved pre-activation written by the epilogue).  Backward per layer:
weight gradient ``dW += dYᵀ X`` (split-K, fp32 atomics), bias gradient as a
column sum, and data gradient ``dX = dY W`` with the previous layer's
activation derivative fused into the epilogue.  Master weights stay fp32;
BF16 copies are refreshed when a parameter's version changes.
"""

from __future__ import annotations

import weakref

import torch
import torch.nn as nn

from tornado_gcm_b200.ops import _ext

ACT_CODES = {"none": 0, "relu": 1, "gelu": 2, "gelu_tanh": 3, "silu": 4, "tanh": 5}


def _pad8(n: int) -> int:
    return (n + 7) // 8 * 8


def supports(x: torch.Tensor, layers) -> bool:
    if not x.is_cuda or not _ext.available():
        return False
    for lyr in layers:
        if not isinstance(lyr, nn.Linear) or lyr.weight.dtype not in (torch.float32, torch.bfloat16):
            return False
    return True


class _WeightCache:
    """Persistent BF16 zero-padded copies of Linear weights.

    A copy is refreshed on the first use after :func:`begin_step` (the
    trainer calls it once per optimizer step, also inside CUDA-graph
    capture so the refresh is part of the replayed graph) or when the
    master weight's version counter changed.
    """

    def __init__(self):
        self.store = {}
        self.token = 0

    def get(self, lin: nn.Linear):
        w = lin.weight
        key = id(lin)
        ver = (w._version, w.data_ptr(), str(w.device))
        ent = self.store.get(key)
        if ent is not None and ent[3]() is not lin:
            ent = None  # the id belonged to a module that no longer exists
        if ent is not None and ent[0] == ver and ent[1] == self.token:
            return ent[2]
        O, K = w.shape
        if ent is None or ent[2].device != w.device or ent[2].shape != (_pad8(O), _pad8(K)):
            buf = torch.zeros(_pad8(O), _pad8(K), dtype=torch.bfloat16, device=w.device)
        else:
            buf = ent[2]
        buf[:O, :K].copy_(w.detach())
        self.store[key] = (ver, self.token, buf, weakref.ref(lin))
        return buf


_CACHE = _WeightCache()


class _BiasCache:
    """fp32 copies of Linear biases zero-padded to the padded output width (refreshed per step)."""

    def __init__(self):
        self.store = {}

    def get(self, lin: nn.Linear, width: int):
        b = lin.bias
        key = id(lin)
        ver = (b._version, b.data_ptr(), str(b.device))
        ent = self.store.get(key)
        if ent is not None and (ent[3]() is not lin or ent[2].shape[0] != width or ent[2].device != b.device):
            ent = None
        if ent is not None and ent[0] == ver and ent[1] == _CACHE.token:
            return ent[2]
        buf = ent[2] if ent is not None else torch.zeros(width, dtype=torch.float32, device=b.device)
        buf[: b.shape[0]].copy_(b.detach())
        self.store[key] = (ver, _CACHE.token, buf, weakref.ref(lin))
        return buf


_BIAS = _BiasCache()


def begin_step() -> None:
    """Mark a new optimizer step: BF16 weight copies refresh on next use."""
    _CACHE.token += 1


# ── in-place gradient accumulation ─────────────────────────────────────────
# A column network is applied once per physics step, i.e. dozens of times per
# training step.  Returning a fresh weight gradient for every use makes
# autograd add it into ``.grad`` (one fill, one copy and one add per use and
# parameter).  With in-place accumulation on, the weight-gradient GEMM adds
# straight into ``weight.grad`` (its epilogue reads the destination; split-K
# partial tiles are reduced there with atomics) and the bias gradient's column
# sum adds into ``bias.grad``.  Layers whose padded shape differs from the
# parameter's (feature counts not a multiple of 8) accumulate into a padded
# fp32 buffer that is added into ``.grad`` once, at the end of the backward
# pass (an autograd engine callback).  Callers must zero the gradients before
# each backward pass (``GCMTrainer`` does); the mode is off by default because
# ``torch.autograd.grad`` callers expect gradients returned, not accumulated.
_ACCUMULATE = {"on": False, "queued": False}
_PADDED_ACC: dict = {}   # id(lin) -> (weakref(lin), fp32 (Op, Kp) buffer)
_PENDING: dict = {}      # id(lin) -> lin, layers with padded gradients to flush


def set_fused_grad_accumulation(enabled: bool) -> None:
    """Accumulate weight and bias gradients in place (see above)."""
    _ACCUMULATE["on"] = bool(enabled)


def fused_grad_accumulation() -> bool:
    return _ACCUMULATE["on"]


def _grad_of(p: torch.Tensor) -> torch.Tensor:
    if p.grad is None:
        p.grad = torch.zeros_like(p)
    return p.grad


def _padded_acc(lin: nn.Linear, shape) -> torch.Tensor:
    ent = _PADDED_ACC.get(id(lin))
    if ent is None or ent[0]() is not lin or tuple(ent[1].shape) != tuple(shape):
        buf = torch.zeros(shape, dtype=torch.float32, device=lin.weight.device)
        ent = (weakref.ref(lin), buf)
        _PADDED_ACC[id(lin)] = ent
    return ent[1]


def _flush_padded() -> None:
    _ACCUMULATE["queued"] = False
    for key, lin in list(_PENDING.items()):
        acc = _PADDED_ACC[key][1]
        O, K = lin.weight.shape
        _grad_of(lin.weight).add_(acc[:O, :K])
        acc.zero_()
    _PENDING.clear()


def _queue_flush() -> None:
    if not _ACCUMULATE["queued"]:
        torch.autograd.Variable._execution_engine.queue_callback(_flush_padded)
        _ACCUMULATE["queued"] = True


def _accumulate_layer_grads(ops, lin: nn.Linear, dy, x, wshape, err) -> None:
    """Weight and bias gradients of one use of ``lin`` added in place."""
    O, K = lin.weight.shape
    w = lin.weight
    if w.requires_grad:
        g = _grad_of(w)
        if (tuple(wshape) == (O, K) and g.dtype == torch.float32 and g.is_contiguous()
                and g.data_ptr() % 16 == 0):
            ops.linear_wgrad(dy, x, g, 0, err)
        else:
            ops.linear_wgrad(dy, x, _padded_acc(lin, wshape), 0, err)
            _PENDING[id(lin)] = lin
            _queue_flush()
    if lin.bias is not None and lin.bias.requires_grad:
        gb = _grad_of(lin.bias)
        if gb.dtype == torch.float32 and gb.is_contiguous():
            ops.colsum_bf16_acc(dy, O, gb)
        else:
            gb.add_(ops.colsum_bf16(dy, O).to(gb.dtype))


class MlpFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2d, acts, last_bf16, layers, *params):
        ops = _ext.require("column MLP")
        err = _ext.error_flag(x2d.device)
        T, K0 = x2d.shape
        if x2d.dtype == torch.bfloat16 and K0 % 8 == 0 and x2d.is_contiguous():
            h = x2d  # already BF16 rows of the padded width (token rows)
        else:
            h = torch.zeros(T, _pad8(K0), dtype=torch.bfloat16, device=x2d.device)
            h[:, :K0] = x2d
        hs, zs, ws = [h], [], []
        n = len(layers)
        for i, lin in enumerate(layers):
            wp = _CACHE.get(lin)
            ws.append(wp)
            Op = wp.shape[0]
            bias = _BIAS.get(lin, Op) if lin.bias is not None else None
            last = i == n - 1
            out_dt = torch.bfloat16 if (not last or last_bf16) else torch.float32
            out = _ext.empty(T, Op, dtype=out_dt, device=x2d.device)
            code = ACT_CODES[acts[i]]
            aux = _ext.empty(T, Op, dtype=torch.bfloat16, device=x2d.device) if (code and not last) else None
            ops.linear_fwd(hs[-1], wp, bias, code, out, aux, err)
            zs.append(aux)
            hs.append(out)
        ctx.acts, ctx.layers, ctx.K0, ctx.x_dtype = acts, layers, K0, x2d.dtype
        ctx.save_for_backward(*(hs[:-1] + [z if z is not None else torch.empty(0) for z in zs] + ws))
        ctx.n = n
        O_last = layers[-1].weight.shape[0]
        return hs[-1][:, :O_last]

    @staticmethod
    def backward(ctx, g):
        ops = _ext.require("column MLP backward")
        n = ctx.n
        saved = ctx.saved_tensors
        hs, zs, ws = saved[:n], saved[n:2 * n], saved[2 * n:]
        err = _ext.error_flag(g.device)
        T = g.shape[0]
        O_last = ctx.layers[-1].weight.shape[0]
        Op_last = ws[-1].shape[0]
        full = getattr(g, "_tgcm_zero_padded", None)
        if (full is not None and full.dtype == torch.bfloat16 and tuple(full.shape) == (T, Op_last)
                and full.is_contiguous() and full.data_ptr() == g.data_ptr()):
            dy = full  # zero-padded BF16 rows written by the consumer's adjoint
        else:
            dy = torch.zeros(T, Op_last, dtype=torch.bfloat16, device=g.device)
            dy[:, :O_last] = g
        grads = []
        dx_out = None
        in_place = _ACCUMULATE["on"]
        for i in range(n - 1, -1, -1):
            lin = ctx.layers[i]
            wp = ws[i]
            if in_place:
                _accumulate_layer_grads(ops, lin, dy, hs[i], wp.shape, err)
                grads.append((None, None))
            else:
                dw = torch.zeros(wp.shape, dtype=torch.float32, device=g.device)
                ops.linear_wgrad(dy, hs[i], dw, 0, err)
                O, K = lin.weight.shape
                gb = ops.colsum_bf16(dy, O) if lin.bias is not None else None
                grads.append((dw[:O, :K].to(lin.weight.dtype), gb))
            if i > 0:
                prev = zs[i - 1]
                code = ACT_CODES[ctx.acts[i - 1]]
                dprev = _ext.empty(T, wp.shape[1], dtype=torch.bfloat16, device=g.device)
                ops.linear_dgrad(dy, wp, dprev, prev if prev.numel() else None, code, err)
                dy = dprev
            else:
                dx_dt = torch.bfloat16 if ctx.x_dtype == torch.bfloat16 else torch.float32
                dx = _ext.empty(T, wp.shape[1], dtype=dx_dt, device=g.device)
                ops.linear_dgrad(dy, wp, dx, None, 0, err)
                dx_out = dx[:, : ctx.K0] if ctx.K0 < dx.shape[1] else dx
                if dx_out.dtype != ctx.x_dtype:
                    dx_out = dx_out.to(ctx.x_dtype)
        grads.reverse()
        flat = []
        for lin, (gw, gb) in zip(ctx.layers, grads):
            flat.append(gw)
            if lin.bias is not None:
                flat.append(gb)
        return (dx_out, None, None, None) + tuple(flat)


def mlp_forward(x: torch.Tensor, layers, acts, last_bf16: bool = False) -> torch.Tensor:
    """The network on the last axis; ``last_bf16`` makes the final layer write BF16 (Z3 output)."""
    lead = x.shape[:-1]
    params = []
    for lin in layers:
        params.append(lin.weight)
        if lin.bias is not None:
            params.append(lin.bias)
    out = MlpFn.apply(x.reshape(-1, x.shape[-1]), tuple(acts), bool(last_bf16), tuple(layers), *params)
    return out.reshape(*lead, out.shape[-1])
