"""Neural building blocks (Z3) — reference ``neural/standard_layers.py:24-332``.

Same module names, constructor signatures and parameter names
(``layers.{i}.weight/bias``) as the reference so ``.pt`` state dicts load
unchanged.  On CUDA the MLP forward/backward runs through the sm_100a BF16
GEMM kernels of :mod:`tornado_gcm_b200.ops.linear` (tcgen05 + TMEM with the
bias and activation fused into the epilogue); elsewhere plain torch.
"""

from __future__ import annotations

import functools
from typing import Callable, Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

gelu_tanh = functools.partial(F.gelu, approximate="tanh")
gelu_tanh.__name__ = "gelu_tanh"


def identity(x):
    return x


_ACTIVATION_NAMES = {}


def _register_activation(fn, name):
    _ACTIVATION_NAMES[id(fn)] = name


for _fn, _name in [(F.relu, "relu"), (torch.relu, "relu"), (F.gelu, "gelu"), (gelu_tanh, "gelu_tanh"),
                   (F.silu, "silu"), (identity, "none"), (torch.tanh, "tanh")]:
    _register_activation(_fn, _name)


def activation_name(fn: Optional[Callable]) -> Optional[str]:
    """Name of a fusable activation, or None if the callable is not known."""
    if fn is None:
        return "none"
    name = _ACTIVATION_NAMES.get(id(fn))
    if name is not None:
        return name
    if isinstance(fn, functools.partial) and fn.func is F.gelu:
        return "gelu_tanh" if fn.keywords.get("approximate") == "tanh" else "gelu"
    if isinstance(fn, nn.GELU):
        return "gelu_tanh" if fn.approximate == "tanh" else "gelu"
    if isinstance(fn, nn.ReLU):
        return "relu"
    if isinstance(fn, nn.SiLU):
        return "silu"
    return None


def apply_activation(name: str, x: torch.Tensor) -> torch.Tensor:
    if name == "relu":
        return F.relu(x)
    if name == "gelu":
        return F.gelu(x)
    if name == "gelu_tanh":
        return F.gelu(x, approximate="tanh")
    if name == "silu":
        return F.silu(x)
    if name == "tanh":
        return torch.tanh(x)
    return x


def lecun_normal_(weight: torch.Tensor):
    nn.init.kaiming_normal_(weight, mode="fan_in", nonlinearity="linear")


class Mlp(nn.Module):
    """Multi-layer perceptron; activation between layers (and optionally last)."""

    def __init__(self, input_size: int, output_size: int, *, intermediate_sizes: Sequence[int],
                 activation: Callable = F.relu, activate_final: bool = False, use_bias: bool = True):
        super().__init__()
        self.input_size = input_size
        self.output_size = output_size
        self.activation = activation
        self.activate_final = activate_final
        sizes = (input_size,) + tuple(intermediate_sizes) + (output_size,)
        self.layers = nn.ModuleList(nn.Linear(a, b, bias=use_bias) for a, b in zip(sizes[:-1], sizes[1:]))
        self._init_weights()

    def _init_weights(self):
        for layer in self.layers:
            lecun_normal_(layer.weight)
            if layer.bias is not None:
                nn.init.zeros_(layer.bias)

    def layer_activations(self) -> list[Optional[str]]:
        act = activation_name(self.activation)
        n = len(self.layers)
        return [act if (i < n - 1 or self.activate_final) else "none" for i in range(n)]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        acts = self.layer_activations()
        if x.is_cuda and None not in acts:
            from tornado_gcm_b200.ops import linear as linear_ops

            if linear_ops.supports(x, self.layers):
                return linear_ops.mlp_forward(x, self.layers, acts)
        n = len(self.layers)
        for i, layer in enumerate(self.layers):
            x = layer(x)
            if i < n - 1 or self.activate_final:
                x = self.activation(x)
        return x

    @classmethod
    def uniform(cls, input_size: int, output_size: int, *, hidden_size: int, hidden_layers: int,
                activation: Callable = F.gelu, activate_final: bool = False, use_bias: bool = True) -> "Mlp":
        return cls(input_size, output_size, intermediate_sizes=(hidden_size,) * hidden_layers,
                   activation=activation, activate_final=activate_final, use_bias=use_bias)


class MlpUniform(Mlp):
    def __init__(self, input_size: int, output_size: int, *, hidden_size: int, n_hidden_layers: int,
                 activation: Callable = F.gelu, activate_final: bool = False, use_bias: bool = True):
        super().__init__(input_size, output_size, intermediate_sizes=(hidden_size,) * n_hidden_layers,
                         activation=activation, activate_final=activate_final, use_bias=use_bias)


class ConvLevel(nn.Module):
    """1-D convolution along the level axis with 'same' padding."""

    def __init__(self, input_size: int, output_size: int, kernel_size: int = 3, use_bias: bool = True,
                 padding: str = "same", stride: int = 1, dilation: int = 1):
        super().__init__()
        self.conv = nn.Conv1d(input_size, output_size, kernel_size, stride=stride, padding=padding,
                              dilation=dilation, bias=use_bias)
        lecun_normal_(self.conv.weight)
        if self.conv.bias is not None:
            nn.init.zeros_(self.conv.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.conv(x)


class CnnLevel(nn.Module):
    """Stack of ConvLevel layers with activations."""

    def __init__(self, input_size: int, output_size: int, *, channels: Sequence[int] = (), kernel_size: int = 3,
                 activation: Callable = F.gelu, activate_final: bool = False, use_bias: bool = True,
                 kernel_sizes=None, strides=1, dilations=1):
        """``kernel_sizes`` / ``strides`` / ``dilations``: one value for every layer or one per
        layer (the reference's names; ``kernel_sizes`` overrides ``kernel_size``)."""
        super().__init__()
        sizes = (input_size,) + tuple(channels) + (output_size,)
        n = len(sizes) - 1
        per = lambda v: list(v) if isinstance(v, (list, tuple)) else [v] * n  # noqa: E731
        ks, st, dl = per(kernel_size if kernel_sizes is None else kernel_sizes), per(strides), per(dilations)
        if not (len(ks) == len(st) == len(dl) == n):
            raise ValueError(f"per-layer settings must have {n} entries")
        self.layers = nn.ModuleList(ConvLevel(a, b, ks[i], use_bias, stride=st[i], dilation=dl[i])
                                    for i, (a, b) in enumerate(zip(sizes[:-1], sizes[1:])))
        self.activation = activation
        self.activate_final = activate_final

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        n = len(self.layers)
        for i, layer in enumerate(self.layers):
            x = layer(x)
            if i < n - 1 or self.activate_final:
                x = self.activation(x)
        return x


class Epd(nn.Module):
    """Encode-process-decode with residual process blocks."""

    def __init__(self, encode: nn.Module, decode: nn.Module, process_blocks: Sequence[nn.Module],
                 post_encode_activation: Callable | None = None, pre_decode_activation: Callable | None = None,
                 final_activation: Callable | None = None):
        super().__init__()
        self.encode = encode
        self.decode = decode
        self.process_blocks = nn.ModuleList(process_blocks)
        self.post_encode_activation = post_encode_activation
        self.pre_decode_activation = pre_decode_activation
        self.final_activation = final_activation

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = self.encode(x)
        if self.post_encode_activation is not None:
            h = self.post_encode_activation(h)
        for block in self.process_blocks:
            h = h + block(h)
        if self.pre_decode_activation is not None:
            h = self.pre_decode_activation(h)
        out = self.decode(h)
        if self.final_activation is not None:
            out = self.final_activation(out)
        return out

    @classmethod
    def build(cls, input_size: int, output_size: int, *, latent_size: int, num_process_blocks: int,
              hidden_layers: int = 2, hidden_size: int | None = None, activation: Callable = F.gelu) -> "Epd":
        hs = latent_size if hidden_size is None else hidden_size
        mk = lambda i, o: Mlp.uniform(i, o, hidden_size=hs, hidden_layers=hidden_layers, activation=activation)
        return cls(mk(input_size, latent_size), mk(latent_size, output_size),
                   [mk(latent_size, latent_size) for _ in range(num_process_blocks)],
                   post_encode_activation=activation)


class Sequential(nn.Module):
    def __init__(self, layers: Sequence[nn.Module]):
        super().__init__()
        self.layers = nn.ModuleList(layers)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        for layer in self.layers:
            x = layer(x)
        return x


class ConvLonLat(nn.Module):
    """2-D conv on (lon, lat): circular padding in lon, zero padding in lat."""

    def __init__(self, input_size: int | None = None, output_size: int | None = None,
                 kernel_size: tuple[int, int] = (3, 3), dilation: int = 1, use_bias: bool = True,
                 input_channels: int | None = None, output_channels: int | None = None):
        """``input_channels`` / ``output_channels`` are the reference's names for the sizes."""
        super().__init__()
        input_size = input_size if input_size is not None else input_channels
        output_size = output_size if output_size is not None else output_channels
        if input_size is None or output_size is None:
            raise ValueError("ConvLonLat needs input and output channel counts")
        self.kernel_size = tuple(kernel_size)
        self.dilation = dilation
        self.conv = nn.Conv2d(input_size, output_size, self.kernel_size, dilation=dilation, bias=use_bias)
        lecun_normal_(self.conv.weight)
        if self.conv.bias is not None:
            nn.init.zeros_(self.conv.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        kl, kt = self.kernel_size
        pl = self.dilation * (kl - 1) // 2
        pt = self.dilation * (kt - 1) // 2
        squeeze = x.ndim == 3
        if squeeze:
            x = x.unsqueeze(0)
        x = F.pad(x, (0, 0, pl, pl), mode="circular")
        x = F.pad(x, (pt, pt, 0, 0), mode="constant", value=0.0)
        y = self.conv(x)
        return y.squeeze(0) if squeeze else y
