"""Towers: apply per-column networks over the sphere (reference ``neural/towers.py``).

All towers accept arbitrary leading batch dims before the feature axis.
"""

from __future__ import annotations

from typing import Callable, Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from tornado_gcm_b200.neural.standard_layers import ConvLevel, ConvLonLat


def _net_dtype(net: nn.Module, x: torch.Tensor) -> torch.Tensor:
    p = next(net.parameters(), None)
    if p is not None and x.dtype != p.dtype:
        return x.to(p.dtype)
    return x


class ForwardTower(nn.Module):
    """Apply ``neural_net`` on the feature axis, vectorised over all other axes."""

    def __init__(self, neural_net: nn.Module, feature_axis: int = -3, final_activation: Callable | None = None):
        super().__init__()
        self.neural_net = neural_net
        self.feature_axis = feature_axis
        self.final_activation = final_activation

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        fa = self.feature_axis % x.ndim
        xt = torch.movedim(x, fa, -1)
        lead = xt.shape[:-1]
        flat = _net_dtype(self.neural_net, xt.reshape(-1, xt.shape[-1]))
        out = self.neural_net(flat)
        out = torch.movedim(out.reshape(*lead, out.shape[-1]), -1, fa)
        if self.final_activation is not None:
            out = self.final_activation(out)
        return out


class ColumnTower(nn.Module):
    """Flatten (levels, features) per column, apply net, unflatten."""

    def __init__(self, neural_net: nn.Module):
        super().__init__()
        self.neural_net = neural_net

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        *batch, levels, features, lon, lat = x.shape
        xt = x.movedim((-2, -1), (-4, -3)).reshape(*batch, lon * lat, levels * features)
        out = self.neural_net(_net_dtype(self.neural_net, xt))
        of = out.shape[-1] // levels
        return out.reshape(*batch, lon, lat, levels, of).movedim((-4, -3), (-2, -1))


class ColumnTransformerTower(ColumnTower):
    """Column tower whose net takes optional latent / positional inputs."""

    def forward(self, x: torch.Tensor, latents: Optional[torch.Tensor] = None,
                positional_encoding: Optional[torch.Tensor] = None) -> torch.Tensor:
        *batch, levels, features, lon, lat = x.shape
        xt = x.movedim((-2, -1), (-4, -3)).reshape(-1, levels, features)
        kwargs = {}
        if latents is not None:
            kwargs["latents"] = latents
        if positional_encoding is not None:
            kwargs["positional_encoding"] = positional_encoding
        out = self.neural_net(_net_dtype(self.neural_net, xt), **kwargs)
        of = out.shape[-1]
        return out.reshape(*batch, lon, lat, levels, of).movedim((-4, -3), (-2, -1))


class VerticalConvTower(nn.Module):
    """Conv1d stack over levels with lon·lat as the batch axis.

    Input ``(..., channels, levels, lon, lat)`` → ``(..., out_channels, levels, lon, lat)``.
    """

    def __init__(self, input_size: int | None = None, output_size: int | None = None,
                 channels: Sequence[int] = (64, 64, 64, 64), kernel_size: int = 3, activation: Callable = F.relu,
                 activate_final: bool = False, use_bias: bool = True, *, input_channels: int | None = None,
                 output_channels: int | None = None, hidden_channels: Sequence[int] | None = None,
                 checkpoint_tower: bool = False):
        """The reference's names are accepted: ``input_channels``, ``output_channels``,
        ``hidden_channels``; ``checkpoint_tower`` recomputes the tower in backward instead of
        keeping its activations."""
        super().__init__()
        input_size = input_size if input_size is not None else input_channels
        output_size = output_size if output_size is not None else output_channels
        if input_size is None or output_size is None:
            raise ValueError("VerticalConvTower needs input and output channel counts")
        channels = tuple(hidden_channels) if hidden_channels is not None else tuple(channels)
        self.checkpoint_tower = checkpoint_tower
        sizes = (input_size,) + tuple(channels) + (output_size,)
        self.layers = nn.ModuleList(ConvLevel(a, b, kernel_size, use_bias) for a, b in zip(sizes[:-1], sizes[1:]))
        self.activation = activation
        self.activate_final = activate_final

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.checkpoint_tower and self.training and torch.is_grad_enabled():
            from torch.utils.checkpoint import checkpoint

            return checkpoint(self._forward, x, use_reentrant=False)
        return self._forward(x)

    def _forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.is_cuda:
            from tornado_gcm_b200.ops import levelconv

            if levelconv.supports(self, x):
                # level convolutions as tcgen05 GEMMs on (column, level) token rows
                return levelconv.level_conv_tower(self, x)
        *batch, c, levels, lon, lat = x.shape
        xt = x.movedim((-2, -1), (-4, -3)).reshape(-1, c, levels)
        xt = _net_dtype(self, xt)
        n = len(self.layers)
        for i, layer in enumerate(self.layers):
            xt = layer(xt)
            if i < n - 1 or self.activate_final:
                xt = self.activation(xt)
        oc = xt.shape[1]
        return xt.reshape(*batch, lon, lat, oc, levels).movedim((-4, -3), (-2, -1))


class Conv2DTower(nn.Module):
    """Stack of ConvLonLat layers on ``(..., channels, lon, lat)``."""

    def __init__(self, input_size: int | None = None, output_size: int | None = None, *,
                 channels: Sequence[int] | None = None, kernel_size: tuple[int, int] = (3, 3),
                 activation: Callable = F.relu, activate_final: bool = False, use_bias: bool = True,
                 input_channels: int | None = None, output_channels: int | None = None,
                 num_hidden_units: int = 32, num_hidden_layers: int = 2):
        """Hidden widths: ``channels``, else ``num_hidden_layers`` layers of ``num_hidden_units``
        (the reference's parameters); ``input_channels`` / ``output_channels`` name the sizes."""
        super().__init__()
        input_size = input_size if input_size is not None else input_channels
        output_size = output_size if output_size is not None else output_channels
        if input_size is None or output_size is None:
            raise ValueError("Conv2DTower needs input and output channel counts")
        channels = tuple(channels) if channels is not None else (num_hidden_units,) * num_hidden_layers
        sizes = (input_size,) + tuple(channels) + (output_size,)
        self.layers = nn.ModuleList(ConvLonLat(a, b, kernel_size, use_bias=use_bias)
                                    for a, b in zip(sizes[:-1], sizes[1:]))
        self.activation = activation
        self.activate_final = activate_final

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.is_cuda:
            from tornado_gcm_b200.ops import levelconv

            if levelconv.supports_lonlat(self, x):
                # lon-lat convolutions as tcgen05 GEMMs on (batch, lon, lat) token rows
                return levelconv.lonlat_conv_tower(self, x)
        *batch, c, lon, lat = x.shape
        xt = _net_dtype(self, x.reshape(-1, c, lon, lat))
        n = len(self.layers)
        for i, layer in enumerate(self.layers):
            xt = layer(xt)
            if i < n - 1 or self.activate_final:
                xt = self.activation(xt)
        return xt.reshape(*batch, xt.shape[1], lon, lat)
