"""Streaming feature normalisation — reference ``neural/normalizations.py:15-61``."""

from __future__ import annotations

import torch
import torch.nn as nn


class StreamNorm(nn.Module):
    """Normalise the last axis with exponential-moving-average mean / variance.

    Statistics update in training mode only (``x`` is detached for them) and
    are frozen in eval mode; :meth:`unnormalize` inverts the map.
    """

    def __init__(self, num_features: int, momentum: float = 0.01, eps: float = 1e-5):
        super().__init__()
        self.num_features = num_features
        self.momentum = momentum
        self.eps = eps
        self.register_buffer("running_mean", torch.zeros(num_features))
        self.register_buffer("running_var", torch.ones(num_features))
        self.register_buffer("num_batches_tracked", torch.tensor(0, dtype=torch.long))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.training:
            with torch.no_grad():
                flat = x.detach().reshape(-1, x.shape[-1]).to(self.running_mean.dtype)
                var, mean = torch.var_mean(flat, dim=0, unbiased=False)
                self.running_mean.lerp_(mean, self.momentum)
                self.running_var.lerp_(var, self.momentum)
                self.num_batches_tracked += 1
        return (x - self.running_mean.to(x.dtype)) * torch.rsqrt(self.running_var + self.eps).to(x.dtype)

    def unnormalize(self, x: torch.Tensor) -> torch.Tensor:
        return x * torch.sqrt(self.running_var + self.eps).to(x.dtype) + self.running_mean.to(x.dtype)
