"""Sparse / split-precision spectral state storage — reference
``precision/sparse/spectral_sparse.py:22-231``.

* ``structural``: coefficients outside ``|m| ≤ l`` zeroed;
* ``adaptive``: additionally coefficients below a threshold;
* ``mixed``: ``l < cutoff`` kept FP32, ``l ≥ cutoff`` stored BF16.

Inference/storage only: the representations carry no autograd.
"""

from __future__ import annotations

from typing import Optional

import torch

from tornado_gcm_b200.precision.sda import SparseConfig
from tornado_gcm_b200.precision.sparse.ops import triangular_mask

__all__ = ["MixedPrecisionSparse", "SparseConfig", "SpectralSparseState"]


class MixedPrecisionSparse:
    """``(..., M, L)`` split at ``cutoff_l``: FP32 low block + BF16 (default) high block."""

    def __init__(self, low_order: torch.Tensor, high_order: torch.Tensor, cutoff_l: int):
        self.low = low_order
        self.high = high_order
        self.cutoff_l = int(cutoff_l)

    @classmethod
    def from_dense(cls, x: torch.Tensor, cutoff_l: int, high_dtype: torch.dtype = torch.bfloat16):
        return cls(x[..., :cutoff_l].to(torch.float32), x[..., cutoff_l:].to(high_dtype), cutoff_l)

    def to_dense(self) -> torch.Tensor:
        return torch.cat([self.low, self.high.to(torch.float32)], dim=-1)

    @property
    def shape(self) -> tuple:
        return (*self.low.shape[:-1], self.low.shape[-1] + self.high.shape[-1])

    @property
    def device(self) -> torch.device:
        return self.low.device

    def memory_bytes(self) -> int:
        return self.low.numel() * self.low.element_size() + self.high.numel() * self.high.element_size()

    def dense_memory_bytes(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n * 4

    @property
    def memory_savings(self) -> float:
        d = self.dense_memory_bytes()
        return 0.0 if d == 0 else 1.0 - self.memory_bytes() / d


class SpectralSparseState:
    def __init__(self, fields: dict, config: SparseConfig, modal_shape: Optional[tuple] = None):
        self.fields = fields
        self.config = config
        self.modal_shape = modal_shape

    @classmethod
    def from_state_dict(cls, state_dict: dict, config: SparseConfig) -> "SpectralSparseState":
        fields, modal_shape = {}, None
        for name, t in state_dict.items():
            if not torch.is_tensor(t) or t.dim() < 2:
                fields[name] = t
                continue
            M, L = t.shape[-2:]
            modal_shape = modal_shape or (M, L)
            if config.mode == "structural":
                fields[name] = t * triangular_mask(M, L, t.device)
            elif config.mode == "adaptive":
                fields[name] = t * (triangular_mask(M, L, t.device) & (t.abs() >= config.adaptive_threshold))
            elif config.mode == "mixed":
                fields[name] = MixedPrecisionSparse.from_dense(t, int(config.high_order_cutoff * L),
                                                               config.high_order_dtype)
            else:
                fields[name] = t
        return cls(fields, config, modal_shape)

    def to_dense_dict(self) -> dict:
        out = {}
        for k, v in self.fields.items():
            if isinstance(v, MixedPrecisionSparse):
                out[k] = v.to_dense()
            elif torch.is_tensor(v) and v.is_floating_point():
                out[k] = v.to(torch.float32)
            else:
                out[k] = v
        return out

    @property
    def memory_bytes(self) -> int:
        tot = 0
        for v in self.fields.values():
            if isinstance(v, MixedPrecisionSparse):
                tot += v.memory_bytes()
            elif torch.is_tensor(v):
                tot += v.numel() * v.element_size()
        return tot

    @property
    def dense_memory_bytes(self) -> int:
        tot = 0
        for v in self.fields.values():
            if isinstance(v, MixedPrecisionSparse):
                tot += v.dense_memory_bytes()
            elif torch.is_tensor(v):
                tot += v.numel() * 4
        return tot

    @property
    def memory_savings(self) -> float:
        d = self.dense_memory_bytes
        return 0.0 if d == 0 else 1.0 - self.memory_bytes / d
