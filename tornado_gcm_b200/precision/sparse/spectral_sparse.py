"""Compact storage of spectral (modal) states.

Behaviour parity: reference ``precision/sparse/spectral_sparse.py:22-231``
(modes ``structural``, ``adaptive`` and ``mixed``; ``SpectralSparseState``
built from a state dict and turned back into dense tensors).  The reference
keeps every mode as dense ``(..., M, L)`` tensors with zeros written in, so
its "sparse" states take as much memory as the dense ones.  Here the
storage is packed:

* The valid coefficients ``|m| ≤ l`` of a ``(2M-1, L)`` modal array are
  stored as one vector in *l-major* order (all rows of ``l = 0``, then
  ``l = 1``, …) — :class:`TriangleLayout`.  Triangular truncation leaves
  about half of the rectangle unused, so ``structural`` halves the bytes.
* ``mixed`` splits that vector at the first entry with ``l ≥ cutoff``
  (one split point thanks to the l-major order): the low-l part is kept in
  FP32, the high-l part in BF16 (or the configured dtype).
* ``adaptive`` keeps only the packed entries with ``|x| ≥ threshold`` as
  (int32 position, value) pairs, and falls back to the packed triangle for a
  field where that would not save memory.

Storage only: none of these carry autograd.
"""

from __future__ import annotations

from typing import Optional

import torch

from tornado_gcm_b200.precision.sda import SparseConfig

__all__ = ["MixedPrecisionSparse", "PackedTriangle", "SparseConfig", "SpectralSparseState", "ThresholdPacked",
           "TriangleLayout"]


class TriangleLayout:
    """Packed l-major order of the valid entries of an ``(M2, L)`` modal array.

    Row ``r`` of the modal layout carries ``|m| = (r + 1) // 2`` (rows ordered
    ``m = 0, +1, -1, +2, -2, …``).  ``index[k]`` is the flat ``r * L + l``
    offset of packed entry ``k``; ``l_offsets[l]`` is the packed position of
    the first entry of total wavenumber ``l`` (``l_offsets[L]`` = count).
    """

    _cache: dict = {}

    def __init__(self, M2: int, L: int, device: torch.device | str = "cpu"):
        self.M2, self.L = int(M2), int(L)
        mabs = (torch.arange(self.M2) + 1) // 2
        per_l = torch.clamp(torch.arange(self.L) * 2 + 1, max=self.M2)  # rows with |m| <= l
        offs = torch.zeros(self.L + 1, dtype=torch.int64)
        offs[1:] = torch.cumsum(per_l, 0)
        rows = torch.cat([torch.nonzero(mabs <= l).flatten() for l in range(self.L)])
        ls = torch.repeat_interleave(torch.arange(self.L), per_l)
        self.index = (rows * self.L + ls).to(device)
        self.l_offsets = offs
        self.count = int(offs[-1])

    @classmethod
    def get(cls, M2: int, L: int, device) -> "TriangleLayout":
        key = (int(M2), int(L), str(device))
        lay = cls._cache.get(key)
        if lay is None:
            lay = cls(M2, L, device)
            cls._cache[key] = lay
        return lay

    def split(self, cutoff_l: int) -> int:
        """Packed position of the first entry with ``l >= cutoff_l``."""
        return int(self.l_offsets[max(0, min(int(cutoff_l), self.L))])

    def pack(self, x: torch.Tensor) -> torch.Tensor:
        return x.reshape(*x.shape[:-2], self.M2 * self.L).index_select(-1, self.index)

    def unpack(self, v: torch.Tensor, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        out = torch.zeros(*v.shape[:-1], self.M2 * self.L, dtype=dtype, device=v.device)
        out.index_copy_(-1, self.index, v.to(dtype))
        return out.reshape(*v.shape[:-1], self.M2, self.L)


def _nbytes(t: torch.Tensor) -> int:
    return t.numel() * t.element_size()


class PackedTriangle:
    """``structural`` mode: the valid coefficients only, in the state's dtype."""

    def __init__(self, values: torch.Tensor, modal_shape: tuple, dtype: torch.dtype):
        self.values, self.modal_shape, self.dtype = values, tuple(modal_shape), dtype

    @classmethod
    def from_dense(cls, x: torch.Tensor) -> "PackedTriangle":
        lay = TriangleLayout.get(*x.shape[-2:], x.device)
        return cls(lay.pack(x), tuple(x.shape[-2:]), x.dtype)

    def to_dense(self) -> torch.Tensor:
        return TriangleLayout.get(*self.modal_shape, self.values.device).unpack(self.values, self.dtype)

    def memory_bytes(self) -> int:
        return _nbytes(self.values)

    def dense_memory_bytes(self) -> int:
        return self.values[..., :1].numel() * self.modal_shape[0] * self.modal_shape[1] * 4


class ThresholdPacked:
    """``adaptive`` mode: packed entries with ``|x| >= threshold`` as (position, value) pairs."""

    def __init__(self, positions: torch.Tensor, values: torch.Tensor, lead: tuple, modal_shape: tuple):
        self.positions, self.values, self.lead, self.modal_shape = positions, values, tuple(lead), tuple(modal_shape)

    @classmethod
    def from_dense(cls, x: torch.Tensor, threshold: float):
        lay = TriangleLayout.get(*x.shape[-2:], x.device)
        packed = lay.pack(x).reshape(-1)
        keep = torch.nonzero(packed.abs() >= threshold).flatten()
        if keep.numel() * 8 >= packed.numel() * 4:  # pairs would not beat the packed triangle
            return PackedTriangle(packed.reshape(*x.shape[:-2], lay.count), tuple(x.shape[-2:]), x.dtype)
        return cls(keep.to(torch.int32), packed[keep].to(torch.float32), tuple(x.shape[:-2]), tuple(x.shape[-2:]))

    def to_dense(self) -> torch.Tensor:
        lay = TriangleLayout.get(*self.modal_shape, self.values.device)
        n = 1
        for s in self.lead:
            n *= s
        packed = torch.zeros(n * lay.count, dtype=torch.float32, device=self.values.device)
        packed[self.positions.long()] = self.values
        return lay.unpack(packed.reshape(*self.lead, lay.count))

    def memory_bytes(self) -> int:
        return _nbytes(self.positions) + _nbytes(self.values)

    def dense_memory_bytes(self) -> int:
        n = 1
        for s in self.lead:
            n *= s
        return n * self.modal_shape[0] * self.modal_shape[1] * 4


class MixedPrecisionSparse:
    """``mixed`` mode: packed triangle split at ``cutoff_l`` into FP32 low-l and low-precision high-l parts.

    ``low`` / ``high`` are the packed parts; :meth:`low_block` /
    :meth:`high_block` give them back as dense ``(..., M2, cutoff)`` /
    ``(..., M2, L - cutoff)`` blocks for the split-precision transform.
    """

    def __init__(self, low: torch.Tensor, high: torch.Tensor, cutoff_l: int, modal_shape: tuple):
        self.low, self.high = low, high
        self.cutoff_l = int(cutoff_l)
        self.modal_shape = tuple(modal_shape)

    @classmethod
    def from_dense(cls, x: torch.Tensor, cutoff_l: int, high_dtype: torch.dtype = torch.bfloat16):
        lay = TriangleLayout.get(*x.shape[-2:], x.device)
        v = lay.pack(x)
        s = lay.split(cutoff_l)
        return cls(v[..., :s].to(torch.float32), v[..., s:].to(high_dtype), cutoff_l, tuple(x.shape[-2:]))

    @classmethod
    def from_blocks(cls, low_block: torch.Tensor, high_block: torch.Tensor,
                    high_dtype: torch.dtype = torch.bfloat16) -> "MixedPrecisionSparse":
        """From dense ``(..., M2, cutoff)`` and ``(..., M2, L - cutoff)`` blocks."""
        cut = low_block.shape[-1]
        full = torch.cat([low_block.to(torch.float32), high_block.to(torch.float32)], dim=-1)
        return cls.from_dense(full, cut, high_dtype)

    def to_dense(self) -> torch.Tensor:
        lay = TriangleLayout.get(*self.modal_shape, self.low.device)
        return lay.unpack(torch.cat([self.low, self.high.to(torch.float32)], dim=-1))

    def low_block(self) -> torch.Tensor:
        return self.to_dense()[..., :self.cutoff_l]

    def high_block(self) -> torch.Tensor:
        return self.to_dense()[..., self.cutoff_l:]

    @property
    def shape(self) -> tuple:
        return (*self.low.shape[:-1], *self.modal_shape)

    @property
    def device(self) -> torch.device:
        return self.low.device

    def memory_bytes(self) -> int:
        return _nbytes(self.low) + _nbytes(self.high)

    def dense_memory_bytes(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n * 4

    @property
    def memory_savings(self) -> float:
        d = self.dense_memory_bytes()
        return 0.0 if d == 0 else 1.0 - self.memory_bytes() / d


_PACKED = (PackedTriangle, ThresholdPacked, MixedPrecisionSparse)


class SpectralSparseState:
    """A state dict whose modal fields are held packed (see the module docstring)."""

    def __init__(self, fields: dict, config: SparseConfig, modal_shape: Optional[tuple] = None):
        self.fields = fields
        self.config = config
        self.modal_shape = modal_shape

    @staticmethod
    def _encode(t: torch.Tensor, config: SparseConfig):
        mode = config.mode
        if mode == "structural":
            return PackedTriangle.from_dense(t)
        if mode == "adaptive":
            return ThresholdPacked.from_dense(t, float(config.adaptive_threshold))
        if mode == "mixed":
            return MixedPrecisionSparse.from_dense(t, int(config.high_order_cutoff * t.shape[-1]),
                                                   config.high_order_dtype)
        return t

    @classmethod
    def from_state_dict(cls, state_dict: dict, config: SparseConfig) -> "SpectralSparseState":
        fields, modal_shape = {}, None
        for name, t in state_dict.items():
            if torch.is_tensor(t) and t.is_floating_point() and t.dim() >= 2:
                modal_shape = modal_shape or tuple(t.shape[-2:])
                fields[name] = cls._encode(t, config)
            else:
                fields[name] = t
        return cls(fields, config, modal_shape)

    def to_dense_dict(self) -> dict:
        out = {}
        for k, v in self.fields.items():
            if isinstance(v, _PACKED):
                out[k] = v.to_dense().to(torch.float32)
            elif torch.is_tensor(v) and v.is_floating_point():
                out[k] = v.to(torch.float32)
            else:
                out[k] = v
        return out

    @property
    def memory_bytes(self) -> int:
        return sum(v.memory_bytes() if isinstance(v, _PACKED) else _nbytes(v)
                   for v in self.fields.values() if isinstance(v, _PACKED) or torch.is_tensor(v))

    @property
    def dense_memory_bytes(self) -> int:
        return sum(v.dense_memory_bytes() if isinstance(v, _PACKED) else v.numel() * 4
                   for v in self.fields.values() if isinstance(v, _PACKED) or torch.is_tensor(v))

    @property
    def memory_savings(self) -> float:
        d = self.dense_memory_bytes
        return 0.0 if d == 0 else 1.0 - self.memory_bytes / d
