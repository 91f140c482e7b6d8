"""Tensor codecs for mixed-precision storage — reference ``precision/storage/codec.py:23-221``.

* :class:`ExactCodec` — lossless: the tensor's bytes (optionally in a wider
  dtype) plus a general-purpose compressor;
* :class:`LossyCodec` — quantise to BF16/FP16 (on the tensor's device, so a
  GPU tensor crosses PCIe at half size) and compress; BF16 is stored as its
  16-bit pattern.

Compressors: ``"zstd"`` and ``"lz4"`` when their Python packages are
importable, else the standard library's ``"zlib"`` (deflate) and ``"lzma"``;
``"none"`` stores raw bytes.  The compressor actually used is recorded in
the encoded record, so files remain readable wherever that compressor is.
"""

from __future__ import annotations

import dataclasses
import logging
import lzma
import zlib
from typing import Optional

import numpy as np
import torch

logger = logging.getLogger(__name__)


def _resolve(compressor: str) -> str:
    if compressor == "zstd":
        try:
            import zstandard  # noqa: F401

            return "zstd"
        except ImportError:
            return "zlib"
    if compressor == "lz4":
        try:
            import lz4.frame  # noqa: F401

            return "lz4"
        except ImportError:
            return "zlib"
    if compressor in ("zlib", "lzma", "none"):
        return compressor
    raise ValueError(f"unknown compressor {compressor!r}")


def _compress(data: bytes, compressor: str, level: int) -> bytes:
    if compressor == "none":
        return data
    if compressor == "zlib":
        return zlib.compress(data, max(1, min(9, level)))
    if compressor == "lzma":
        return lzma.compress(data, preset=max(0, min(9, level)))
    if compressor == "zstd":
        import zstandard

        return zstandard.ZstdCompressor(level=level).compress(data)
    if compressor == "lz4":
        import lz4.frame

        return lz4.frame.compress(data, compression_level=level)
    raise ValueError(f"unknown compressor {compressor!r}")


def _decompress(data: bytes, compressor: str) -> bytes:
    if compressor == "none":
        return data
    if compressor == "zlib":
        return zlib.decompress(data)
    if compressor == "lzma":
        return lzma.decompress(data)
    if compressor == "zstd":
        import zstandard

        return zstandard.ZstdDecompressor().decompress(data)
    if compressor == "lz4":
        import lz4.frame

        return lz4.frame.decompress(data)
    raise ValueError(f"unknown compressor {compressor!r}")


@dataclasses.dataclass
class _EncodedTensor:
    data: bytes
    shape: tuple
    dtype_name: str
    original_dtype_name: str
    compressor: str


def _to_host_bytes(t: torch.Tensor) -> tuple[bytes, str]:
    t = t.detach()
    if t.dtype == torch.bfloat16:
        arr = t.view(torch.int16).cpu().numpy()
        return arr.tobytes(), "bfloat16"
    arr = t.cpu().numpy()
    return arr.tobytes(), str(arr.dtype)


def _from_bytes(raw: bytes, dtype_name: str, shape) -> torch.Tensor:
    if dtype_name in ("bfloat16", "int16-bf16"):
        arr = np.frombuffer(raw, dtype=np.int16).reshape(shape)
        return torch.from_numpy(arr.copy()).view(torch.bfloat16)
    arr = np.frombuffer(raw, dtype=np.dtype(dtype_name)).reshape(shape)
    return torch.from_numpy(arr.copy())


class ExactCodec:
    def __init__(self, compressor: str = "zstd", compression_level: int = 3) -> None:
        self._compressor = _resolve(compressor)
        self._level = compression_level

    def encode(self, tensor: torch.Tensor, target_dtype: Optional[torch.dtype] = None) -> _EncodedTensor:
        orig = str(tensor.dtype)
        if target_dtype is not None:
            if torch.finfo(target_dtype).bits < torch.finfo(tensor.dtype).bits and tensor.is_floating_point():
                raise ValueError(f"exact storage cannot narrow {tensor.dtype} to {target_dtype}")
            tensor = tensor.to(target_dtype)
        raw, dname = _to_host_bytes(tensor)
        return _EncodedTensor(_compress(raw, self._compressor, self._level), tuple(tensor.shape), dname, orig,
                              self._compressor)

    def decode(self, encoded: _EncodedTensor) -> torch.Tensor:
        return _from_bytes(_decompress(encoded.data, encoded.compressor), encoded.dtype_name, encoded.shape)


class LossyCodec:
    def __init__(self, target_dtype: torch.dtype = torch.bfloat16, compressor: str = "zstd",
                 compression_level: int = 3, error_bound: float = 1e-2) -> None:
        self._target_dtype = target_dtype
        self._compressor = _resolve(compressor)
        self._level = compression_level
        self._error_bound = error_bound
        self.last_max_rel_error: Optional[float] = None

    def encode(self, tensor: torch.Tensor, verify: bool = True) -> _EncodedTensor:
        q = tensor.detach().to(self._target_dtype)  # quantise where the data lives
        if verify and tensor.numel() > 0:
            err = ((tensor.detach() - q.to(tensor.dtype)).abs() / tensor.detach().abs().clamp(min=1e-12)).max()
            self.last_max_rel_error = float(err)
            if self.last_max_rel_error > self._error_bound:
                logger.warning("LossyCodec: max relative error %.3e exceeds bound %.3e",
                               self.last_max_rel_error, self._error_bound)
        raw, dname = _to_host_bytes(q)
        if q.dtype == torch.bfloat16:
            dname = "int16"  # BF16 bit patterns under the record name the reference's files use
        return _EncodedTensor(_compress(raw, self._compressor, self._level), tuple(tensor.shape), dname,
                              str(tensor.dtype), self._compressor)

    def decode(self, encoded: _EncodedTensor, restore_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        t = _from_bytes(_decompress(encoded.data, encoded.compressor), encoded.dtype_name, encoded.shape)
        if encoded.dtype_name == "int16" and self._target_dtype == torch.bfloat16:
            t = t.view(torch.bfloat16)
        return t.to(restore_dtype) if restore_dtype is not None else t
