"""Split-precision spherical-harmonic transform — reference
``precision/sparse/adaptive_sparse.py:22-170``.

The Legendre basis is split at ``cutoff_l``: the low-order block is
contracted with FP64 accumulation, the high-order block (BF16 coefficients)
with FP32 — both as plain library GEMMs (``torch.einsum``), which on a GPU
run on cuBLAS.
"""

from __future__ import annotations

import torch

from tornado_gcm_b200.precision.sda import SparseConfig
from tornado_gcm_b200.precision.sparse.spectral_sparse import MixedPrecisionSparse


class SparseSpectralTransform:
    def __init__(self, legendre_basis, config: SparseConfig, fourier_basis=None):
        p = torch.as_tensor(legendre_basis, dtype=torch.float64)
        L = p.shape[2]
        self.cutoff_l = int(config.high_order_cutoff * L)
        self.config = config
        self.P_low = p[:, :, :self.cutoff_l].clone()
        self.P_high = p[:, :, self.cutoff_l:].clone()
        self.fourier_basis = None if fourier_basis is None else torch.as_tensor(fourier_basis)
        self._dev: dict = {}

    def _on(self, device):
        key = str(device)
        d = self._dev.get(key)
        if d is None:
            d = (self.P_low.to(device), self.P_high.to(device, torch.float32))
            self._dev[key] = d
        return d

    def inverse_legendre(self, sparse_coeff: MixedPrecisionSparse) -> torch.Tensor:
        lo, hi = self._on(sparse_coeff.device)
        y = torch.einsum("mjl,...ml->...mj", lo, sparse_coeff.low_block().double())
        y = y + torch.einsum("mjl,...ml->...mj", hi, sparse_coeff.high_block().float()).double()
        return y.float()

    def forward_legendre(self, x: torch.Tensor) -> MixedPrecisionSparse:
        lo, hi = self._on(x.device)
        low = torch.einsum("mjl,...mj->...ml", lo, x.double()).float()
        high = torch.einsum("mjl,...mj->...ml", hi, x.float())
        return MixedPrecisionSparse.from_blocks(low, high, self.config.high_order_dtype)

    def inverse_transform(self, sparse_coeff: MixedPrecisionSparse) -> torch.Tensor:
        mid = self.inverse_legendre(sparse_coeff)
        if self.fourier_basis is None:
            return mid
        return torch.einsum("im,...mj->...ij", self.fourier_basis.to(mid.device, mid.dtype), mid)

    def forward_transform(self, x: torch.Tensor) -> MixedPrecisionSparse:
        mid = x if self.fourier_basis is None else torch.einsum(
            "im,...ij->...mj", self.fourier_basis.to(x.device, x.dtype), x)
        return self.forward_legendre(mid)

    @property
    def memory_savings_estimate(self) -> dict:
        M, J, Ll = self.P_low.shape
        Lh = self.P_high.shape[2]
        dense = M * (Ll + Lh) * 4
        mixed = M * Ll * 4 + M * Lh * 2
        return {"dense_fp32_bytes_per_field": dense, "mixed_bytes_per_field": mixed,
                "savings_fraction": 1.0 - mixed / dense, "cutoff_l": self.cutoff_l, "L_total": Ll + Lh}
