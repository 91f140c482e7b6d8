"""Per-wavenumber Legendre transforms — reference
``precision/accelerator/triton_sht.py:40-337`` (kernels K1/K2).

``inverse``: ``out[b, m, j] = Σ_l P[m, j, l] · x[b, m, l]``;
``forward``: ``out[b, m, l] = Σ_j P[m, j, l] · x[b, m, j]``.

The sm100 versions run one tcgen05 TF32 grouped GEMM (group = m, TMA-fed
K-major tiles, TMEM accumulator) through the ``bgemm_tf32`` op; the basis is
kept on the device, row-padded to a 16-byte multiple, per (basis, device).
The torch versions accumulate in FP64 (the oracle).
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from tornado_gcm_b200.ops import _ext

_BASIS_CACHE: dict = {}


def _pad4(n: int) -> int:
    return (n + 3) // 4 * 4


def _device_basis(basis, device, transposed: bool) -> torch.Tensor:
    key = (id(basis), tuple(basis.shape), str(device), transposed)
    ent = _BASIS_CACHE.get(key)
    if ent is not None and ent[0] is basis:
        return ent[1]
    b = torch.as_tensor(np.asarray(basis) if not torch.is_tensor(basis) else basis.detach().cpu(),
                        dtype=torch.float64)
    M2, J, L = b.shape
    if transposed:  # (M2, L, Jp)
        out = torch.zeros(M2, L, _pad4(J), dtype=torch.float32)
        out[:, :, :J] = b.permute(0, 2, 1).float()
    else:  # (M2, J, Lp)
        out = torch.zeros(M2, J, _pad4(L), dtype=torch.float32)
        out[:, :, :L] = b.float()
    out = out.to(device)
    _BASIS_CACHE[key] = (basis, out)
    return out


def sht_legendre_inverse_torch(basis, x: torch.Tensor, use_fp64: bool = True) -> torch.Tensor:
    b = torch.as_tensor(basis, device=x.device)
    if use_fp64:
        return torch.einsum("mjl,...ml->...mj", b.double(), x.double()).to(torch.float32)
    return torch.einsum("mjl,...ml->...mj", b.to(x.dtype), x)


def sht_legendre_forward_torch(basis, x: torch.Tensor, use_fp64: bool = True) -> torch.Tensor:
    b = torch.as_tensor(basis, device=x.device)
    if use_fp64:
        return torch.einsum("mjl,...mj->...ml", b.double(), x.double()).to(torch.float32)
    return torch.einsum("mjl,...mj->...ml", b.to(x.dtype), x)


def sht_legendre_inverse_sm100(basis, x: torch.Tensor) -> torch.Tensor:
    ops = _ext.require("Legendre synthesis")
    M2, L = x.shape[-2], x.shape[-1]
    lead = x.shape[:-2]
    P = _device_basis(basis, x.device, False)  # (M2, J, Lp)
    J, Lp = P.shape[1], P.shape[2]
    xp = torch.zeros(int(np.prod(lead)) if lead else 1, M2, Lp, dtype=torch.float32, device=x.device)
    xp[..., :L] = x.reshape(-1, M2, L)
    out = torch.empty(xp.shape[0], M2, J, dtype=torch.float32, device=x.device)
    ops.bgemm_tf32(xp.permute(1, 0, 2), P, out.permute(1, 0, 2), 1.0, _ext.error_flag(x.device))
    return out.reshape(*lead, M2, J)


def sht_legendre_forward_sm100(basis, x: torch.Tensor) -> torch.Tensor:
    ops = _ext.require("Legendre analysis")
    M2, J = x.shape[-2], x.shape[-1]
    lead = x.shape[:-2]
    Pt = _device_basis(basis, x.device, True)  # (M2, L, Jp)
    L, Jp = Pt.shape[1], Pt.shape[2]
    xp = torch.zeros(int(np.prod(lead)) if lead else 1, M2, Jp, dtype=torch.float32, device=x.device)
    xp[..., :J] = x.reshape(-1, M2, J)
    out = torch.empty(xp.shape[0], M2, L, dtype=torch.float32, device=x.device)
    ops.bgemm_tf32(xp.permute(1, 0, 2), Pt, out.permute(1, 0, 2), 1.0, _ext.error_flag(x.device))
    return out.reshape(*lead, M2, L)


def has_sm100() -> bool:
    return torch.cuda.is_available() and _ext.available()


def sht_legendre_inverse(basis, x: torch.Tensor, use_fp64: bool = False, backend: Optional[str] = None) -> torch.Tensor:
    """``backend``: ``"sm100"`` (the TF32 tensor-core kernel), ``"torch"`` or ``None`` (sm100 for
    CUDA tensors).  ``use_fp64`` asks for FP64 accumulation and selects the FP64 einsum (the
    reference's ``use_fp64`` switch; it defaults on there, where the default kernel is FP64)."""
    if not use_fp64 and (backend == "sm100" or (backend is None and x.is_cuda and _ext.available())):
        return sht_legendre_inverse_sm100(basis, x)
    return sht_legendre_inverse_torch(basis, x)  # FP64 accumulation


def sht_legendre_forward(basis, x: torch.Tensor, use_fp64: bool = False, backend: Optional[str] = None) -> torch.Tensor:
    """Analysis counterpart of :func:`sht_legendre_inverse` (same switches)."""
    if not use_fp64 and (backend == "sm100" or (backend is None and x.is_cuda and _ext.available())):
        return sht_legendre_forward_sm100(basis, x)
    return sht_legendre_forward_torch(basis, x)  # FP64 accumulation
