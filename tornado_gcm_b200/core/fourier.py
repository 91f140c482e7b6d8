"""Real Fourier basis along longitude (reference ``core/fourier.py:20-140``).

Column layout of the basis ``F[i, k]`` (``nodes`` × ``2W-1``):
``k=0`` → 1/√(2π); ``k=2j-1`` → cos(j x_i)/√π; ``k=2j`` → sin(j x_i)/√π, with
``x_i = 2πi/nodes``.  Built directly from cos/sin in FP64.
"""

from __future__ import annotations

import numpy as np
import torch


def real_basis(wavenumbers: int, nodes: int) -> np.ndarray:
    if nodes < wavenumbers:
        raise ValueError(
            f"`real_basis` requires nodes >= wavenumbers; got nodes = {nodes} "
            f"and wavenumbers = {wavenumbers}."
        )
    x = 2.0 * np.pi * np.arange(nodes, dtype=np.float64) / nodes
    j = np.arange(1, wavenumbers, dtype=np.float64)
    f = np.empty((nodes, 2 * wavenumbers - 1), dtype=np.float64)
    f[:, 0] = 1.0 / np.sqrt(2.0 * np.pi)
    phase = np.outer(x, j)
    f[:, 1::2] = np.cos(phase) / np.sqrt(np.pi)
    f[:, 2::2] = np.sin(phase) / np.sqrt(np.pi)
    return f


def real_basis_with_zero_imag(wavenumbers: int, nodes: int) -> np.ndarray:
    if nodes < wavenumbers:
        raise ValueError("`real_basis` requires nodes >= wavenumbers")
    base = real_basis(wavenumbers, nodes)
    f = np.zeros((nodes, 2 * wavenumbers), dtype=np.float64)
    f[:, 0] = base[:, 0]
    f[:, 2::2] = base[:, 1::2]
    f[:, 3::2] = base[:, 2::2]
    return f


_DERIV_CACHE: dict = {}


def derivative_index_and_scale(n: int, device=None, dtype=torch.float32):
    """Gather index and signed scale implementing d/dλ on an odd-length axis.

    out[k] = scale[k] * u[src[k]] with out[2j-1] = j u[2j], out[2j] = -j u[2j-1].
    Cached per (n, device, dtype) so repeated calls (and CUDA-graph capture)
    issue no host-to-device copies.
    """
    key = (n, str(device), dtype)
    hit = _DERIV_CACHE.get(key)
    if hit is not None:
        return hit
    k = np.arange(n)
    j = (k + 1) // 2
    src = np.clip(np.where(k % 2 == 1, k + 1, k - 1), 0, n - 1)
    scale = np.where(k % 2 == 1, j, -j).astype(np.float64)
    scale[0] = 0.0
    out = (torch.as_tensor(src, device=device), torch.as_tensor(scale, dtype=dtype, device=device))
    _DERIV_CACHE[key] = out
    return out


def real_basis_derivative(u: torch.Tensor, /, axis: int = -1) -> torch.Tensor:
    """∂/∂λ in the real Fourier basis along ``axis`` (must be negative, odd size)."""
    if axis >= 0:
        raise ValueError("axis must be negative")
    n = u.shape[axis]
    if n % 2 != 1:
        raise ValueError(f"u.shape along axis={axis} must be odd, got {n}")
    src, scale = derivative_index_and_scale(n, u.device, u.dtype)
    shape = [1] * u.ndim
    shape[axis] = n
    return u.index_select(u.ndim + axis, src) * scale.reshape(shape)


def real_basis_derivative_with_zero_imag(
    u: torch.Tensor, axis: int = -1, frequency_offset: int = 0
) -> torch.Tensor:
    if axis >= 0:
        raise ValueError("axis must be negative")
    n = u.shape[axis]
    if n % 2:
        raise ValueError(f"u.shape along axis={axis} must be even, got {n}")
    k = torch.arange(n, device=u.device)
    j = frequency_offset + k // 2
    src = torch.where(k % 2 == 0, k + 1, k - 1)
    scale = torch.where(k % 2 == 0, j, -j).to(u.dtype)
    shape = [1] * u.ndim
    shape[axis] = n
    return u.index_select(u.ndim + axis, src) * scale.reshape(shape)


def quadrature_nodes(nodes: int) -> tuple[np.ndarray, float]:
    xs = 2.0 * np.pi * np.arange(nodes, dtype=np.float64) / nodes
    return xs, 2.0 * np.pi / nodes
