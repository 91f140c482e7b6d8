"""Spherical-harmonic transforms on sm_100a (tcgen05 TF32 GEMMs).

``to_nodal`` = Legendre synthesis (grouped per zonal wavenumber m, cos/sin
rows paired so one tile row-block serves both) followed by the real-DFT
synthesis against a resident Fourier basis; ``to_modal`` = quadrature-
weighted DFT analysis followed by Legendre analysis.  Both are
``torch.autograd.Function`` s whose adjoints are the opposite transforms:

* adjoint of synthesis  = analysis without quadrature weights;
* adjoint of analysis   = w_j ⊙ synthesis.

Bases are built once per grid in FP64, cast to fp32 and kept on the device:
``P (Mw, J, Lp)``, ``Pt (Mw, L, J)``, ``F (I, M2p)``, ``Ft (M2, I)``, ``w (J)``.
The "highest" precision setting runs FP64 torch contractions instead (the
numerical oracle mode).
"""

from __future__ import annotations

import numpy as np
import torch

from tornado_gcm_b200.ops import _ext


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class _Bases:
    def __init__(self, sh, device):
        Mw = sh.longitude_wavenumbers
        L = sh.total_wavenumbers
        I = sh.longitude_nodes
        J = sh.latitude_nodes
        M2 = 2 * Mw - 1
        self.L, self.Lp, self.I, self.J, self.M2 = L, _round_up(L, 4), I, J, M2
        self.M2p = _round_up(M2, 4)
        p = sh.legendre_table  # (Mw, J, L)
        pp = np.zeros((Mw, J, self.Lp))
        pp[:, :, :L] = p
        f = sh.basis.f  # (I, M2)
        fp = np.zeros((I, self.M2p))
        fp[:, :M2] = f
        dev = torch.device(device)
        t = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float32, device=dev)
        self.P = t(pp)
        self.Pt = t(np.transpose(p, (0, 2, 1)))
        # quadrature weights folded into the Legendre bases: the weighted
        # analysis and its adjoint then run the one-GEMM Fourier steps
        wj = np.asarray(sh.basis.w, dtype=np.float64)
        self.Pw = t(pp * wj[None, :, None])
        self.Ptw = t(np.transpose(p, (0, 2, 1)) * wj[None, None, :])
        self.F = t(fp)
        self.Ft = t(f.T)
        self.w = t(sh.basis.w)
        if I % 4 or J % 4:
            raise ValueError("GPU transforms need lon/lat node counts divisible by 4")


_BASES: dict = {}


def bases(sh, device) -> _Bases:
    key = (id(sh), str(device))
    entry = _BASES.get(key)
    if entry is None:
        entry = (_Bases(sh, device), sh)  # keep sh alive so id() stays unique
        _BASES[key] = entry
    return entry[0]


def _synth(x3: torch.Tensor, b: _Bases, col_scale=None, lat_major: bool = False,
           weighted: bool = False) -> torch.Tensor:
    """Modal (S, M2, L) → nodal; x3 may be a strided view of a row-padded buffer."""
    ops = _ext.require("spherical-harmonic synthesis")
    S = x3.shape[0]
    x3 = x3.float()
    ok = (x3.stride(-1) == 1 and (x3.stride(-2) * 4) % 16 == 0 and (x3.stride(0) * 4) % 16 == 0
          and x3.data_ptr() % 16 == 0)
    if not ok:
        x3 = torch.nn.functional.pad(x3, (0, b.Lp - b.L)).contiguous() if b.Lp != b.L else x3.contiguous()
        if b.Lp != b.L:
            x3 = x3[..., : b.L]
    ws = _ext.empty(S * b.J * b.M2p, dtype=torch.float32, device=x3.device)
    return ops.sht_synth(x3, b.L, b.Pw if weighted else b.P, b.F, ws, col_scale, _ext.error_flag(x3.device),
                         lat_major)


def _anal(n3: torch.Tensor, b: _Bases, col_scale=None, lat_major: bool = False,
          weighted: bool = False) -> torch.Tensor:
    """Nodal (S, I, J) (or (S, J, I) when lat_major) → modal (S, M2, L).

    The lat-major (internal) result is the ``[..., :L]`` view of rows padded
    to ``Lp`` (a multiple of 4): the Legendre epilogue then stores whole
    16-byte vectors, and the spectral operators that consume it take strided
    rows.  The public lon-major result stays contiguous.
    """
    ops = _ext.require("spherical-harmonic analysis")
    S = n3.shape[0]
    ws = _ext.empty(S * b.M2 * b.J, dtype=torch.float32, device=n3.device)
    lo = b.Lp if lat_major else b.L
    out = ops.sht_anal(n3.float(), b.Ft, b.Ptw if weighted else b.Pt, lo, ws, col_scale,
                       _ext.error_flag(n3.device), lat_major)
    return out[..., : b.L] if lo != b.L else out


class ToNodalFn(torch.autograd.Function):
    """Synthesis; adjoint = unweighted analysis (same nodal layout)."""

    @staticmethod
    def forward(ctx, x3, b, lat_major=False):
        ctx.b, ctx.lat_major = b, lat_major
        return _synth(x3, b, None, lat_major)

    @staticmethod
    def backward(ctx, g):
        return _anal(g, ctx.b, None, ctx.lat_major), None, None


class ToModalFn(torch.autograd.Function):
    """Quadrature-weighted analysis; adjoint = w_j ⊙ synthesis."""

    @staticmethod
    def forward(ctx, n3, b, lat_major=False):
        ctx.b, ctx.lat_major = b, lat_major
        return _anal(n3, b, None, lat_major, weighted=True)

    @staticmethod
    def backward(ctx, g):
        return _synth(g, ctx.b, None, ctx.lat_major, weighted=True), None, None


def to_nodal(x: torch.Tensor, sh) -> torch.Tensor:
    """Modal (…, 2M-1, L) → nodal (…, I, J) on the GPU."""
    if sh.precision == "highest":
        return _highest(x, sh, inverse=True)
    b = bases(sh, x.device)
    lead = x.shape[:-2]
    out = ToNodalFn.apply(x.reshape(-1, b.M2, b.L).float(), b, False)
    return out.reshape(*lead, b.I, b.J).to(x.dtype)


def to_modal(x: torch.Tensor, sh) -> torch.Tensor:
    """Nodal (…, I, J) → modal (…, 2M-1, L) on the GPU."""
    if sh.precision == "highest":
        return _highest(x, sh, inverse=False)
    b = bases(sh, x.device)
    lead = x.shape[:-2]
    out = ToModalFn.apply(x.reshape(-1, b.I, b.J).float(), b, False)
    return out.reshape(*lead, b.M2, b.L).to(x.dtype)


def to_nodal_lat_major(x3: torch.Tensor, sh) -> torch.Tensor:
    """(S, 2M-1, L) modal (may be a row-padded view) → (S, J, I) nodal (internal layout)."""
    if sh.precision == "highest":
        return _highest(x3, sh, inverse=True).transpose(-1, -2).contiguous()
    return ToNodalFn.apply(x3, bases(sh, x3.device), True)


def to_modal_lat_major(n3: torch.Tensor, sh) -> torch.Tensor:
    """(S, J, I) nodal → (S, 2M-1, L) modal."""
    if sh.precision == "highest":
        return _highest(n3.transpose(-1, -2), sh, inverse=False)
    return ToModalFn.apply(n3, bases(sh, n3.device), True)


def _highest(x, sh, inverse: bool):
    p = sh.device_basis("p", x.device, torch.float64)
    f = sh.device_basis("f", x.device, torch.float64)
    x64 = x.to(torch.float64)
    if inverse:
        out = torch.einsum("im,...mj->...ij", f, torch.einsum("mjl,...ml->...mj", p, x64))
    else:
        w = sh.device_basis("w", x.device, torch.float64)
        out = torch.einsum("mjl,...mj->...ml", p, torch.einsum("im,...ij->...mj", f, x64 * w))
    return out.to(x.dtype)
