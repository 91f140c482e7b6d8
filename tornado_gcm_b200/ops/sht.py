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
The "highest" precision setting runs the FP64 transforms on the FP64 tensor
cores instead (``csrc/dgemm.cu``; the Z0 zone and the numerical oracle mode).
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


# ── FP64 transforms on the FP64 tensor cores (csrc/dgemm.cu) ────────────────
# Four batched strided DGEMMs, no transposed copies:
#   synthesis  W[k, s, j]   = sum_l x[s, k, l] p[k, j, l]           (batch: zonal row k)
#              out[s, i, j] = sum_k F[i, k] W[k, s, j]              (batch: slice s)
#   analysis   Z[k, s, j]   = w_j sum_i F[i, k] x[s, i, j]          (batch: slice s)
#              out[s, k, l] = sum_j Z[k, s, j] p[k, j, l]           (batch: zonal row k)
# with p the per-row Legendre table (M2, J, L).  The adjoint of synthesis is
# the unweighted analysis and the adjoint of analysis the weighted synthesis.
def _f64_synth(x3: torch.Tensor, sh, weighted: bool) -> torch.Tensor:
    ops = _ext.require("FP64 synthesis")
    S, M2, L = x3.shape
    p = sh.device_basis("p", x3.device, torch.float64)
    f = sh.device_basis("f", x3.device, torch.float64)
    I, J = f.shape[0], p.shape[1]
    x3 = x3.to(torch.float64).contiguous()
    if weighted:
        p = p * sh.device_basis("w", x3.device, torch.float64)[None, :, None]
    W = torch.empty(M2, S, J, dtype=torch.float64, device=x3.device)
    ops.dgemm_strided(x3, p, W, S, J, L, M2, [M2 * L, 1, L], [L, 1, J * L], [J, 1, S * J], 1.0, 0.0, None)
    out = torch.empty(S, I, J, dtype=torch.float64, device=x3.device)
    ops.dgemm_strided(f, W, out, I, J, M2, S, [M2, 1, 0], [1, S * J, J], [J, 1, I * J], 1.0, 0.0, None)
    return out


def _f64_anal(n3: torch.Tensor, sh, weighted: bool) -> torch.Tensor:
    ops = _ext.require("FP64 analysis")
    S, I, J = n3.shape
    p = sh.device_basis("p", n3.device, torch.float64)
    f = sh.device_basis("f", n3.device, torch.float64)
    M2, L = p.shape[0], p.shape[2]
    n3 = n3.to(torch.float64).contiguous()
    w = sh.device_basis("w", n3.device, torch.float64) if weighted else None
    Z = torch.empty(M2, S, J, dtype=torch.float64, device=n3.device)
    ops.dgemm_strided(f, n3, Z, M2, J, I, S, [1, M2, 0], [1, J, I * J], [S * J, 1, J], 1.0, 0.0, w)
    out = torch.empty(S, M2, L, dtype=torch.float64, device=n3.device)
    ops.dgemm_strided(Z, p, out, S, L, J, M2, [J, 1, S * J], [1, L, J * L], [M2 * L, 1, L], 1.0, 0.0, None)
    return out


class _F64SynthFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x3, sh):
        ctx.sh = sh
        return _f64_synth(x3, sh, False)

    @staticmethod
    def backward(ctx, g):
        return _f64_anal(g, ctx.sh, False), None


class _F64AnalFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, n3, sh):
        ctx.sh = sh
        return _f64_anal(n3, sh, True)

    @staticmethod
    def backward(ctx, g):
        return _f64_synth(g, ctx.sh, True), None


def _highest(x, sh, inverse: bool):
    """FP64 transform of a CUDA tensor on the FP64 tensor cores; the result keeps ``x``'s dtype."""
    lead = x.shape[:-2]
    x3 = x.reshape((-1,) + tuple(x.shape[-2:]))
    if x3.shape[0] == 0:
        shape = (sh.longitude_nodes, sh.latitude_nodes) if inverse else tuple(sh.modal_shape)
        return x.new_zeros(lead + shape)
    out = _F64SynthFn.apply(x3, sh) if inverse else _F64AnalFn.apply(x3, sh)
    return out.reshape(lead + tuple(out.shape[-2:])).to(x.dtype)
