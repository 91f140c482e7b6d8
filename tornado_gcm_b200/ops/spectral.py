"""Table-driven spectral linear operators (``csrc/spectral_ops.cu``).

A :class:`SpectralRecipe` describes a linear map from stacked modal fields
``x (B, C_in, 2M-1, L)`` to ``y (B, C_out, 2M-1, L)`` as, for every output
slice, a sum of terms ``coef · post[l] · D(pre[l] · x[src])`` where ``D`` is a
spherical-harmonic stencil (identity, ∂/∂λ, cosθ∂/∂θ, secθ∂/∂θ cos², the
transposes of the latitudinal two) or one row of a vertical matrix.  The
adjoint of a recipe is obtained by transposing its term table, so every
recipe becomes an autograd op whose backward is the same kernel.

Recipes built here:

* :func:`explicit_pre_recipe` — packed prognostic state → the stacked
  modal inputs of the explicit-tendency column kernel (ζ, δ, T', u, v,
  tracers, ∇q, ∇ln ps, ∇² ln ps);
* :func:`explicit_post_recipe` — forward-transformed column outputs → the
  packed explicit tendency (curl/div of fluxes, ∇² of kinetic energy and
  of the moist geopotential correction, last-wavenumber clip).

Packed channel order: ``[ζ (n) | δ (n) | T' (n) | ln ps (1) | tracers (n each, sorted keys)]``.
"""

from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np
import torch

from tornado_gcm_b200.ops import _ext

ID, DLON, CDLAT, HDLAT, CDLAT_T, HDLAT_T, VERT, VERT_T = range(8)
_TRANSPOSE = {ID: ID, DLON: DLON, CDLAT: CDLAT_T, HDLAT: HDLAT_T, CDLAT_T: CDLAT, HDLAT_T: HDLAT,
              VERT: VERT_T, VERT_T: VERT}
_SIGN_T = {DLON: -1.0}


@dataclasses.dataclass
class Term:
    dst: int
    src: int
    stencil: int = ID
    pre: int = -1
    post: int = -1
    coef: float = 1.0
    mat: int = 0
    row: int = 0


class SpectralRecipe:
    def __init__(self, grid, c_in: int, c_out: int, terms: list, diags: list, mats: list, nlev: int):
        self.grid = grid
        self.c_in, self.c_out = c_in, c_out
        self.terms = sorted(terms, key=lambda t: t.dst)
        self.diags = diags
        self.mats = mats
        self.nlev = nlev
        self._dev: dict = {}
        self._transpose: Optional["SpectralRecipe"] = None

    def transpose(self) -> "SpectralRecipe":
        if self._transpose is None:
            tt = []
            for t in self.terms:
                st = _TRANSPOSE[t.stencil]
                tt.append(Term(dst=t.src, src=t.dst, stencil=st, pre=t.post, post=t.pre,
                               coef=t.coef * _SIGN_T.get(t.stencil, 1.0), mat=t.mat, row=t.row))
            # vertical terms: dst/src name the first level of the block; the transposed
            # term for output row r reads the block of n outputs starting at src base.
            fixed = []
            for t, orig in zip(tt, self.terms):
                if orig.stencil in (VERT, VERT_T):
                    # original: y[dst] += Σ_k M[row,k] x[src+k]  → x̄[src+k] += M[row,k] ȳ[dst]
                    # express per destination level k as one term over the n-block of ȳ:
                    # handled by expanding into per-level transposed terms below
                    continue
                fixed.append(t)
            for orig in self.terms:
                if orig.stencil in (VERT, VERT_T):
                    for k in range(self.nlev):
                        w = self.mats[orig.mat][orig.row, k] if orig.stencil == VERT else self.mats[orig.mat][k, orig.row]
                        if w == 0.0:
                            continue
                        fixed.append(Term(dst=orig.src + k, src=orig.dst, stencil=ID, pre=orig.post, post=orig.pre,
                                          coef=orig.coef * float(w)))
            r = SpectralRecipe(self.grid, self.c_out, self.c_in, fixed, self.diags, self.mats, self.nlev)
            r._transpose = self
            self._transpose = r
        return self._transpose

    def tables(self, device):
        key = str(device)
        d = self._dev.get(key)
        if d is None:
            rows = np.zeros(self.c_out + 1, dtype=np.int32)
            for t in self.terms:
                rows[t.dst + 1] += 1
            rows = np.cumsum(rows).astype(np.int32)
            terms = np.array([[t.dst, t.src, t.stencil, t.pre, t.post, t.mat, t.row] for t in self.terms],
                             dtype=np.int32).reshape(-1, 7)
            coef = np.array([t.coef for t in self.terms], dtype=np.float32)
            L = self.grid.modal_shape[-1]
            diag = np.stack(self.diags) if self.diags else np.zeros((1, L))
            a, b = self.grid._derivative_recurrence_weights
            mats = np.stack(self.mats) if self.mats else np.zeros((1, 1, 1))
            f32 = lambda x: torch.as_tensor(np.ascontiguousarray(x), dtype=torch.float32, device=device)
            d = (torch.as_tensor(rows, device=device), torch.as_tensor(terms, device=device), f32(coef), f32(diag),
                 f32(a), f32(b), f32(mats))
            self._dev[key] = d
        return d

    def apply(self, x: torch.Tensor, out_lpad: Optional[int] = None) -> torch.Tensor:
        ops = _ext.require("spectral linear operator")
        L = self.grid.modal_shape[-1]
        out_lpad = L if out_lpad is None else out_lpad
        # a wavenumber-sharded grid supplies |m| of each local row (for ∂/∂λ)
        row_m = self.grid.row_wavenumbers(x.device) if hasattr(self.grid, "row_wavenumbers") else None
        err = _ext.error_flag(x.device) if x.is_cuda else None
        return ops.spectral_linear(x, L, self.c_out, out_lpad, *self.tables(x.device), self.nlev, row_m, err)


class SpectralLinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, recipe: SpectralRecipe, out_lpad: int, grad_lpad: int):
        ctx.recipe, ctx.grad_lpad = recipe, grad_lpad
        L = recipe.grid.modal_shape[-1]
        y = recipe.apply(x, out_lpad)
        # rows padded to out_lpad (16-byte aligned for TMA); expose the logical L view
        return y[..., :L] if out_lpad > L else y

    @staticmethod
    def backward(ctx, gy):
        L = ctx.recipe.grid.modal_shape[-1]
        g = ctx.recipe.transpose().apply(gy if gy.stride(-1) == 1 else gy.contiguous(), ctx.grad_lpad)
        return (g[..., :L] if ctx.grad_lpad > L else g), None, None, None


def spectral_linear(x: torch.Tensor, recipe: SpectralRecipe, out_lpad: Optional[int] = None,
                    grad_lpad: Optional[int] = None) -> torch.Tensor:
    L = recipe.grid.modal_shape[-1]
    return SpectralLinearFn.apply(x, recipe, out_lpad or L, grad_lpad or L)


# ── recipe builders ─────────────────────────────────────────────────────────
class _Builder:
    def __init__(self, grid, nlev):
        self.grid = grid
        self.nlev = nlev
        L = grid.modal_shape[-1]
        lam = np.asarray(grid.laplacian_eigenvalues, dtype=np.float64)
        ilam = np.zeros_like(lam)
        ilam[1:] = 1.0 / lam[1:]
        clip = np.ones(L)
        clip[-1] = 0.0
        self.diags = [lam, ilam, clip, lam * clip]
        self.LAP, self.ILAP, self.CLIP, self.LAPCLIP = 0, 1, 2, 3
        self.mats: list = []
        self.terms: list = []

    def add(self, dst, src, stencil=ID, pre=-1, post=-1, coef=1.0, mat=0, row=0):
        self.terms.append(Term(dst, src, stencil, pre, post, float(coef), mat, row))

    def recipe(self, c_in, c_out) -> SpectralRecipe:
        return SpectralRecipe(self.grid, c_in, c_out, self.terms, self.diags, self.mats, self.nlev)


def packed_channels(n: int, tracer_keys) -> dict:
    ch = {"vort": 0, "div": n, "temp": 2 * n, "lnps": 3 * n}
    for i, k in enumerate(tracer_keys):
        ch["tr:" + k] = 3 * n + 1 + i * n
    ch["C"] = 3 * n + 1 + len(tracer_keys) * n
    return ch


def explicit_pre_recipe(eq, tracer_keys, grid=None) -> SpectralRecipe:
    grid = eq.grid if grid is None else grid
    n = eq.vertical.layers
    inv_r = 1.0 / grid.radius
    b = _Builder(grid, n)
    ch = packed_channels(n, tracer_keys)
    nt = len(tracer_keys)
    h = 1 if eq.humidity_key is not None else 0
    s = 0
    for k in range(n):
        b.add(s + k, ch["vort"] + k)
    s += n
    for k in range(n):
        b.add(s + k, ch["div"] + k)
    s += n
    for k in range(n):
        b.add(s + k, ch["temp"] + k)
    s += n
    for k in range(n):  # u = ∂λ χ − cosθ∂θ ψ
        b.add(s + k, ch["div"] + k, DLON, pre=b.ILAP, coef=inv_r)
        b.add(s + k, ch["vort"] + k, CDLAT, pre=b.ILAP, coef=-inv_r)
    s += n
    for k in range(n):  # v = cosθ∂θ χ + ∂λ ψ
        b.add(s + k, ch["div"] + k, CDLAT, pre=b.ILAP, coef=inv_r)
        b.add(s + k, ch["vort"] + k, DLON, pre=b.ILAP, coef=inv_r)
    s += n
    for key in tracer_keys:
        for k in range(n):
            b.add(s + k, ch["tr:" + key] + k)
        s += n
    if h:
        hk = eq.humidity_key
        if ("tr:" + hk) in ch:
            for k in range(n):
                b.add(s + k, ch["tr:" + hk] + k, DLON, coef=inv_r)
                b.add(s + n + k, ch["tr:" + hk] + k, CDLAT, coef=inv_r)
        s += 2 * n
    b.add(s, ch["lnps"], DLON, coef=inv_r)
    b.add(s + 1, ch["lnps"], CDLAT, coef=inv_r)
    s += 2
    if h:
        b.add(s, ch["lnps"], ID, post=b.LAP)
        s += 1
    assert s == (5 + nt + 2 * h) * n + 2 + h
    return b.recipe(ch["C"], s)


def explicit_post_recipe(eq, tracer_keys, g_fused: bool = False, grid=None) -> SpectralRecipe:
    """``g_fused``: the column kernel already applied G to the tdiff outputs."""
    grid = eq.grid if grid is None else grid
    n = eq.vertical.layers
    inv_r = 1.0 / grid.radius
    b = _Builder(grid, n)
    ch = packed_channels(n, tracer_keys)
    nt = len(tracer_keys)
    h = 1 if eq.humidity_key is not None else 0
    o_fu, o_fv, o_ke, o_tn, o_tu, o_tv = 0, n, 2 * n, 3 * n, 4 * n, 5 * n
    o_tr = 6 * n
    o_td = (6 + 3 * nt) * n
    o_hd, o_hv = o_td + n, o_td + 2 * n
    o_lnps = (6 + 3 * nt + 3 * h) * n
    C, CL, LC = b.CLIP, b.CLIP, b.LAPCLIP
    if h and not g_fused:
        b.mats.append(np.asarray(eq._G_matrix, dtype=np.float64))
    for k in range(n):
        # vorticity: −(∂λ Fv − H Fu) + hum_vort
        b.add(ch["vort"] + k, o_fv + k, DLON, post=CL, coef=-inv_r)
        b.add(ch["vort"] + k, o_fu + k, HDLAT, post=CL, coef=inv_r)
        # divergence: −(∂λ Fu + H Fv) − ∇² ke − ∇² (G·tdiff) − hum_div
        b.add(ch["div"] + k, o_fu + k, DLON, post=CL, coef=-inv_r)
        b.add(ch["div"] + k, o_fv + k, HDLAT, post=CL, coef=-inv_r)
        b.add(ch["div"] + k, o_ke + k, ID, post=LC, coef=-1.0)
        # temperature: T-nodal term − (∂λ Tu + H Tv)
        b.add(ch["temp"] + k, o_tn + k, ID, post=CL)
        b.add(ch["temp"] + k, o_tu + k, DLON, post=CL, coef=-inv_r)
        b.add(ch["temp"] + k, o_tv + k, HDLAT, post=CL, coef=-inv_r)
        for i, key in enumerate(tracer_keys):
            base = o_tr + 3 * i * n
            b.add(ch["tr:" + key] + k, base + k, ID, post=CL)
            b.add(ch["tr:" + key] + k, base + n + k, DLON, post=CL, coef=-inv_r)
            b.add(ch["tr:" + key] + k, base + 2 * n + k, HDLAT, post=CL, coef=-inv_r)
        if h:
            b.add(ch["vort"] + k, o_hv + k, ID, post=CL)
            b.add(ch["div"] + k, o_hd + k, ID, post=CL, coef=-1.0)
            if g_fused:
                b.add(ch["div"] + k, o_td + k, ID, post=LC, coef=-1.0)
            else:
                b.add(ch["div"] + k, o_td, VERT, post=LC, coef=-1.0, mat=0, row=k)
    b.add(ch["lnps"], o_lnps, ID, post=CL)
    return b.recipe(o_lnps + 1, ch["C"])


def _state_parts(state, tracer_keys) -> list:
    parts = [state.vorticity, state.divergence, state.temperature_variation, state.log_surface_pressure]
    return parts + [state.tracers[k] for k in tracer_keys]


def _views_of(parts: list, packed: torch.Tensor) -> bool:
    """Every part is still the channel slice of ``packed`` that unpack_state made."""
    step = packed.stride(-3) * packed.element_size()
    off = 0
    for t in parts:
        if (t.dim() != packed.dim() or t.data_ptr() != packed.data_ptr() + off * step
                or t.shape[:-3] != packed.shape[:-3] or t.shape[-2:] != packed.shape[-2:]
                or t.stride() != packed.stride() or t.requires_grad != packed.requires_grad):
            return False
        off += t.shape[-3]
    return off == packed.shape[-3]


def pack_state(state, tracer_keys) -> torch.Tensor:
    """Channels ``[ζ | δ | T' | ln ps | tracers]`` of ``state`` as one tensor.

    A state made by :func:`unpack_state` whose fields are still the slices of
    that packed tensor returns the tensor itself: re-packing copies nothing in
    the forward pass, and backward does not rebuild the packed gradient from
    per-slice zero-filled copies and additions.
    """
    parts = _state_parts(state, tracer_keys)
    src = getattr(state, "_packed_src", None)
    if src is not None and src[1] == tuple(tracer_keys) and _views_of(parts, src[0]):
        return src[0]
    return torch.cat(parts, dim=-3)


def unpack_state(packed: torch.Tensor, n: int, tracer_keys, sim_time=None, extra_tracers=None):
    from tornado_gcm_b200.core.primitive_equations import State

    vort, div, temp, lnps = packed[..., :n, :, :], packed[..., n:2 * n, :, :], packed[..., 2 * n:3 * n, :, :], \
        packed[..., 3 * n:3 * n + 1, :, :]
    tr = {}
    for i, k in enumerate(tracer_keys):
        tr[k] = packed[..., 3 * n + 1 + i * n:3 * n + 1 + (i + 1) * n, :, :]
    if extra_tracers:
        tr.update(extra_tracers)
    st = State(vort, div, temp, lnps, tr, sim_time)
    if not extra_tracers and packed.shape[-3] == (3 + len(tracer_keys)) * n + 1:
        st._packed_src = (packed, tuple(tracer_keys))
    return st


def carry_packed(src_state, dst_state):
    """Keep the packed-tensor link of ``src_state`` on a copy with other metadata (e.g. sim_time)."""
    link = getattr(src_state, "_packed_src", None)
    if link is not None:
        dst_state._packed_src = link
    return dst_state


def param_pre_recipe(grid, n: int, state_keys, param_keys) -> SpectralRecipe:
    """Packed state → modal column-physics inputs ``[cosθ·u | cosθ·v | T' | tracers | ln ps]``.

    ``param_keys`` is the parameterization's tracer order; a tracer missing
    from ``state_keys`` stays zero (no terms).  The velocity rows are the
    unclipped cosθ-weighted wind of reference
    ``core/spherical_harmonic.py`` ``get_cos_lat_vector`` (ψ, χ by inverse
    Laplacian, then ∂λ and cosθ∂θ).
    """
    inv_r = 1.0 / grid.radius
    b = _Builder(grid, n)
    ch = packed_channels(n, state_keys)
    for k in range(n):
        b.add(k, ch["div"] + k, DLON, pre=b.ILAP, coef=inv_r)
        b.add(k, ch["vort"] + k, CDLAT, pre=b.ILAP, coef=-inv_r)
        b.add(n + k, ch["div"] + k, CDLAT, pre=b.ILAP, coef=inv_r)
        b.add(n + k, ch["vort"] + k, DLON, pre=b.ILAP, coef=inv_r)
        b.add(2 * n + k, ch["temp"] + k)
    s = 3 * n
    for key in param_keys:
        if ("tr:" + key) in ch:
            for k in range(n):
                b.add(s + k, ch["tr:" + key] + k)
        s += n
    b.add(s, ch["lnps"])
    return b.recipe(ch["C"], s + 1)


def param_post_recipe(grid, n: int, state_keys, param_keys) -> SpectralRecipe:
    """Modal column-physics outputs ``[u/cosθ | v/cosθ | T' | tracers | ln ps]`` → packed tendency.

    ζ and δ tendencies are the clipped curl / divergence of the cosθ-weighted
    velocity tendency (reference ``neural/parameterizations.py``
    ``ModalNeuralDivCurlParameterization``); state tracers that the network
    does not predict get a zero tendency.
    """
    inv_r = 1.0 / grid.radius
    b = _Builder(grid, n)
    ch = packed_channels(n, state_keys)
    for k in range(n):
        b.add(ch["vort"] + k, n + k, DLON, post=b.CLIP, coef=inv_r)
        b.add(ch["vort"] + k, k, HDLAT, post=b.CLIP, coef=-inv_r)
        b.add(ch["div"] + k, k, DLON, post=b.CLIP, coef=inv_r)
        b.add(ch["div"] + k, n + k, HDLAT, post=b.CLIP, coef=inv_r)
        b.add(ch["temp"] + k, 2 * n + k)
    s = 3 * n
    for key in param_keys:
        if ("tr:" + key) in ch:
            for k in range(n):
                b.add(ch["tr:" + key] + k, s + k)
        s += n
    b.add(ch["lnps"], s)
    return b.recipe(s + 1, ch["C"])
