"""Fused dycore path on sm_100a.

* :class:`ColumnSpec` — slice layout and constants of the per-column
  nonlinear tendency kernel (``csrc/dycore_column.h``).
* :class:`ColumnFn` — autograd op: forward kernel, backward = the
  hand-written VJP kernel (both also have CPU twins used as oracles).
* :class:`ImplicitSolveFn` / :class:`ImplicitTermsFn` — per-wavenumber
  vertical operators; backward = their transposes (same kernel, modes 1/3).
* :func:`explicit_terms` — spectral pre-processing → stacked TF32 synthesis
  → column kernel → stacked TF32 analysis → spectral post-processing.
* :class:`FusedSIL3` — one IMEX-SIL3 substep (Whitaker & Kar 2013 tableau,
  same as ``core.time_integration.SIL3_TABLEAU``) with the constant physics
  tendency, the combined spectral filter and the inner-state sanitiser.
  The last stage is returned directly: SIL3 is stiffly accurate (its final
  implicit weight row equals b_im), so y_out = y_3 exactly in exact
  arithmetic and one implicit-terms evaluation is saved.
"""

from __future__ import annotations

import dataclasses
from typing import Optional, Sequence

import numpy as np
import torch

from tornado_gcm_b200.core import primitive_equations as pe
from tornado_gcm_b200.ops import _ext

State = pe.State


@dataclasses.dataclass
class ColumnSpec:
    n: int
    tracer_keys: tuple
    hum: int
    hum_terms: int
    clouds: list
    vadv: int
    R: float
    kappa: float
    rv: float
    cpv: float
    level_consts: torch.Tensor  # (5, n) fp32 on CPU
    sec2: np.ndarray
    cor: np.ndarray
    eq: object = None
    _dev: dict = dataclasses.field(default_factory=dict)
    # (n, n) geopotential matrix applied to the humidity tdiff outputs inside the
    # column kernel (the spectral post-processing then skips its vertical term)
    gmat: Optional[torch.Tensor] = None

    @classmethod
    def from_equation(cls, eq: pe.PrimitiveEquationsSigma, tracer_keys: Sequence[str]) -> "ColumnSpec":
        c = eq.column_constants
        keys = tuple(tracer_keys)
        n = eq.vertical.layers
        hum = keys.index(eq.humidity_key) if (eq.humidity_key is not None and eq.humidity_key in keys) else -1
        clouds = [keys.index(k) for k in (eq.cloud_keys or ()) if k in keys]
        idc = np.zeros(n)
        idc[: n - 1] = c.inv_dcenter
        lc = torch.tensor(np.stack([c.dsigma, c.alpha, c.t_ref, idc, c.cum_dsigma]), dtype=torch.float32)
        return cls(n, keys, hum, 1 if eq.humidity_key is not None else 0, clouds, 1 if c.vertical_advection else 0,
                   c.R, c.kappa, c.rv_ratio, c.cpv_ratio, lc, c.sec2, c.coriolis, eq)

    @property
    def n_in(self) -> int:
        h = self.hum_terms
        return (5 + len(self.tracer_keys) + 2 * h) * self.n + 2 + h

    @property
    def n_out(self) -> int:
        return (6 + 3 * len(self.tracer_keys) + 3 * self.hum_terms) * self.n + 1

    def device_consts(self, device):
        key = str(device)
        d = self._dev.get(key)
        if d is None:
            d = (torch.as_tensor(self.sec2, dtype=torch.float32, device=device),
                 torch.as_tensor(self.cor, dtype=torch.float32, device=device))
            self._dev[key] = d
        return d

    def device_gmat(self, device):
        if self.gmat is None:
            return None
        key = "gmat:" + str(device)
        g = self._dev.get(key)
        if g is None:
            g = self.gmat.to(device=device, dtype=torch.float32).contiguous()
            self._dev[key] = g
        return g

    def with_fused_g(self) -> "ColumnSpec":
        """A copy whose column kernel applies the geopotential matrix G to tdiff."""
        g = torch.as_tensor(np.asarray(self.eq._G_matrix), dtype=torch.float32) if self.hum_terms else None
        return dataclasses.replace(self, gmat=g, _dev={})

    def args(self):
        return (self.level_consts, self.n, len(self.tracer_keys), self.hum, self.hum_terms, list(self.clouds),
                self.vadv, self.R, self.kappa, self.rv, self.cpv)

    # helpers for tests: dict <-> stacked (B*S, I, J)
    def stack_inputs(self, inp: dict) -> torch.Tensor:
        parts = [inp["vort"], inp["div"], inp["temp"], inp["u"], inp["v"]]
        parts += [inp["tracers"][k] for k in self.tracer_keys]
        if self.hum_terms:
            parts += [inp["qx"], inp["qy"]]
        parts += [inp["gx"], inp["gy"]]
        if self.hum_terms:
            parts += [inp["lap_lnps"]]
        x = torch.cat(parts, dim=-3)
        return x.reshape(-1, *x.shape[-2:])

    def stack_outputs(self, out: dict) -> torch.Tensor:
        parts = [out[k] for k in ("flux_u", "flux_v", "ke", "temp", "temp_u", "temp_v")]
        for k in self.tracer_keys:
            parts += [out["tr:" + k], out["tr_u:" + k], out["tr_v:" + k]]
        if self.hum_terms:
            parts += [out["tdiff"], out["hum_div"], out["hum_vort"]]
        parts += [out["lnps"]]
        x = torch.cat(parts, dim=-3)
        return x.reshape(-1, *x.shape[-2:])


def column_forward_raw(spec: ColumnSpec, nin: torch.Tensor, batch: int, lat_major: bool = False) -> torch.Tensor:
    ops = _ext.require("column tendency")
    s2, co = spec.device_consts(nin.device)
    return ops.column_fwd(nin.contiguous(), s2, co, *_args_with_batch(spec, batch), lat_major,
                          spec.device_gmat(nin.device))


def column_vjp_raw(spec: ColumnSpec, nin: torch.Tensor, gout: torch.Tensor, batch: int,
                   lat_major: bool = False) -> torch.Tensor:
    ops = _ext.require("column tendency VJP")
    s2, co = spec.device_consts(nin.device)
    return ops.column_vjp(nin.contiguous(), gout.contiguous(), s2, co, *_args_with_batch(spec, batch), lat_major,
                          spec.device_gmat(nin.device))


def _args_with_batch(spec, batch):
    a = spec.args()
    return (a[0], batch) + a[1:]


class ColumnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, nin, spec, batch):
        ctx.spec, ctx.batch = spec, batch
        ctx.save_for_backward(nin)
        return column_forward_raw(spec, nin, batch)

    @staticmethod
    def backward(ctx, gout):
        (nin,) = ctx.saved_tensors
        return column_vjp_raw(ctx.spec, nin, gout, ctx.batch), None, None


# ── implicit operators ─────────────────────────────────────────────────────
class _ImplicitConsts:
    def __init__(self, eq: pe.PrimitiveEquationsSigma):
        self.eq = eq
        self.G = torch.tensor(eq._G_matrix, dtype=torch.float32)
        self.H = torch.tensor(eq._H_matrix, dtype=torch.float32)
        self.lam = torch.tensor(np.asarray(eq.grid.laplacian_eigenvalues, np.float64), dtype=torch.float32)
        self.tref = torch.tensor(eq.T_ref, dtype=torch.float32)
        self.dsig = torch.tensor(eq._dsigma, dtype=torch.float32)
        self._dev: dict = {}
        self._minv: dict = {}

    def on(self, device):
        key = str(device)
        d = self._dev.get(key)
        if d is None:
            d = tuple(t.to(device) for t in (self.G, self.H, self.lam, self.tref, self.dsig))
            self._dev[key] = d
        return d

    def minv(self, eta: float, device):
        key = (round(float(eta), 15), str(device))
        m = self._minv.get(key)
        if m is None:
            eq = self.eq
            g, h = eq._G_matrix, eq._H_matrix
            lam = np.asarray(eq.grid.laplacian_eigenvalues, np.float64)
            n = g.shape[0]
            core = g @ h + eq.R * np.outer(eq.T_ref, eq._dsigma)
            mats = np.eye(n)[None] - (eta * eta) * lam[:, None, None] * core[None]
            m = torch.tensor(np.linalg.inv(mats), dtype=torch.float32, device=device)
            self._minv[key] = m
        return m


def _consts(eq) -> _ImplicitConsts:
    c = getattr(eq, "_fused_implicit_consts", None)
    if c is None:
        c = _ImplicitConsts(eq)
        eq._fused_implicit_consts = c
    return c


def implicit_apply(eq, d, t, p, eta: float, mode: int):
    ops = _ext.require("implicit solve")
    c = _consts(eq)
    G, H, lam, tref, dsig = c.on(d.device)
    minv = c.minv(eta, d.device) if mode <= 1 else None
    squeeze = d.dim() == 3
    if squeeze:
        d, t, p = d.unsqueeze(0), t.unsqueeze(0), p.unsqueeze(0)
    out = ops.implicit_apply(d, t, p, G, H, minv, lam, tref, dsig, float(eq.R), float(eta), int(mode))
    if squeeze:
        out = [o.squeeze(0) for o in out]
    return out


class ImplicitSolveFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, d, t, p, eq, eta):
        ctx.eq, ctx.eta = eq, eta
        return tuple(implicit_apply(eq, d, t, p, eta, 0))

    @staticmethod
    def backward(ctx, gd, gt, gp):
        od, ot, op = implicit_apply(ctx.eq, gd.contiguous(), gt.contiguous(), gp.contiguous(), ctx.eta, 1)
        return od, ot, op, None, None


class ImplicitTermsFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, d, t, p, eq):
        ctx.eq = eq
        return tuple(implicit_apply(eq, d, t, p, 0.0, 2))

    @staticmethod
    def backward(ctx, gd, gt, gp):
        od, ot, op = implicit_apply(ctx.eq, gd.contiguous(), gt.contiguous(), gp.contiguous(), 0.0, 3)
        return od, ot, op, None


# ── explicit terms ─────────────────────────────────────────────────────────
def explicit_terms(eq: pe.PrimitiveEquationsSigma, state: State) -> State:
    """Fused GPU explicit tendency (TF32 transforms + column kernel)."""
    grid = eq.grid
    if grid.resolved_precision == "highest":
        return eq.explicit_terms_reference(state)
    keys = tuple(sorted(state.tracers))
    spec = _spec_for(eq, keys)
    lead = state.vorticity.shape[:-3]
    batch = int(np.prod(lead)) if len(lead) else 1
    dtype = state.vorticity.dtype
    st = state.tree_map(lambda x: x.float()) if dtype != torch.float32 else state
    modal_in = eq.modal_pre_stack(st, grid)
    nodal_in = grid.to_nodal(modal_in).reshape(batch * spec.n_in, *grid.nodal_shape)
    nodal_out = ColumnFn.apply(nodal_in, spec, batch)
    modal_out = grid.to_modal(nodal_out).reshape(*lead, spec.n_out, *grid.modal_shape)
    out = eq.modal_post(modal_out, st, grid)
    return out.tree_map(lambda x: x.to(dtype)) if dtype != torch.float32 else out


def _spec_for(eq, keys) -> ColumnSpec:
    cache = getattr(eq, "_column_specs", None)
    if cache is None:
        cache = {}
        eq._column_specs = cache
    s = cache.get(keys)
    if s is None:
        s = ColumnSpec.from_equation(eq, keys)
        cache[keys] = s
    return s


def implicit_terms(eq, state: State) -> State:
    d, t, p = ImplicitTermsFn.apply(state.divergence, state.temperature_variation, state.log_surface_pressure, eq)
    return State(torch.zeros_like(state.vorticity), d, t, p, {k: torch.zeros_like(v) for k, v in state.tracers.items()},
                 state.sim_time)


def implicit_inverse(eq, state: State, eta: float) -> State:
    d, t, p = ImplicitSolveFn.apply(state.divergence, state.temperature_variation, state.log_surface_pressure, eq,
                                    float(eta))
    return State(state.vorticity, d, t, p, state.tracers, state.sim_time)


# ── SIL3 substep ───────────────────────────────────────────────────────────
def _lin(terms):
    """Σ c_i · x_i over (coefficient, State) pairs (coefficients may be 0)."""
    out = None
    for c, x in terms:
        if c == 0:
            continue
        out = x * c if out is None else out + x * c
    return out


class FusedSIL3:
    """One SIL3 substep of dycore + constant physics, then filter + sanitise."""

    A_EX = [[1 / 3], [1 / 6, 1 / 2], [1 / 2, -1 / 2, 1]]
    A_IM = [[1 / 6, 1 / 6], [1 / 3, 0, 1 / 3], [3 / 8, 0, 3 / 8, 1 / 4]]

    def __init__(self, eq: pe.PrimitiveEquationsSigma, dt: float, filter_scaling: np.ndarray,
                 clamp_abs: float = 1.0e12, sanitize: bool = True):
        self.eq = eq
        self.dt = float(dt)
        self.filter_scaling = np.asarray(filter_scaling, dtype=np.float64)
        self.clamp_abs = clamp_abs
        self.sanitize = sanitize
        self._filt: dict = {}

    def _filter(self, device):
        key = str(device)
        f = self._filt.get(key)
        if f is None:
            f = torch.as_tensor(self.filter_scaling, dtype=torch.float32, device=device)
            self._filt[key] = f
        return f

    def step(self, y0: State, phys: State) -> State:
        eq, dt = self.eq, self.dt
        E = []
        ys = [y0]
        G0 = implicit_terms(eq, y0)
        Gs = {0: G0}
        for i in range(1, 4):
            E.append(explicit_terms(eq, ys[-1]) + phys)
            a_ex = self.A_EX[i - 1]
            a_im = self.A_IM[i - 1]
            terms = [(1.0, y0)] + [(dt * a_ex[j], E[j]) for j in range(i)]
            terms += [(dt * a_im[j], Gs[j]) for j in range(i) if a_im[j] != 0]
            y_star = _lin(terms)
            yi = implicit_inverse(eq, y_star, dt * a_im[i])
            ys.append(yi)
            if i == 2:
                Gs[2] = implicit_terms(eq, yi)
        out = ys[-1]
        f = self._filter(out.vorticity.device)
        out = out.tree_map(lambda x: x * f)
        if self.sanitize:
            c = self.clamp_abs
            out = out.tree_map(lambda x: torch.clamp(torch.nan_to_num(x, nan=0.0, posinf=c, neginf=-c), -c, c))
        return dataclasses.replace(out, sim_time=y0.sim_time)


# ── packed-state SIL3 (the production GPU path) ─────────────────────────────
def _synth_lat(x3: torch.Tensor, grid) -> torch.Tensor:
    """(S, M2, L) modal (possibly a padded-row view) → (S, J, I) nodal."""
    if getattr(grid, "sharded", False):
        return grid.to_nodal_lat_major(x3)
    if x3.is_cuda:
        from tornado_gcm_b200.ops import sht as sht_ops

        return sht_ops.to_nodal_lat_major(x3, grid.spherical_harmonics)
    return grid.to_nodal(x3).transpose(-1, -2).contiguous()


def _anal_lat(n3: torch.Tensor, grid) -> torch.Tensor:
    """(S, J, I) nodal → (S, M2, L) modal."""
    if getattr(grid, "sharded", False):
        return grid.to_modal_lat_major(n3)
    if n3.is_cuda:
        from tornado_gcm_b200.ops import sht as sht_ops

        return sht_ops.to_modal_lat_major(n3, grid.spherical_harmonics)
    return grid.to_modal(n3.transpose(-1, -2).contiguous())


class ColumnLatFn(torch.autograd.Function):
    """Column tendency on latitude-major nodal slices (S, J, I)."""

    @staticmethod
    def forward(ctx, nin, spec, batch):
        ctx.spec, ctx.batch = spec, batch
        ctx.save_for_backward(nin)
        ops = _ext.require("column tendency")
        s2, co = spec.device_consts(nin.device)
        return ops.column_fwd(nin.contiguous(), s2, co, *_args_with_batch(spec, batch), True,
                              spec.device_gmat(nin.device))

    @staticmethod
    def backward(ctx, gout):
        (nin,) = ctx.saved_tensors
        ops = _ext.require("column tendency VJP")
        s2, co = ctx.spec.device_consts(nin.device)
        g = ops.column_vjp(nin, gout.contiguous(), s2, co, *_args_with_batch(ctx.spec, ctx.batch), True,
                           ctx.spec.device_gmat(nin.device))
        return g, None, None


class StageFn(torch.autograd.Function):
    """One SIL3 stage on the packed state (explicit combination + implicit solve)."""

    @staticmethod
    def forward(ctx, y0, P, y2, E0, E1, E2, meta):
        ops = _ext.require("SIL3 stage")
        Es = [e for e in (E0, E1, E2) if e is not None]
        G, H, lam, tref, dsig = meta["consts"]
        out = ops.sil3_stage(y0.contiguous(), [e.contiguous() for e in Es], P.contiguous(), y2, meta["ce"],
                             meta["cp"], meta["cg"], meta["eta"], G, H, meta["minv"], lam, tref, dsig,
                             meta["filt"], meta["clamp"], meta["R"], meta["final"], meta["n"], meta.get("minv_t"))
        ctx.meta, ctx.nE, ctx.has_y2 = meta, len(Es), y2 is not None
        if meta["final"]:
            ctx.save_for_backward(out)
        return out

    @staticmethod
    def backward(ctx, g):
        ops = _ext.require("SIL3 stage adjoint")
        meta = ctx.meta
        G, H, lam, tref, dsig = meta["consts"]
        out = ctx.saved_tensors[0] if meta["final"] else g
        res = ops.sil3_stage_adjoint(g.contiguous(), out, ctx.nE, int(ctx.has_y2), meta["ce"], meta["cp"],
                                     meta["cg"], meta["eta"], G, H, meta["minv"], lam, tref, dsig, meta["filt"],
                                     meta["clamp"], meta["R"], meta["final"], meta["n"], meta.get("minv_t"))
        g_y0 = res[0]
        gE = list(res[1:1 + ctx.nE]) + [None] * (3 - ctx.nE)
        g_P = res[1 + ctx.nE]
        g_y2 = res[2 + ctx.nE] if ctx.has_y2 else None
        return g_y0, g_P, g_y2, gE[0], gE[1], gE[2], None


class PackedSIL3:
    """SIL3 substep on packed states ``[ζ | δ | T' | ln ps | tracers]`` (B, C, 2M-1, L).

    Per substep: 3 × (pre recipe → TF32 synthesis → column kernel → TF32
    analysis → post recipe) and 3 stage kernels; every piece has a kernel
    adjoint, so backward-through-rollout runs the same number of kernels.
    """

    def __init__(self, eq: pe.PrimitiveEquationsSigma, dt: float, filter_scaling: np.ndarray, tracer_keys,
                 clamp_abs: float = 1.0e12, grid=None):
        """``grid``: a sharded grid (parallel.spectral_shard.ShardedGrid) for a model
        step spread over ranks: modal rows of the owned wavenumbers, nodal rows of
        the owned latitude block; ``None`` runs on the equation's full grid."""
        from tornado_gcm_b200.ops import spectral

        self.eq = eq
        self.grid = grid if grid is not None else eq.grid
        self.dt = float(dt)
        self.keys = tuple(tracer_keys)
        self.n = eq.vertical.layers
        self.pre = spectral.explicit_pre_recipe(eq, self.keys, grid=self.grid)
        # the column kernel applies G to the moist tdiff term; the post recipe keeps only ∇²
        self.post = spectral.explicit_post_recipe(eq, self.keys, g_fused=True, grid=self.grid)
        self.spec = ColumnSpec.from_equation(eq, self.keys).with_fused_g()
        if grid is not None and getattr(grid, "sharded", False):
            sl = grid.layout.lat_slice()
            self.spec = dataclasses.replace(self.spec, sec2=np.asarray(self.spec.sec2)[..., sl],
                                            cor=np.asarray(self.spec.cor)[..., sl], _dev={})
        self.ch = spectral.packed_channels(self.n, self.keys)
        self.filter_scaling = np.asarray(filter_scaling, dtype=np.float64)
        self.clamp = float(clamp_abs)
        self._dev: dict = {}
        g = self.grid
        self.L = g.modal_shape[-1]
        self.Lp = (self.L + 3) // 4 * 4

    def _consts(self, device):
        key = str(device)
        d = self._dev.get(key)
        if d is None:
            c = _consts(self.eq)
            base = c.on(device)
            dt = self.dt
            minv = {e: c.minv(e, device) for e in (dt / 6, dt / 3, dt / 4)}
            # l-fastest copies (n*n, L) for the column-parallel stage kernel
            minv_t = {e: m.reshape(m.shape[0], -1).t().contiguous() for e, m in minv.items()}
            filt = torch.as_tensor(self.filter_scaling, dtype=torch.float32, device=device)
            g = self.grid
            oro = self.eq.orography_tendency(device, torch.float32)
            oro = self.eq.grid.clip_wavenumbers(oro)
            if getattr(g, "sharded", False):
                oro = g.layout.scatter_modal(oro)
            packed_oro = torch.zeros(self.ch["C"], *g.modal_shape, dtype=torch.float32, device=device)
            packed_oro[self.n:2 * self.n] = oro
            d = {"base": base, "minv": minv, "minv_t": minv_t, "filt": filt, "oro": packed_oro}
            self._dev[key] = d
        return d

    def orography_packed(self, device) -> torch.Tensor:
        return self._consts(device)["oro"]

    def explicit(self, y: torch.Tensor) -> torch.Tensor:
        from tornado_gcm_b200.ops import spectral

        B = y.shape[0]
        grid = self.grid
        lp = self.Lp if y.is_cuda else self.L
        x_in = spectral.spectral_linear(y, self.pre, out_lpad=lp, grad_lpad=self.L)
        S_in = self.spec.n_in
        nodal = _synth_lat(x_in.reshape(B * S_in, *grid.modal_shape), grid)
        nout = ColumnLatFn.apply(nodal, self.spec, B)
        modal = _anal_lat(nout, grid).reshape(B, self.spec.n_out, *grid.modal_shape)
        return spectral.spectral_linear(modal, self.post, out_lpad=self.L, grad_lpad=lp)

    def _meta(self, device, ce, cp, cg, eta, final):
        d = self._consts(device)
        return {"consts": d["base"], "minv": d["minv"][eta], "minv_t": d["minv_t"][eta],
                "filt": d["filt"] if final else None, "ce": ce,
                "cp": cp, "cg": cg, "eta": eta, "clamp": self.clamp, "R": float(self.eq.R), "final": int(final),
                "n": self.n}

    def step_packed(self, y0: torch.Tensor, P: torch.Tensor) -> torch.Tensor:
        """One substep; ``P`` = packed physics tendency plus the orography term."""
        dt = self.dt
        dev = y0.device
        E0 = self.explicit(y0)
        y1 = StageFn.apply(y0, P, None, E0, None, None, self._meta(dev, [dt / 3], dt / 3, dt / 6, dt / 6, False))
        E1 = self.explicit(y1)
        y2 = StageFn.apply(y0, P, None, E0, E1, None,
                           self._meta(dev, [dt / 6, dt / 2], dt * (1 / 6 + 1 / 2), dt / 3, dt / 3, False))
        E2 = self.explicit(y2)
        y3 = StageFn.apply(y0, P, y2, E0, E1, E2,
                           self._meta(dev, [dt / 2, -dt / 2, dt], dt, 3 * dt / 8, dt / 4, True))
        return y3
