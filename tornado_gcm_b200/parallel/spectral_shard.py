"""The sphere as the sequence: the spectral model sharded over W ranks.

Behaviour parity: reference ``distributed/dtensor_sharding.py:779-846``
(``SpectralShardingContext``: a latitude-sharded nodal grid with the
spectral transforms crossing ranks) and ``training/trainer.py:184-206`` (the
state bridged through the sharding context during training).  The reference
keeps modal fields replicated and moves whole nodal fields through DTensor
redistributions.  Here both sides are sharded:

* **nodal** fields ``(…, I, J)`` are split into W contiguous latitude blocks
  of ``Jr = J / W`` rows (``Jr`` a multiple of 4);
* **modal** fields ``(…, 2M-1, L)`` are split by zonal wavenumber m: rank r
  holds the rows of the wavenumbers it owns, in a local layout
  ``[m = 0 slot | (cos, sin) rows of each owned m > 0 | zero padding]`` of
  ``M2_loc = 1 + 2·k_max`` rows (the m = 0 slot is a zero row on ranks that
  do not own m = 0).  Wavenumbers are dealt out in a snake order
  (0, 1, …, W-1, W-1, …, 0, 0, 1, …) so the triangular work (L - m per m)
  balances.

Everything spectral — the recipe kernels, the SIL3 stages with the implicit
solve, the filters, the fixer — then works on 1/W of the rows; everything
nodal — the column kernels, the towers, encoder and decoder — on 1/W of
the columns.  The transforms are where the data cross ranks:

* synthesis: rank r runs the Legendre GEMM for its own wavenumbers over ALL
  latitudes; the GEMM epilogue stores every output column j straight into the
  intermediate buffer of the rank that owns latitude j (NVLink peer stores);
  after a peer barrier each rank runs the Fourier GEMM on its block.
* analysis: rank r runs the Fourier GEMM on its block and the Legendre GEMM
  for ALL wavenumbers over its latitudes; the epilogue adds each partial sum
  into the output buffer of the rank that owns the wavenumber (system-scope
  reductions over NVLink), then a peer barrier.

The adjoints are the opposite transforms (synthesis ↔ unweighted analysis,
analysis ↔ quadrature-weighted synthesis), so backward crosses ranks the
same way.  :class:`CollectiveTransforms` computes the same operators with
``torch.distributed`` collectives (all-gather / all-reduce); it runs on any
backend (gloo on CPU for the tests, NCCL as the baseline of the fused path).
"""

from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist

from tornado_gcm_b200.core import spherical_harmonic as sh


def snake_owners(n_items: int, world: int) -> np.ndarray:
    """Owner rank of items 0..n-1 dealt out in snake order (0..W-1, W-1..0, 0..)."""
    own = np.empty(n_items, dtype=np.int64)
    for i in range(n_items):
        rnd, pos = divmod(i, world)
        own[i] = pos if rnd % 2 == 0 else world - 1 - pos
    return own


class ShardLayout:
    """Index maps between the full grid and one rank's shards (pure host data)."""

    def __init__(self, grid: sh.Grid, world: int, rank: int):
        shp = grid.spherical_harmonics
        self.grid = grid
        self.world, self.rank = int(world), int(rank)
        self.Mw = shp.longitude_wavenumbers
        self.L = shp.total_wavenumbers
        self.M2 = 2 * self.Mw - 1
        self.I, self.J = shp.longitude_nodes, shp.latitude_nodes
        if self.J % self.world or (self.J // self.world) % 4:
            raise ValueError(f"{self.J} latitudes do not split into {self.world} blocks of a multiple of 4 rows")
        self.Jr = self.J // self.world
        self.lat0 = self.rank * self.Jr
        self.owner = snake_owners(self.Mw, self.world)
        pos = [[m for m in range(1, self.Mw) if self.owner[m] == r] for r in range(self.world)]
        self.kmax = max(len(p) for p in pos)
        self.G = 1 + self.kmax                  # local groups (slot 0 = m = 0)
        self.M2_loc = 1 + 2 * self.kmax
        self.Lp = (self.L + 3) // 4 * 4
        # per rank: global m of each local group (-1 = empty), global row of each local row
        self.group_m = np.full((self.world, self.G), -1, dtype=np.int32)
        self.rows = np.full((self.world, self.M2_loc), -1, dtype=np.int64)
        self.row_m = np.zeros((self.world, self.M2_loc), dtype=np.int32)
        group_dest = np.zeros(self.Mw, dtype=np.int32)
        for r in range(self.world):
            if self.owner[0] == r:
                self.group_m[r, 0] = 0
                self.rows[r, 0] = 0
            for i, m in enumerate(pos[r]):
                g = i + 1
                self.group_m[r, g] = m
                self.rows[r, 2 * g - 1], self.rows[r, 2 * g] = 2 * m - 1, 2 * m
                self.row_m[r, 2 * g - 1] = self.row_m[r, 2 * g] = m
                group_dest[m] = (r << 16) | g
        group_dest[0] = int(self.owner[0]) << 16
        self.group_dest = group_dest
        self.local_m = [int(m) for m in self.group_m[self.rank] if m >= 0]

    # ── host-side views of the local shards ──
    @property
    def my_rows(self) -> np.ndarray:
        return self.rows[self.rank]

    def lat_slice(self) -> slice:
        return slice(self.lat0, self.lat0 + self.Jr)

    def rows_of(self, a: np.ndarray, rank: Optional[int] = None, fill=0.0) -> np.ndarray:
        """Rows of a full ``(M2, …)`` array in the local layout of ``rank`` (``fill`` in empty rows)."""
        rows = self.rows[self.rank if rank is None else rank]
        out = np.full((self.M2_loc,) + a.shape[1:], fill, dtype=a.dtype)
        ok = rows >= 0
        out[ok] = a[rows[ok]]
        return out

    def scatter_modal(self, x: torch.Tensor, rank: Optional[int] = None) -> torch.Tensor:
        """Full ``(…, M2, L)`` → the local ``(…, M2_loc, L)`` rows (zeros in empty slots)."""
        rows = torch.as_tensor(self.rows[self.rank if rank is None else rank], device=x.device)
        out = x.new_zeros(x.shape[:-2] + (self.M2_loc, x.shape[-1]))
        ok = rows >= 0
        out[..., ok, :] = x[..., rows[ok], :]
        return out

    def place_modal(self, local: torch.Tensor, rank: int, full: torch.Tensor) -> None:
        """Write ``rank``'s local rows into a full ``(…, M2, L)`` tensor."""
        rows = torch.as_tensor(self.rows[rank], device=local.device)
        ok = rows >= 0
        full[..., rows[ok], :] = local[..., ok, :]

    def scatter_nodal(self, x: torch.Tensor) -> torch.Tensor:
        """Full ``(…, I, J)`` → this rank's ``(…, I, Jr)`` block."""
        return x[..., self.lat_slice()]


# ── transform engines ───────────────────────────────────────────────────────
class _Bases:
    """Device bases of the sharded transforms (fp32), built once per device."""

    def __init__(self, lay: ShardLayout, device):
        shp = lay.grid.spherical_harmonics
        p = np.asarray(shp.legendre_table, dtype=np.float64)       # (Mw, J, L)
        w = np.asarray(shp.basis.w, dtype=np.float64)             # (J,)
        f = np.asarray(shp.basis.f, dtype=np.float64)             # (I, M2)
        L, Lp, Jr = lay.L, lay.Lp, lay.Jr
        sl = lay.lat_slice()
        gm = lay.group_m[lay.rank]
        ploc = np.zeros((lay.G, lay.J, Lp))
        for g, m in enumerate(gm):
            if m >= 0:
                ploc[g, :, :L] = p[m]
        t = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float32, device=device)
        self.P_loc = t(ploc)                                       # (G, J, Lp) local wavenumbers
        self.Pw_loc = t(ploc * w[None, :, None])
        pt = np.transpose(p, (0, 2, 1))[:, :, sl]                  # (Mw, L, Jr) local latitudes
        self.Pt_lat = t(pt)
        self.Ptw_lat = t(pt * w[None, None, sl])
        M2p = (lay.M2 + 3) // 4 * 4
        fp = np.zeros((lay.I, M2p))
        fp[:, :lay.M2] = f
        self.F = t(fp)                                             # (I, M2p)
        self.Ft = t(f.T)                                           # (M2, I)
        self.group_m = torch.as_tensor(gm, dtype=torch.int32, device=device)
        self.row_valid = torch.as_tensor((lay.rows[lay.rank] >= 0).astype(np.int32), device=device)
        self.group_dest = torch.as_tensor(lay.group_dest, dtype=torch.int32, device=device)
        # fp64 host-precision copies for the collective engine
        self.p64 = torch.as_tensor(p, dtype=torch.float64, device=device)
        self.p64_lat = torch.as_tensor(np.ascontiguousarray(p[:, sl, :]), dtype=torch.float64, device=device)
        self.w64_lat = torch.as_tensor(w[sl], dtype=torch.float64, device=device)
        self.f64 = torch.as_tensor(f, dtype=torch.float64, device=device)


class CollectiveTransforms:
    """Sharded transforms with ``torch.distributed`` collectives (any backend).

    synthesis: all-gather the modal rows, synthesise this rank's latitudes;
    analysis: partial Legendre sums over this rank's latitudes, all-reduce,
    keep the local rows.  fp32 inputs are transformed in fp32.
    """

    name = "collective"

    def __init__(self, lay: ShardLayout, group=None):
        self.lay = lay
        self.group = group
        self._bases: dict = {}

    def bases(self, device) -> _Bases:
        key = str(device)
        b = self._bases.get(key)
        if b is None:
            b = _Bases(self.lay, device)
            self._bases[key] = b
        return b

    def _gather_full(self, x_loc: torch.Tensor) -> torch.Tensor:
        lay = self.lay
        parts = [torch.empty_like(x_loc) for _ in range(lay.world)]
        dist.all_gather(parts, x_loc.contiguous(), group=self.group)
        full = x_loc.new_zeros(x_loc.shape[:-2] + (lay.M2, x_loc.shape[-1]))
        for r, p in enumerate(parts):
            lay.place_modal(p, r, full)
        return full

    def _reduce_local(self, full: torch.Tensor) -> torch.Tensor:
        full = full.contiguous()
        dist.all_reduce(full, op=dist.ReduceOp.SUM, group=self.group)
        return self.lay.scatter_modal(full)

    def synth(self, x_loc: torch.Tensor, weighted: bool) -> torch.Tensor:
        """(S, M2_loc, L) → (S, I, Jr); ``weighted`` multiplies by the quadrature weights (adjoint of analysis)."""
        b = self.bases(x_loc.device)
        full = self._gather_full(x_loc).to(torch.float64)
        p = b.p64_lat * b.w64_lat[None, :, None] if weighted else b.p64_lat
        # Legendre per m on the (cos, sin) rows, then the real DFT
        m_of_row = torch.as_tensor((np.arange(self.lay.M2) + 1) // 2, device=x_loc.device)
        pr = p[m_of_row]                                            # (M2, Jr, L)
        mid = torch.einsum("mjl,sml->smj", pr, full)
        out = torch.einsum("im,smj->sij", b.f64, mid)
        return out.to(x_loc.dtype)

    def anal(self, n_loc: torch.Tensor, weighted: bool) -> torch.Tensor:
        """(S, I, Jr) → (S, M2_loc, L); ``weighted`` applies the quadrature weights (the forward analysis)."""
        b = self.bases(n_loc.device)
        x = n_loc.to(torch.float64)
        if weighted:
            x = x * b.w64_lat
        mid = torch.einsum("im,sij->smj", b.f64, x)
        m_of_row = torch.as_tensor((np.arange(self.lay.M2) + 1) // 2, device=n_loc.device)
        part = torch.einsum("mjl,smj->sml", b.p64_lat[m_of_row], mid)
        return self._reduce_local(part).to(n_loc.dtype)


class FusedTransforms:
    """Sharded transforms on sm_100a with the transpose fused into the Legendre GEMMs.

    Each rank's intermediate ``W (M2, S·Jr)`` and output ``(S, M2_loc, Lp)``
    buffers live in symmetric memory (two of each, alternating between calls:
    one peer barrier per call then orders both the remote writes of this call
    and the reuse of the other buffer).  Buffers grow on demand; every rank
    calls the transforms in the same order, so the collective re-allocations
    match.  Analysis results are copied out of the shared buffer, which is
    zeroed for its next use.
    """

    name = "fused"

    def __init__(self, lay: ShardLayout, group=None):
        self.lay = lay
        self.group = group or dist.group.WORLD
        self._bases: dict = {}
        self._w = None      # [(tensor, ptr table)] x 2
        self._out = None
        self._w_cap = 0
        self._out_cap = 0
        self._pad = None
        self._pad_tab = None
        self._handles = []
        self._k_w = 0
        self._k_out = 0

    def bases(self, device) -> _Bases:
        key = str(device)
        b = self._bases.get(key)
        if b is None:
            b = _Bases(self.lay, device)
            self._bases[key] = b
        return b

    def _sym(self, numel: int, device, dtype=torch.float32):
        import torch.distributed._symmetric_memory as symm_mem

        t = symm_mem.empty(numel, dtype=dtype, device=device)
        t.zero_()
        h = symm_mem.rendezvous(t, self.group.group_name)
        self._handles.append(h)
        return t, torch.tensor([int(x) for x in h.buffer_ptrs], dtype=torch.int64)

    # analysis destinations hold one slot per source rank (plain peer stores, summed by the owner)
    def _ensure(self, device, w_numel: int, out_numel: int) -> None:
        if self._pad is None:
            self._pad, self._pad_tab = self._sym(2 * 8, device, torch.int32)
        if w_numel > self._w_cap:
            cap = max(w_numel, int(self._w_cap * 1.25))
            self._w = [self._sym(cap, device) for _ in range(2)]
            self._w_cap = cap
        if out_numel > self._out_cap:
            cap = max(out_numel, int(self._out_cap * 1.25))
            self._out = [self._sym(cap * self.lay.world, device) for _ in range(2)]
            self._out_cap = cap
        torch.cuda.synchronize(device)

    def _grow(self, device, w_numel: int = 0, out_numel: int = 0) -> None:
        # every rank makes the same sequence of transform calls, so every rank
        # reaches this collective re-allocation at the same call
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("sharded transform buffers must be sized before CUDA-graph capture "
                               "(run a warm-up step first or call prepare())")
        self._ensure(device, w_numel, out_numel)

    def prepare(self, device, max_slices: int) -> None:
        """Reserve buffers for up to ``max_slices`` fields per call (collective; call on every rank)."""
        lay = self.lay
        self._ensure(torch.device(device), lay.M2 * max_slices * lay.Jr, max_slices * lay.M2_loc * lay.Lp)
        dist.barrier(group=self.group)

    def _barrier(self, device, flag) -> None:
        from tornado_gcm_b200.ops import _ext

        _ext.require("peer barrier").peer_barrier(self._pad_tab, self.lay.rank, flag, device.index)

    def synth(self, x_loc: torch.Tensor, weighted: bool) -> torch.Tensor:
        """(S, M2_loc, L) → (S, Jr, I) latitude-major."""
        from tornado_gcm_b200.ops import _ext

        ops = _ext.require("sharded synthesis")
        lay = self.lay
        dev = x_loc.device
        S = x_loc.shape[0]
        b = self.bases(dev)
        x3 = x_loc.float()
        if not (x3.stride(-1) == 1 and (x3.stride(-2) * 4) % 16 == 0 and (x3.stride(0) * 4) % 16 == 0
                and x3.data_ptr() % 16 == 0):
            x3 = torch.nn.functional.pad(x3, (0, lay.Lp - lay.L)).contiguous()[..., :lay.L]
        if lay.M2 * S * lay.Jr > self._w_cap or self._pad is None:
            self._grow(dev, w_numel=lay.M2 * S * lay.Jr)
        k = self._k_w
        self._k_w ^= 1
        wbuf, wtab = self._w[k]
        flag = _ext.error_flag(dev)
        ops.sht_synth_routed(x3, lay.L, b.Pw_loc if weighted else b.P_loc, b.group_m, wtab, lay.Jr, lay.M2, flag)
        self._barrier(dev, flag)
        return ops.sht_synth_dft(wbuf[: lay.M2 * S * lay.Jr], S, lay.Jr, b.F, flag)

    def anal(self, n_lat: torch.Tensor, weighted: bool) -> torch.Tensor:
        """(S, Jr, I) latitude-major → (S, M2_loc, L)."""
        from tornado_gcm_b200.ops import _ext

        ops = _ext.require("sharded analysis")
        lay = self.lay
        dev = n_lat.device
        S = n_lat.shape[0]
        b = self.bases(dev)
        n = S * lay.M2_loc * lay.Lp
        if n > self._out_cap or self._pad is None:
            self._grow(dev, out_numel=n)
        k = self._k_out
        self._k_out ^= 1
        obuf, otab = self._out[k]
        flag = _ext.error_flag(dev)
        ws = _ext.empty(S * lay.M2 * lay.Jr, dtype=torch.float32, device=dev)
        # this rank's partial sums go into slot `rank` of every owner's buffer (slot stride n)
        ops.sht_anal_routed(n_lat.float().contiguous(), b.Ft, b.Ptw_lat if weighted else b.Pt_lat, lay.Lp,
                            lay.M2_loc, ws, b.group_dest, otab, flag, lay.rank * n)
        self._barrier(dev, flag)
        out = ops.slot_sum(obuf, lay.world, S * lay.M2_loc, lay.Lp, lay.L, b.row_valid)
        return out.view(S, lay.M2_loc, lay.L)


# ── autograd ops ────────────────────────────────────────────────────────────
class _SynthFn(torch.autograd.Function):
    """Sharded synthesis (S, M2_loc, L) → nodal; adjoint = unweighted sharded analysis."""

    @staticmethod
    def forward(ctx, x, eng, lat_major: bool):
        ctx.eng, ctx.lat_major = eng, lat_major
        return _synth_raw(eng, x, False, lat_major)

    @staticmethod
    def backward(ctx, g):
        return _anal_raw(ctx.eng, g, False, ctx.lat_major), None, None


class _AnalFn(torch.autograd.Function):
    """Sharded quadrature-weighted analysis; adjoint = weighted sharded synthesis."""

    @staticmethod
    def forward(ctx, n, eng, lat_major: bool):
        ctx.eng, ctx.lat_major = eng, lat_major
        return _anal_raw(eng, n, True, lat_major)

    @staticmethod
    def backward(ctx, g):
        return _synth_raw(ctx.eng, g, True, ctx.lat_major), None, None


def _synth_raw(eng, x, weighted: bool, lat_major: bool) -> torch.Tensor:
    if isinstance(eng, FusedTransforms):
        out = eng.synth(x, weighted)                    # (S, Jr, I)
        return out if lat_major else out.transpose(-1, -2).contiguous()
    out = eng.synth(x, weighted)                        # (S, I, Jr)
    return out.transpose(-1, -2).contiguous() if lat_major else out


def _anal_raw(eng, n, weighted: bool, lat_major: bool) -> torch.Tensor:
    if isinstance(eng, FusedTransforms):
        nl = n if lat_major else n.transpose(-1, -2)
        return eng.anal(nl.contiguous(), weighted)
    return eng.anal(n.transpose(-1, -2) if lat_major else n, weighted)


# ── the sharded grid ────────────────────────────────────────────────────────
class ShardedGrid:
    """Grid operations on one rank's shards (the subset the model step uses).

    Modal tensors are ``(…, M2_loc, L)`` in the local wavenumber layout,
    nodal tensors ``(…, I, Jr)`` (or ``(…, Jr, I)`` for the latitude-major
    internal layout).  Per-l operators (Laplacian, filters, clipping) act as
    on the full grid; per-row tables (recurrence weights, |m|) are the local
    rows; per-latitude constants are the local block.
    """

    sharded = True

    def __init__(self, grid: sh.Grid, layout: ShardLayout, engine, group=None):
        self.base = grid
        self.layout = layout
        self.engine = engine
        self.group = group
        self.radius = grid.radius
        self.longitude_wavenumbers = grid.longitude_wavenumbers
        self.total_wavenumbers = grid.total_wavenumbers
        self.latitude_spacing = grid.latitude_spacing
        self.precision = "tf32" if isinstance(engine, FusedTransforms) else "float32"
        self._cache: dict = {}

    # ── shapes and tables ──
    @property
    def resolved_precision(self) -> str:
        return self.precision

    def with_precision(self, precision: str) -> "ShardedGrid":
        return self

    @property
    def spherical_harmonics(self):
        return self.base.spherical_harmonics

    @property
    def modal_shape(self):
        return (self.layout.M2_loc, self.layout.L)

    @property
    def nodal_shape(self):
        return (self.layout.I, self.layout.Jr)

    @property
    def mask(self) -> np.ndarray:
        return self.layout.rows_of(np.asarray(self.base.mask), fill=False)

    @property
    def modal_mesh(self):
        m, l = self.base.modal_mesh
        return self.layout.rows_of(m), self.layout.rows_of(l)

    @property
    def laplacian_eigenvalues(self) -> np.ndarray:
        return self.base.laplacian_eigenvalues

    @property
    def cos_lat(self) -> np.ndarray:
        return np.asarray(self.base.cos_lat)[self.layout.lat_slice()]

    @property
    def sec2_lat(self) -> np.ndarray:
        return np.asarray(self.base.sec2_lat)[self.layout.lat_slice()]

    @property
    def latitudes(self) -> np.ndarray:
        return np.asarray(self.base.latitudes)[self.layout.lat_slice()]

    @property
    def longitudes(self) -> np.ndarray:
        return self.base.longitudes

    @property
    def _derivative_recurrence_weights(self):
        a, b = self.base._derivative_recurrence_weights
        return self.layout.rows_of(a), self.layout.rows_of(b)

    def row_wavenumbers(self, device) -> torch.Tensor:
        key = ("row_m", str(device))
        t = self._cache.get(key)
        if t is None:
            t = torch.as_tensor(self.layout.row_m[self.layout.rank], dtype=torch.int32, device=device)
            self._cache[key] = t
        return t

    def const(self, name: str, device, dtype) -> torch.Tensor:
        key = ("const", name, str(device), dtype)
        t = self._cache.get(key)
        if t is None:
            if name in ("cos_lat", "sec2_lat"):
                t = self.base.const(name, device, dtype)[..., self.layout.lat_slice()].contiguous()
            elif name in ("recurrence_a", "recurrence_b", "l"):
                full = self.base.const(name, "cpu", torch.float64).numpy()
                t = torch.as_tensor(self.layout.rows_of(full), dtype=dtype, device=device)
            else:
                t = self.base.const(name, device, dtype)
            self._cache[key] = t
        return t

    # ── transforms ──
    def to_nodal(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-2]
        out = _SynthFn.apply(x.reshape((-1,) + tuple(x.shape[-2:])), self.engine, False)
        return out.reshape(lead + tuple(out.shape[-2:]))

    def to_modal(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-2]
        out = _AnalFn.apply(x.reshape((-1,) + tuple(x.shape[-2:])), self.engine, False)
        return out.reshape(lead + tuple(out.shape[-2:]))

    def to_nodal_lat_major(self, x3: torch.Tensor) -> torch.Tensor:
        return _SynthFn.apply(x3, self.engine, True)

    def to_modal_lat_major(self, n3: torch.Tensor) -> torch.Tensor:
        return _AnalFn.apply(n3, self.engine, True)

    # ── spectral operators (per-l ones as on the full grid) ──
    laplacian = sh.Grid.laplacian
    inverse_laplacian = sh.Grid.inverse_laplacian
    clip_wavenumbers = sh.Grid.clip_wavenumbers
    _l_couple = sh.Grid._l_couple
    cos_lat_d_dlat = sh.Grid.cos_lat_d_dlat
    sec_lat_d_dlat_cos2 = sh.Grid.sec_lat_d_dlat_cos2
    cos_lat_grad = sh.Grid.cos_lat_grad
    k_cross = sh.Grid.k_cross
    div_cos_lat = sh.Grid.div_cos_lat
    curl_cos_lat = sh.Grid.curl_cos_lat

    def d_dlon(self, x: torch.Tensor) -> torch.Tensor:
        """∂/∂λ on the local rows: out[2g-1] = m·x[2g], out[2g] = -m·x[2g-1] (slot 0: zero)."""
        key = ("dlon", str(x.device), x.dtype)
        ent = self._cache.get(key)
        if ent is None:
            n = self.layout.M2_loc
            k = np.arange(n)
            src = np.clip(np.where(k % 2 == 1, k + 1, k - 1), 0, n - 1)
            m = self.layout.row_m[self.layout.rank].astype(np.float64)
            scale = np.where(k % 2 == 1, m, -m)
            scale[0] = 0.0
            ent = (torch.as_tensor(src, device=x.device), torch.as_tensor(scale, dtype=x.dtype, device=x.device))
            self._cache[key] = ent
        src, scale = ent
        return x.index_select(x.ndim - 2, src) * scale.reshape(-1, 1)

    def integrate(self, z: torch.Tensor) -> torch.Tensor:
        """∫ z dΩ over the whole sphere (all-reduce of the local blocks' quadrature sums)."""
        w = torch.as_tensor(self.base.spherical_harmonics.basis.w[self.layout.lat_slice()] * self.radius ** 2,
                            dtype=z.dtype, device=z.device)
        part = torch.einsum("y,...xy->...", w, z).contiguous()
        dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
        return part


def make_sharded_grid(grid: sh.Grid, group=None, engine: str = "auto", device=None) -> ShardedGrid:
    """The sharded view of ``grid`` for this rank of ``group``.

    ``engine``: ``fused`` (NVLink transport: routed Legendre epilogues),
    ``collective`` (NCCL on CUDA, gloo on the CPU), a transport name, or
    ``auto`` (:func:`tornado_gcm_b200.parallel.transport.get_transport`).
    """
    from tornado_gcm_b200.parallel.transport import get_transport

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    lay = ShardLayout(grid, world, rank)
    kind = {"fused": "nvlink", "collective": "gloo" if device is None or torch.device(device).type == "cpu"
            else "nccl"}.get(engine, engine)
    eng = get_transport(kind, group, device).spectral_engine(lay)
    return ShardedGrid(grid, lay, eng, group)


# ── conservation fixer across wavenumber shards ──────────────────────────────
class ShardedPackedFixFn(torch.autograd.Function):
    """The packed FP64 fixer with its energy sums and deficit cotangent reduced over the ranks.

    The energy proxy sums over every modal row, so the per-rank partial sums
    are added (an all-reduce of a (B, 64, 2) fp64 array) before the
    correction; the (0,0) modes live on the owner of m = 0, whose deficit
    cotangent is likewise all-reduced (the other ranks contribute zero).
    """

    @staticmethod
    def forward(ctx, y, y_before, n: int, fix_mass: bool, fix_energy: int, group):
        from tornado_gcm_b200.ops import _ext

        ops = _ext.require("conservation fixer")
        y = y.contiguous()
        y_before = y_before.contiguous()
        part = ops.packed_fix_partial(y, y_before, n, fix_mass, fix_energy)
        dist.all_reduce(part, op=dist.ReduceOp.SUM, group=group)
        out, _ = ops.packed_fix(y, y_before, n, fix_mass, fix_energy, part)
        ctx.save_for_backward(y, y_before, part)
        ctx.cfg = (n, fix_mass, fix_energy, group)
        return out

    @staticmethod
    def backward(ctx, gout):
        from tornado_gcm_b200.ops import _ext

        y, yb, part = ctx.saved_tensors
        n, fm, fe, group = ctx.cfg
        ops = _ext.require("conservation fixer adjoint")
        gout = gout.contiguous()
        gd = _deficit_cotangent(gout, y, part, n, fe)
        dist.all_reduce(gd, op=dist.ReduceOp.SUM, group=group)
        need_b = ctx.needs_input_grad[1]
        res = ops.packed_fix_adjoint(gout, y, yb, part, n, fm, fe, need_b, gd)
        return res[0], (res[1] if need_b else None), None, None, None, None


def _deficit_cotangent(gout, y, part, n: int, fix_energy: int) -> torch.Tensor:
    """Per-sample cotangent of the raw energy deficit from this rank's (0,0) temperature modes.

    Zero on ranks without m = 0 (their slot-0 rows are zero, and sign(0) = 0).
    """
    B = y.shape[0]
    if not fix_energy:
        return torch.zeros(B, dtype=torch.float64, device=y.device)
    dscale = 1.0 / n if fix_energy == 2 else 1.0
    tot = part.sum(dim=1)                                   # (B, 2)
    D = (tot[:, 1] - tot[:, 0]) * dscale                    # (B,)
    t = y[:, 2 * n:3 * n, 0, 0].double()                    # (B, n)
    g = gout[:, 2 * n:3 * n, 0, 0].double()
    s = torch.sqrt(torch.clamp(t * t + D[:, None], min=0.0))
    ok = ((t * t + D[:, None]) > 0).all(dim=1, keepdim=True)
    terms = torch.where(s > 0, g * torch.sign(t) / (2.0 * torch.where(s > 0, s, torch.ones_like(s))),
                        torch.zeros_like(s))
    return (torch.where(ok, terms, torch.zeros_like(terms)).sum(dim=1) * dscale).contiguous()


def sharded_packed_fix(y, y_before, n: int, group, fix_mass=True, fix_energy=True, energy_split="levels"):
    from tornado_gcm_b200.ops.fixers import ENERGY_SPLIT

    if not (fix_mass or fix_energy):
        return y
    mode = ENERGY_SPLIT[energy_split] if fix_energy else 0
    return ShardedPackedFixFn.apply(y, y_before, int(n), bool(fix_mass), mode, group)


@dataclasses.dataclass
class ShardContext:
    """What a latitude/wavenumber-sharded model needs at run time."""

    grid: ShardedGrid
    group: object
    world: int
    rank: int

    @property
    def layout(self) -> ShardLayout:
        return self.grid.layout


def shard_hybrid_gcm(gcm, group=None, engine: str = "auto"):
    """Spread a :class:`~tornado_gcm_b200.models.builders.HybridGCM` over the ranks of ``group``.

    Weights stay replicated; every spectral field keeps the rows of this
    rank's wavenumbers and every nodal field this rank's latitude block.  The
    model then takes latitude blocks of the data (:func:`scatter_fields`),
    its loss is this rank's share of the global loss (``loss_scale = 1/W``),
    and the weight gradients are summed over the ranks after backward
    (``GCMTrainer(data_parallel=True, grad_average=False)``).
    """
    dev = next(gcm.parameters()).device
    base = gcm.model.config.coords.horizontal
    sgrid = make_sharded_grid(base, group, engine, dev)
    ctx = ShardContext(sgrid, group, sgrid.layout.world, sgrid.layout.rank)
    m = gcm.model
    m.shard = ctx
    m._fused = None
    p = m.parameterization
    if p is not None and hasattr(p, "grid"):
        p.grid = sgrid
        for k in ("_recipes", "_latf2d"):
            p.__dict__.pop(k, None)
    for codec in (gcm.encoder, gcm.decoder):
        if hasattr(codec, "grid"):
            codec.grid = sgrid
    gcm.loss_scale = 1.0 / ctx.world
    gcm.shard = ctx
    return gcm


def scatter_fields(fields: dict, ctx: ShardContext) -> dict:
    """This rank's latitude block of every nodal field ``(…, I, J)`` of a dict."""
    sl = ctx.layout.lat_slice()
    return {k: v[..., sl].contiguous() for k, v in fields.items()}
