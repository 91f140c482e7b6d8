"""Latitude-sharded spherical-harmonic transforms (the sphere as the "sequence").

Context parallelism for the GCM: nodal fields are split over ranks by
latitude, modal fields stay replicated.  The reference only offers an
all-gather of the nodal field before every transform
(``distributed/dtensor_sharding.py:779-846``); here the transforms work on
the local latitudes directly:

* ``to_nodal`` (modal → local latitudes) needs no communication: each rank
  evaluates the Legendre sums for its own latitude rows only.
* ``to_modal`` (local latitudes → modal) computes the partial quadrature
  sum over the local rows and sums the partials over ranks — one all-reduce
  of the modal field (``(…, 2M-1, L)``, e.g. 1 MB for 32 TL63 levels) instead
  of an all-gather of the nodal field.

With the ``"mirrored"`` partition each rank owns latitude pairs ``(j, J-1-j)``
and the transforms use the equatorial symmetry
``P_l^m(-x) = (-1)^(l+|m|) P_l^m(x)``: the Legendre step runs on the
northern rows only, on even and odd ``l+|m|`` separately, which halves its
flops.  The ``"contiguous"`` partition matches ``torch.chunk`` along the
latitude axis (the DTensor ``Shard`` layout) and uses the plain sums.

Execution paths for ``to_modal`` with several ranks:

* ``fused`` (CUDA, :meth:`enable_fused`): the local transform runs on the
  tcgen05 kernels and the Legendre GEMM's epilogue adds every output value
  straight into all ranks' symmetric output buffers with system-scope
  reductions over NVLink — the cross-GPU sum is fused into the GEMM — followed
  by one peer barrier kernel.  Two output buffers alternate, so a single
  barrier per call orders both the reductions and the re-zeroing.
* ``reducer``: local partial sums, then the peer-memory all-reduce kernel of
  :mod:`tornado_gcm_b200.parallel.fused_allreduce` (``scale=1``);
* otherwise ``torch.distributed.all_reduce`` (the NCCL baseline).

The fused path is forward-only (inference, benchmarks); autograd goes through
the other two.
"""

from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist

PARTITIONS = ("mirrored", "contiguous")


def latitude_partition(latitude_nodes: int, world: int, rank: int, scheme: str = "mirrored") -> np.ndarray:
    """Ascending latitude indices owned by ``rank``.

    ``contiguous``: ``torch.chunk`` semantics (chunks of ``ceil(J/W)`` rows).
    ``mirrored``: the ``J//2`` north/south pairs are chunked the same way and
    each rank owns both rows of its pairs (an odd ``J``'s equator row goes to
    the last rank).
    """
    if scheme not in PARTITIONS:
        raise ValueError(f"unknown latitude partition {scheme!r}; expected one of {PARTITIONS}")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    J = int(latitude_nodes)
    if scheme == "contiguous":
        chunk = -(-J // world)
        return np.arange(min(J, rank * chunk), min(J, (rank + 1) * chunk))
    pairs = J // 2
    chunk = -(-pairs // world)
    north = np.arange(min(pairs, rank * chunk), min(pairs, (rank + 1) * chunk))
    idx = np.concatenate([north, J - 1 - north])
    if J % 2 == 1 and rank == world - 1:
        idx = np.concatenate([idx, [pairs]])
    return np.sort(idx)


def _parity_index(m_abs: np.ndarray, L: int, parity: int) -> np.ndarray:
    """Per-row indices ``l`` with ``(l + |m|) % 2 == parity``, padded with ``L``."""
    n = (L + 1) // 2
    out = np.full((m_abs.size, n), L, dtype=np.int64)
    for r, m in enumerate(m_abs):
        ls = np.arange((m + parity) % 2, L, 2)
        out[r, : ls.size] = ls
    return out


class LatitudeShardedSHT:
    """Transforms between replicated modal fields and this rank's latitude rows."""

    def __init__(self, grid, world: Optional[int] = None, rank: Optional[int] = None, group=None,
                 scheme: str = "mirrored", reducer=None):
        self.grid = grid
        self.group = group
        if world is None:
            world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        if rank is None:
            rank = dist.get_rank(group) if dist.is_available() and dist.is_initialized() else 0
        self.world, self.rank, self.scheme = int(world), int(rank), scheme
        sh = grid.spherical_harmonics
        J = sh.latitude_nodes
        self.lat_index = latitude_partition(J, self.world, self.rank, scheme)
        basis = sh.basis
        self._f = np.asarray(basis.f)                    # (I, M2)
        self._w = np.asarray(basis.w)[self.lat_index]    # (J_loc,)
        p = np.asarray(basis.p)                           # (M2, J, L)
        self.modal_shape = sh.modal_shape
        M2, L = self.modal_shape
        self._mirrored = scheme == "mirrored" and self.lat_index.size > 0
        if self._mirrored:
            lat = np.asarray(sh.nodal_axes[1])
            north = self.lat_index[self.lat_index < J // 2]
            self._north = north
            self._equator = self.lat_index[(self.lat_index == J // 2) & (J % 2 == 1)]
            if not np.allclose(lat[north], -lat[J - 1 - north], atol=1e-12):
                raise ValueError("mirrored partition needs latitude nodes symmetric about the equator")
            pos = {j: i for i, j in enumerate(self.lat_index)}
            self._pos_n = np.array([pos[j] for j in north], dtype=np.int64)
            self._pos_s = np.array([pos[J - 1 - j] for j in north], dtype=np.int64)
            self._pos_e = np.array([pos[j] for j in self._equator], dtype=np.int64)
            m_abs = np.abs(sh.modal_axes[0])
            self._idx_e = _parity_index(m_abs, L, 0)
            self._idx_o = _parity_index(m_abs, L, 1)
            pn = p[:, north, :]
            ppad = np.concatenate([pn, np.zeros((M2, north.size, 1))], axis=-1)
            self._pe = np.take_along_axis(ppad, self._idx_e[:, None, :], axis=-1)   # (M2, Jn, Le)
            self._po = np.take_along_axis(ppad, self._idx_o[:, None, :], axis=-1)
            self._peq = p[:, self._equator, :]                                     # (M2, 0|1, L)
        else:
            self._p = p[:, self.lat_index, :]
        self._cache: dict = {}
        self.reducer = reducer
        self.fused = False

    # ── constants on the device ──
    def _t(self, name: str, device, dtype):
        key = (name, str(device), dtype)
        t = self._cache.get(key)
        if t is None:
            arr = getattr(self, name)
            t = torch.as_tensor(np.ascontiguousarray(arr), device=device,
                                dtype=torch.int64 if arr.dtype.kind == "i" else dtype)
            self._cache[key] = t
        return t

    @property
    def local_latitudes(self) -> int:
        return int(self.lat_index.size)

    def _work_dtype(self, x: torch.Tensor) -> torch.dtype:
        if x.dtype == torch.float64 or self.grid.spherical_harmonics.precision == "highest":
            return torch.float64
        return torch.float32

    # ── modal → local nodal (no communication) ──
    def to_nodal(self, x: torch.Tensor) -> torch.Tensor:
        """``(…, 2M-1, L)`` → ``(…, I, J_local)`` on this rank's latitudes."""
        wd = self._work_dtype(x)
        xd = x.to(wd)
        f = self._t("_f", x.device, wd)
        if not self._mirrored:
            px = torch.einsum("mjl,...ml->...mj", self._t("_p", x.device, wd), xd)
        else:
            xpad = torch.cat([xd, xd.new_zeros(xd.shape[:-1] + (1,))], dim=-1)
            lead = xd.shape[:-2]
            ie = self._t("_idx_e", x.device, wd).expand(lead + self._idx_e.shape)
            io = self._t("_idx_o", x.device, wd).expand(lead + self._idx_o.shape)
            even = torch.einsum("mjk,...mk->...mj", self._t("_pe", x.device, wd), torch.gather(xpad, -1, ie))
            odd = torch.einsum("mjk,...mk->...mj", self._t("_po", x.device, wd), torch.gather(xpad, -1, io))
            px = xd.new_zeros(lead + (self.modal_shape[0], self.local_latitudes))
            px[..., self._pos_n] = even + odd
            px[..., self._pos_s] = even - odd
            if self._pos_e.size:
                px[..., self._pos_e] = torch.einsum("mjl,...ml->...mj", self._t("_peq", x.device, wd), xd)
        return torch.einsum("im,...mj->...ij", f, px).to(x.dtype)

    # ── local nodal → modal ──
    def partial_to_modal(self, nodal_local: torch.Tensor) -> torch.Tensor:
        """This rank's share of the quadrature sum (sum over ranks = ``to_modal``)."""
        wd = self._work_dtype(nodal_local)
        xd = nodal_local.to(wd)
        f = self._t("_f", xd.device, wd)
        g = torch.einsum("im,...ij->...mj", f, xd * self._t("_w", xd.device, wd))   # (…, M2, J_loc)
        if not self._mirrored:
            return torch.einsum("mjl,...mj->...ml", self._t("_p", xd.device, wd), g)
        gn, gs = g[..., self._pos_n], g[..., self._pos_s]
        even = torch.einsum("mjk,...mj->...mk", self._t("_pe", xd.device, wd), gn + gs)
        odd = torch.einsum("mjk,...mj->...mk", self._t("_po", xd.device, wd), gn - gs)
        lead = g.shape[:-2]
        M2, L = self.modal_shape
        out = g.new_zeros(lead + (M2, L + 1))
        out.scatter_(-1, self._t("_idx_e", xd.device, wd).expand(lead + self._idx_e.shape), even)
        out.scatter_add_(-1, self._t("_idx_o", xd.device, wd).expand(lead + self._idx_o.shape), odd)
        out = out[..., :L]
        if self._pos_e.size:
            out = out + torch.einsum("mjl,...mj->...ml", self._t("_peq", xd.device, wd), g[..., self._pos_e])
        return out

    def to_modal(self, nodal_local: torch.Tensor) -> torch.Tensor:
        """``(…, I, J_local)`` on every rank → replicated ``(…, 2M-1, L)``."""
        if self.fused and nodal_local.is_cuda and self.world > 1 and not torch.is_grad_enabled():
            return self.to_modal_fused(nodal_local)
        part = self.partial_to_modal(nodal_local)
        if self.world > 1:
            part = self._all_reduce_sum(part)
        return part.to(nodal_local.dtype)

    def _all_reduce_sum(self, t: torch.Tensor) -> torch.Tensor:
        red = self.reducer
        if red is not None and t.is_cuda and t.dtype == torch.float32 and t.numel() <= red.flat.numel():
            n = t.numel()
            red.flat[:n].copy_(t.reshape(-1))
            if n < red.flat.numel():
                red.flat[n:].zero_()
            red.all_reduce_sum(red.flat)
            return red.flat[:n].view_as(t).clone()
        t = t.contiguous()
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
        return t

    # ── layout helpers ──
    def scatter(self, nodal: torch.Tensor) -> torch.Tensor:
        """Full ``(…, I, J)`` field → this rank's rows (no communication)."""
        return nodal[..., torch.as_tensor(self.lat_index, device=nodal.device)]

    def gather(self, nodal_local: torch.Tensor) -> torch.Tensor:
        """All ranks' rows → the full ``(…, I, J)`` field (all-gather)."""
        if self.world == 1:
            return nodal_local
        J = self.grid.spherical_harmonics.latitude_nodes
        sizes = [latitude_partition(J, self.world, r, self.scheme).size for r in range(self.world)]
        width = max(sizes)
        pad = width - nodal_local.shape[-1]
        loc = torch.nn.functional.pad(nodal_local, (0, pad)).contiguous()
        bufs = [torch.empty_like(loc) for _ in range(self.world)]
        dist.all_gather(bufs, loc, group=self.group)
        out = nodal_local.new_empty(nodal_local.shape[:-1] + (J,))
        for r in range(self.world):
            idx = torch.as_tensor(latitude_partition(J, self.world, r, self.scheme), device=out.device)
            out[..., idx] = bufs[r][..., : sizes[r]]
        return out

    def flops_legendre(self, fields: int) -> int:
        """Multiply-adds of one Legendre step on this rank (for roofline notes)."""
        M2, L = self.modal_shape
        rows = self.local_latitudes / 2 if self._mirrored else self.local_latitudes
        return int(2 * fields * M2 * rows * (math.ceil(L / 2) * 2 if self._mirrored else L))

    # ── fused GPU path ──
    def enable_fused(self, max_fields: int, device) -> None:
        """Allocate the symmetric output buffers and the barrier pad (collective call)."""
        import torch.distributed._symmetric_memory as symm_mem

        from tornado_gcm_b200.ops import _ext
        from tornado_gcm_b200.ops import sht as sht_ops

        _ext.require("fused sharded transform")
        device = torch.device(device)
        sh = self.grid.spherical_harmonics
        M2, L = self.modal_shape
        if self.local_latitudes % 4:
            raise ValueError("the fused path needs a multiple of 4 latitude rows per rank")
        self._Lp = (L + 3) // 4 * 4  # 16-byte rows: the GEMM epilogue adds 4 values per reduction
        self._numel = int(max_fields) * M2 * self._Lp
        group = self.group or dist.group.WORLD
        gname = group.group_name
        self._bufs, self._peer_tabs = [], []
        for _ in range(2):
            b = symm_mem.empty(self._numel, dtype=torch.float32, device=device)
            b.zero_()
            h = symm_mem.rendezvous(b, gname)
            self._bufs.append((b, h))
            self._peer_tabs.append(torch.tensor([int(x) for x in h.buffer_ptrs], dtype=torch.int64))
        pad = symm_mem.empty(2 * 8, dtype=torch.int32, device=device)
        pad.zero_()
        hp = symm_mem.rendezvous(pad, gname)
        self._pad = (pad, hp)
        self._pad_tab = torch.tensor([int(x) for x in hp.buffer_ptrs], dtype=torch.int64)
        self._call = 0
        # bases restricted to this rank's latitude rows
        full = sht_ops.bases(sh, device)
        idx = torch.as_tensor(self.lat_index, device=device)
        self._lb = _LocalBases(full, idx)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)
        self.fused = True

    def to_modal_fused(self, nodal_local: torch.Tensor) -> torch.Tensor:
        """``(…, I, J_local)`` → replicated ``(…, 2M-1, L)`` with the cross-GPU sum in the GEMM epilogue."""
        from tornado_gcm_b200.ops import _ext

        ops = _ext.require("fused sharded transform")
        lead = nodal_local.shape[:-2]
        n3 = nodal_local.reshape((-1,) + tuple(nodal_local.shape[-2:])).float()
        S = n3.shape[0]
        M2, L = self.modal_shape
        Lp = self._Lp
        if S * M2 * Lp > self._numel:
            raise ValueError(f"{S} fields exceed the {self._numel // (M2 * Lp)} reserved by enable_fused")
        k = self._call % 2
        self._call += 1
        buf = self._bufs[k][0]
        lb = self._lb
        ws = _ext.empty(S * lb.M2 * lb.J, dtype=torch.float32, device=n3.device)
        flag = _ext.error_flag(n3.device)
        ops.sht_anal(n3, lb.Ft, lb.Ptw, Lp, ws, None, flag, False, self._peer_tabs[k])
        ops.peer_barrier(self._pad_tab, self.rank, flag, n3.device.index)
        view = buf[: S * M2 * Lp].view(S, M2, Lp)
        out = view[..., :L].contiguous()
        view.zero_()
        return out.reshape(lead + (M2, L)).to(nodal_local.dtype)

    def to_nodal_gpu(self, x: torch.Tensor) -> torch.Tensor:
        """Synthesis on this rank's rows with the tcgen05 kernels (no communication)."""
        from tornado_gcm_b200.ops import _ext

        ops = _ext.require("sharded synthesis")
        lead = x.shape[:-2]
        x3 = x.reshape((-1,) + tuple(x.shape[-2:])).float().contiguous()
        lb = self._lb
        if lb.Lp != lb.L:
            x3 = torch.nn.functional.pad(x3, (0, lb.Lp - lb.L))[..., : lb.L]
        ws = _ext.empty(x3.shape[0] * lb.J * lb.M2p, dtype=torch.float32, device=x3.device)
        out = ops.sht_synth(x3, lb.L, lb.P, lb.F, ws, None, _ext.error_flag(x3.device), False)
        return out.reshape(lead + tuple(out.shape[-2:])).to(x.dtype)


class _LocalBases:
    """The device bases of a grid restricted to a subset of latitude rows."""

    def __init__(self, full, lat_idx: torch.Tensor):
        self.L, self.Lp, self.I, self.M2, self.M2p = full.L, full.Lp, full.I, full.M2, full.M2p
        self.J = int(lat_idx.numel())
        self.P = full.P[:, lat_idx, :].contiguous()
        self.Pt = full.Pt[:, :, lat_idx].contiguous()
        self.Ptw = full.Ptw[:, :, lat_idx].contiguous()
        self.F, self.Ft = full.F, full.Ft

