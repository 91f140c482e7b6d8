"""Real spherical harmonics, the ``Grid`` and spectral differential operators.

Public behaviour follows reference ``core/spherical_harmonic.py:100-634``:

* nodal arrays are ``(..., lon, lat)``; modal arrays are ``(..., 2M-1, L)``
  with the longitudinal-wavenumber axis ordered ``[0, +1, -1, +2, -2, ...]``
  (``+m`` = cosine, ``-m`` = sine) and total wavenumber ``l`` on the last axis;
* ``to_nodal`` = Legendre synthesis (sum over l per m) followed by the real
  DFT synthesis; ``to_modal`` = quadrature-weighted DFT analysis followed by
  Legendre analysis.

What differs from the reference (by design):

* the FP64 bases are built once per grid and kept resident per device
  (the reference re-uploads P and F on every transform);
* the transform precision is an explicit grid attribute (``precision`` =
  ``"highest"`` | ``"float32"`` | ``"tf32"``) so that the PZHA policy's
  ``sht_adaptive_threshold`` is honoured instead of a hard-wired 42;
* on CUDA tensors the transforms run in the sm_100a kernels of
  :mod:`tornado_gcm_b200.ops.sht` (tcgen05 Legendre/DFT GEMMs); on CPU they
  run as FP64/FP32 ``torch`` contractions, which is the numerical oracle.
"""

from __future__ import annotations

import dataclasses
import functools
import math
from typing import Any, Callable, Optional

import numpy as np
import torch

from tornado_gcm_b200.core import fourier, legendre

_CONSTANT_NORMALIZATION_FACTOR = 3.5449077  # sqrt(4π): Y_00 normalisation

_PRECISIONS = ("highest", "float32", "tf32")


def einsum_highest(subscripts: str, *operands: torch.Tensor) -> torch.Tensor:
    """FP64 einsum; result cast to the promoted dtype of non-basis operands."""
    out_dtype = operands[-1].dtype
    res = torch.einsum(subscripts, *[o.to(torch.float64) for o in operands])
    return res.to(out_dtype) if out_dtype != torch.float64 else res


def einsum_adaptive(subscripts: str, *operands: torch.Tensor) -> torch.Tensor:
    return torch.einsum(subscripts, *[o.to(torch.float32) for o in operands])


def sht_precision_for(total_wavenumbers: int, threshold: int = 42) -> str:
    """Resolution-adaptive transform precision: ≤threshold → FP32/TF32, else FP64."""
    return "float32" if total_wavenumbers <= threshold else "highest"


def get_sht_einsum(total_wavenumbers: int, threshold: int = 42):
    return einsum_adaptive if total_wavenumbers <= threshold else einsum_highest


LATITUDE_SPACINGS = legendre.LATITUDE_SPACINGS
get_latitude_nodes = legendre.get_latitude_nodes


@dataclasses.dataclass
class _SphericalHarmonicBasis:
    f: np.ndarray  # (I, 2M-1) Fourier synthesis matrix
    p: np.ndarray  # (2M-1, J, L) Legendre table, rows duplicated for ±m
    w: np.ndarray  # (J,) combined Fourier x Gauss quadrature weights


class _DeviceCache:
    """Per-(device, dtype) resident copies of the basis tensors."""

    def __init__(self):
        self._store: dict[tuple, torch.Tensor] = {}

    def get(self, key, builder):
        t = self._store.get(key)
        if t is None:
            t = builder()
            self._store[key] = t
        return t


@dataclasses.dataclass(frozen=True)
class RealSphericalHarmonics:
    longitude_wavenumbers: int = 0
    total_wavenumbers: int = 0
    longitude_nodes: int = 0
    latitude_nodes: int = 0
    latitude_spacing: str = "gauss"
    precision: str = "highest"
    einsum_fn: Any = None  # compatibility hook: forces a specific CPU einsum

    def __post_init__(self):
        if self.precision not in _PRECISIONS:
            raise ValueError(f"precision must be one of {_PRECISIONS}")
        object.__setattr__(self, "_cache", _DeviceCache())

    @functools.cached_property
    def nodal_axes(self):
        lon, _ = fourier.quadrature_nodes(self.longitude_nodes)
        sin_lat, _ = get_latitude_nodes(self.latitude_nodes, self.latitude_spacing)
        return lon, sin_lat

    @property
    def nodal_shape(self):
        return (self.longitude_nodes, self.latitude_nodes)

    @property
    def nodal_padding(self):
        return (0, 0)

    @functools.cached_property
    def modal_axes(self):
        m_pos = np.arange(1, self.longitude_wavenumbers)
        lon_wn = np.concatenate([[0], np.stack([m_pos, -m_pos], axis=1).ravel()])
        return lon_wn, np.arange(self.total_wavenumbers)

    @property
    def modal_shape(self):
        return (2 * self.longitude_wavenumbers - 1, self.total_wavenumbers)

    @property
    def modal_padding(self):
        return (0, 0)

    @property
    def modal_dtype(self):
        return np.dtype(np.float32)

    @functools.cached_property
    def mask(self) -> np.ndarray:
        m, l = np.meshgrid(*self.modal_axes, indexing="ij")
        return abs(m) <= l

    @functools.cached_property
    def legendre_table(self) -> np.ndarray:
        """Distinct-|m| Legendre table (M, J, L) in FP64."""
        x, _ = get_latitude_nodes(self.latitude_nodes, self.latitude_spacing)
        return legendre.evaluate(self.longitude_wavenumbers, self.total_wavenumbers, x)

    @functools.cached_property
    def basis(self) -> _SphericalHarmonicBasis:
        f = fourier.real_basis(self.longitude_wavenumbers, self.longitude_nodes)
        _, wf = fourier.quadrature_nodes(self.longitude_nodes)
        _, wp = get_latitude_nodes(self.latitude_nodes, self.latitude_spacing)
        p = self.legendre_table
        m_of_row = np.abs(self.modal_axes[0])
        return _SphericalHarmonicBasis(f=f, p=p[m_of_row], w=wf * wp)

    def device_basis(self, name: str, device, dtype=torch.float64) -> torch.Tensor:
        device = torch.device(device)

        def build():
            arr = getattr(self.basis, name)
            return torch.as_tensor(np.ascontiguousarray(arr), dtype=dtype, device=device)

        return self._cache.get((name, str(device), dtype), build)

    # ── transforms ────────────────────────────────────────────────────
    def _cpu_dtype(self, x: torch.Tensor) -> torch.dtype:
        if self.precision == "highest" or x.dtype == torch.float64:
            return torch.float64
        return torch.float32

    def inverse_transform(self, x: torch.Tensor) -> torch.Tensor:
        """Modal (…, 2M-1, L) → nodal (…, I, J)."""
        if x.is_cuda and self.einsum_fn is None:
            from tornado_gcm_b200.ops import sht as sht_ops

            return sht_ops.to_nodal(x, self)
        if self.einsum_fn is not None:
            p = self.device_basis("p", x.device)
            f = self.device_basis("f", x.device)
            px = self.einsum_fn("mjl,...ml->...mj", p, x)
            return self.einsum_fn("im,...mj->...ij", f, px)
        wd = self._cpu_dtype(x)
        p = self.device_basis("p", x.device, wd)
        f = self.device_basis("f", x.device, wd)
        px = torch.einsum("mjl,...ml->...mj", p, x.to(wd))
        out = torch.einsum("im,...mj->...ij", f, px)
        return out.to(x.dtype)

    def transform(self, x: torch.Tensor) -> torch.Tensor:
        """Nodal (…, I, J) → modal (…, 2M-1, L)."""
        if x.is_cuda and self.einsum_fn is None:
            from tornado_gcm_b200.ops import sht as sht_ops

            return sht_ops.to_modal(x, self)
        if self.einsum_fn is not None:
            w = self.device_basis("w", x.device, x.dtype)
            p = self.device_basis("p", x.device)
            f = self.device_basis("f", x.device)
            fwx = self.einsum_fn("im,...ij->...mj", f, w * x)
            return self.einsum_fn("mjl,...mj->...ml", p, fwx)
        wd = self._cpu_dtype(x)
        w = self.device_basis("w", x.device, wd)
        p = self.device_basis("p", x.device, wd)
        f = self.device_basis("f", x.device, wd)
        fwx = torch.einsum("im,...ij->...mj", f, x.to(wd) * w)
        out = torch.einsum("mjl,...mj->...ml", p, fwx)
        return out.to(x.dtype)

    def longitudinal_derivative(self, x: torch.Tensor) -> torch.Tensor:
        return fourier.real_basis_derivative(x, axis=-2)


SphericalHarmonicsImpl = Callable[..., RealSphericalHarmonics]


@dataclasses.dataclass(frozen=True)
class Grid:
    """Nodal/spectral grids on the sphere plus spectral operators."""

    longitude_wavenumbers: int = 0
    total_wavenumbers: int = 0
    longitude_nodes: int = 0
    latitude_nodes: int = 0
    latitude_spacing: str = "gauss"
    longitude_offset: float = 0.0
    radius: float = 1.0
    spherical_harmonics_impl: SphericalHarmonicsImpl = RealSphericalHarmonics
    precision: Optional[str] = None  # None → resolution-adaptive (threshold 42)

    def __post_init__(self):
        if self.radius is None:
            object.__setattr__(self, "radius", 1.0)
        if self.latitude_spacing not in LATITUDE_SPACINGS:
            raise ValueError(
                f'Unsupported latitude_spacing "{self.latitude_spacing}". '
                f"Supported: {list(LATITUDE_SPACINGS)}."
            )
        if self.precision is not None and self.precision not in _PRECISIONS:
            raise ValueError(f"precision must be one of {_PRECISIONS}")

    # ── factories ──────────────────────────────────────────────────────
    @classmethod
    def with_wavenumbers(cls, longitude_wavenumbers: int, dealiasing: str = "quadratic",
                         latitude_spacing: str = "gauss", longitude_offset: float = 0.0,
                         spherical_harmonics_impl=RealSphericalHarmonics, radius: float = 1.0,
                         precision: Optional[str] = None) -> "Grid":
        order = {"linear": 2, "quadratic": 3, "cubic": 4}[dealiasing]
        lon_nodes = order * longitude_wavenumbers + 1
        return cls(longitude_wavenumbers, longitude_wavenumbers + 1, lon_nodes,
                   math.ceil(lon_nodes / 2), latitude_spacing, longitude_offset, radius,
                   spherical_harmonics_impl, precision)

    @classmethod
    def construct(cls, max_wavenumber: int, gaussian_nodes: int, latitude_spacing: str = "gauss",
                  longitude_offset: float = 0.0, radius: float = 1.0,
                  spherical_harmonics_impl=RealSphericalHarmonics,
                  precision: Optional[str] = None) -> "Grid":
        return cls(max_wavenumber + 1, max_wavenumber + 2, 4 * gaussian_nodes, 2 * gaussian_nodes,
                   latitude_spacing, longitude_offset, radius, spherical_harmonics_impl, precision)

    @classmethod
    def T21(cls, **kw): return cls.construct(21, 16, **kw)
    @classmethod
    def T31(cls, **kw): return cls.construct(31, 24, **kw)
    @classmethod
    def T42(cls, **kw): return cls.construct(42, 32, **kw)
    @classmethod
    def T85(cls, **kw): return cls.construct(85, 64, **kw)
    @classmethod
    def T106(cls, **kw): return cls.construct(106, 80, **kw)
    @classmethod
    def T119(cls, **kw): return cls.construct(119, 90, **kw)
    @classmethod
    def T170(cls, **kw): return cls.construct(170, 128, **kw)
    @classmethod
    def T213(cls, **kw): return cls.construct(213, 160, **kw)
    @classmethod
    def T340(cls, **kw): return cls.construct(340, 256, **kw)
    @classmethod
    def T425(cls, **kw): return cls.construct(425, 320, **kw)
    @classmethod
    def TL31(cls, **kw): return cls.construct(31, 16, **kw)
    @classmethod
    def TL47(cls, **kw): return cls.construct(47, 24, **kw)
    @classmethod
    def TL63(cls, **kw): return cls.construct(63, 32, **kw)
    @classmethod
    def TL95(cls, **kw): return cls.construct(95, 48, **kw)
    @classmethod
    def TL127(cls, **kw): return cls.construct(127, 64, **kw)
    @classmethod
    def TL159(cls, **kw): return cls.construct(159, 80, **kw)
    @classmethod
    def TL179(cls, **kw): return cls.construct(179, 90, **kw)
    @classmethod
    def TL255(cls, **kw): return cls.construct(255, 128, **kw)
    @classmethod
    def TL511(cls, **kw): return cls.construct(511, 256, **kw)
    @classmethod
    def TL639(cls, **kw): return cls.construct(639, 320, **kw)
    @classmethod
    def TL1279(cls, **kw): return cls.construct(1279, 640, **kw)

    # ── precision / impl ──────────────────────────────────────────────
    @property
    def resolved_precision(self) -> str:
        if self.precision is not None:
            return self.precision
        return sht_precision_for(self.total_wavenumbers)

    def with_precision(self, precision: str) -> "Grid":
        return dataclasses.replace(self, precision=precision)

    def with_einsum(self, einsum_fn) -> "Grid":
        """Grid whose CPU/GPU transforms go through ``einsum_fn`` (compat hook)."""
        if einsum_fn is einsum_highest:
            return self.with_precision("highest")
        return dataclasses.replace(
            self,
            spherical_harmonics_impl=functools.partial(self.spherical_harmonics_impl, einsum_fn=einsum_fn),
        )

    @functools.cached_property
    def spherical_harmonics(self) -> RealSphericalHarmonics:
        return self.spherical_harmonics_impl(
            longitude_wavenumbers=self.longitude_wavenumbers,
            total_wavenumbers=self.total_wavenumbers,
            longitude_nodes=self.longitude_nodes,
            latitude_nodes=self.latitude_nodes,
            latitude_spacing=self.latitude_spacing,
            precision=self.resolved_precision,
        )

    # ── axes ──────────────────────────────────────────────────────────
    @property
    def longitudes(self) -> np.ndarray:
        return self.nodal_axes[0]

    @property
    def latitudes(self) -> np.ndarray:
        return np.arcsin(self.nodal_axes[1])

    @functools.cached_property
    def nodal_axes(self):
        lon, sin_lat = self.spherical_harmonics.nodal_axes
        return lon + self.longitude_offset, sin_lat

    @property
    def nodal_shape(self):
        return self.spherical_harmonics.nodal_shape

    @property
    def nodal_padding(self):
        return (0, 0)

    @functools.cached_property
    def nodal_mesh(self):
        return np.meshgrid(*self.nodal_axes, indexing="ij")

    @property
    def modal_axes(self):
        return self.spherical_harmonics.modal_axes

    @property
    def modal_shape(self):
        return self.spherical_harmonics.modal_shape

    @property
    def modal_padding(self):
        return (0, 0)

    @property
    def mask(self) -> np.ndarray:
        return self.spherical_harmonics.mask

    @functools.cached_property
    def modal_mesh(self):
        return np.meshgrid(*self.modal_axes, indexing="ij")

    @functools.cached_property
    def cos_lat(self) -> np.ndarray:
        return np.sqrt(1 - self.nodal_axes[1] ** 2)

    @functools.cached_property
    def sec2_lat(self) -> np.ndarray:
        return 1 / (1 - self.nodal_axes[1] ** 2)

    @functools.cached_property
    def laplacian_eigenvalues(self) -> np.ndarray:
        l = self.modal_axes[1]
        return -l * (l + 1) / (self.radius**2)

    # ── device constants (cached) ─────────────────────────────────────
    def const(self, name: str, device, dtype) -> torch.Tensor:
        """Resident device copy of a per-grid numpy constant."""
        cache = self.spherical_harmonics._cache
        device = torch.device(device)

        def build():
            if name == "inv_laplacian":
                eig = self.laplacian_eigenvalues.astype(np.float64)
                inv = np.zeros_like(eig)
                inv[1:] = 1.0 / eig[1:]
                arr = inv
            elif name == "recurrence_a":
                arr = self._derivative_recurrence_weights[0]
            elif name == "recurrence_b":
                arr = self._derivative_recurrence_weights[1]
            elif name == "l":
                arr = self.modal_mesh[1].astype(np.float64)
            elif name.startswith("clip_mask_"):
                k = int(name.rsplit("_", 1)[1])
                arr = np.ones(self.modal_shape[-1])
                arr[-k:] = 0.0
            else:
                arr = getattr(self, name)
            return torch.as_tensor(np.ascontiguousarray(arr), dtype=dtype, device=device)

        return cache.get(("const", name, str(device), dtype), build)

    # ── transforms ────────────────────────────────────────────────────
    def to_nodal(self, x: torch.Tensor) -> torch.Tensor:
        return self.spherical_harmonics.inverse_transform(x)

    def to_modal(self, x: torch.Tensor) -> torch.Tensor:
        return self.spherical_harmonics.transform(x)

    # ── spectral operators ────────────────────────────────────────────
    def laplacian(self, x: torch.Tensor) -> torch.Tensor:
        return x * self.const("laplacian_eigenvalues", x.device, x.dtype)

    def inverse_laplacian(self, x: torch.Tensor) -> torch.Tensor:
        return x * self.const("inv_laplacian", x.device, x.dtype)

    def clip_wavenumbers(self, x, n: int = 1):
        if n <= 0:
            raise ValueError(f"n must be >= 0; got {n}.")

        def clip_fn(t):
            if not isinstance(t, torch.Tensor):
                return t
            return t * self.const(f"clip_mask_{n}", t.device, t.dtype)

        if isinstance(x, tuple):
            return tuple(clip_fn(xi) for xi in x)
        return clip_fn(x)

    @functools.cached_property
    def _derivative_recurrence_weights(self):
        m, l = self.modal_mesh
        mask = self.mask.astype(np.float64)
        with np.errstate(divide="ignore", invalid="ignore"):
            a = np.sqrt(np.where(mask > 0, (l**2 - m**2) / (4.0 * l**2 - 1.0), 0.0))
            b = np.sqrt(np.where(mask > 0, ((l + 1) ** 2 - m**2) / (4.0 * (l + 1) ** 2 - 1.0), 0.0))
        a[:, 0] = 0
        b[:, -1] = 0
        return np.nan_to_num(a), np.nan_to_num(b)

    def _l_couple(self, x: torch.Tensor, up_coef: torch.Tensor, down_coef: torch.Tensor) -> torch.Tensor:
        """out[l] = up_coef[l+1]·x[l+1] + down_coef[l-1]·x[l-1] (zero outside)."""
        y_up = up_coef * x
        y_dn = down_coef * x
        out = torch.zeros_like(x)
        out[..., :-1] = y_up[..., 1:]
        out[..., 1:] = out[..., 1:] + y_dn[..., :-1]
        return out

    def d_dlon(self, x: torch.Tensor) -> torch.Tensor:
        return self.spherical_harmonics.longitudinal_derivative(x)

    def cos_lat_d_dlat(self, x: torch.Tensor) -> torch.Tensor:
        """cosθ ∂x/∂θ: out[l] = (l+2)a[l+1]x[l+1] - (l-1)b[l-1]x[l-1]."""
        a = self.const("recurrence_a", x.device, x.dtype)
        b = self.const("recurrence_b", x.device, x.dtype)
        l = self.const("l", x.device, x.dtype)
        return self._l_couple(x, (l + 1) * a, -l * b)

    def sec_lat_d_dlat_cos2(self, x: torch.Tensor) -> torch.Tensor:
        """secθ ∂(cos²θ x)/∂θ: out[l] = l·a[l+1]x[l+1] - (l+1)b[l-1]x[l-1]."""
        a = self.const("recurrence_a", x.device, x.dtype)
        b = self.const("recurrence_b", x.device, x.dtype)
        l = self.const("l", x.device, x.dtype)
        return self._l_couple(x, (l - 1) * a, -(l + 2) * b)

    def cos_lat_grad(self, x: torch.Tensor, clip: bool = True):
        raw = (self.d_dlon(x) / self.radius, self.cos_lat_d_dlat(x) / self.radius)
        return self.clip_wavenumbers(raw) if clip else raw

    def k_cross(self, v):
        return (-v[1], v[0])

    def div_cos_lat(self, v, clip: bool = True) -> torch.Tensor:
        raw = (self.d_dlon(v[0]) + self.sec_lat_d_dlat_cos2(v[1])) / self.radius
        return self.clip_wavenumbers(raw) if clip else raw

    def curl_cos_lat(self, v, clip: bool = True) -> torch.Tensor:
        raw = (self.d_dlon(v[1]) - self.sec_lat_d_dlat_cos2(v[0])) / self.radius
        return self.clip_wavenumbers(raw) if clip else raw

    @property
    def quadrature_weights(self) -> np.ndarray:
        return np.broadcast_to(self.spherical_harmonics.basis.w, self.nodal_shape)

    def integrate(self, z: torch.Tensor) -> torch.Tensor:
        w = torch.as_tensor(self.spherical_harmonics.basis.w * self.radius**2, dtype=z.dtype, device=z.device)
        return torch.einsum("y,...xy->...", w, z)


def add_constant(x: torch.Tensor, c: float) -> torch.Tensor:
    x = x.clone()
    x[..., 0, 0] = x[..., 0, 0] + _CONSTANT_NORMALIZATION_FACTOR * c
    return x


def get_cos_lat_vector(vorticity, divergence, grid: Grid, clip: bool = True):
    """cosθ·(u, v) from vorticity/divergence via stream function & potential."""
    psi = grid.inverse_laplacian(vorticity)
    chi = grid.inverse_laplacian(divergence)
    gchi = grid.cos_lat_grad(chi, clip=clip)
    kpsi = grid.k_cross(grid.cos_lat_grad(psi, clip=clip))
    return (gchi[0] + kpsi[0], gchi[1] + kpsi[1])


def uv_nodal_to_vor_div_modal(grid: Grid, u_nodal, v_nodal, clip: bool = True):
    cos_lat = grid.const("cos_lat", u_nodal.device, u_nodal.dtype)
    um = grid.to_modal(u_nodal / cos_lat)
    vm = grid.to_modal(v_nodal / cos_lat)
    return grid.curl_cos_lat((um, vm), clip=clip), grid.div_cos_lat((um, vm), clip=clip)


def vor_div_to_uv_nodal(grid: Grid, vorticity, divergence, clip: bool = True):
    uc, vc = get_cos_lat_vector(vorticity, divergence, grid, clip=clip)
    cos_lat = grid.const("cos_lat", uc.device, uc.dtype)
    return grid.to_nodal(uc) / cos_lat, grid.to_nodal(vc) / cos_lat
