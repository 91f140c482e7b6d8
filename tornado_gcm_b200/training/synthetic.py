"""Synthetic reanalysis-shaped data for benchmarks and tests.

Fields follow the benchmark specification: each field is a level-mean
profile plus noise band-limited to total wavenumber ≤ 21 (generated in
spectral space and synthesised on the grid):

* T: 200–300 K profile, noise σ = 5 K;  u, v: 10 m/s rms, mostly rotational
  (divergence 10 % of vorticity in spectral amplitude);  the T, z and wind
  anomalies are vertically coherent (one horizontal pattern per sample, wind
  amplitude growing with height), so columns keep the statically stable mean
  lapse rate and a Richardson number far above 1/4 — independent noise per
  level made ~18 % of adjacent level pairs convectively unstable, which a
  dry dynamical core amplifies at the grid scale;
* q: lognormal in (0, 0.02] kg/kg;  z: hydrostatic 0–4.8e5 m²/s²;
* cloud liquid / ice: lognormal ≤ 1e-4;
* forcings: SST 271–305 K, sea ice U[0, 1], orography 0–3.5 km rising
  smoothly from the coast of the binary land mask.

Everything is deterministic given the seed.  Fields are returned in
physical units on ``(..., levels, lon, lat)`` nodal grids, plus
normalised versions for the network inputs.
"""

from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np
import torch

from tornado_gcm_b200.core.spherical_harmonic import Grid

DATA_FIELDS = ("u", "v", "t", "q", "z", "clwc", "ciwc")
FORCING_FIELDS = ("sea_surface_temperature", "sea_ice_cover", "orography", "land_sea_mask")
PRESSURE_LEVELS_37 = np.array([1, 2, 3, 5, 7, 10, 20, 30, 50, 70, 100, 125, 150, 175, 200, 225, 250, 300, 350, 400,
                               450, 500, 550, 600, 650, 700, 750, 775, 800, 825, 850, 875, 900, 925, 950, 975, 1000],
                              dtype=np.float64)


def band_limited_noise(grid: Grid, n_fields: int, lmax: int, rng: np.random.Generator, batch: int = 1) -> np.ndarray:
    """Unit-variance nodal noise with spectral support l ≤ lmax, shape (batch, n_fields, I, J)."""
    m, l = grid.modal_mesh
    amp = np.where(grid.mask & (l <= lmax) & (l > 0), 1.0, 0.0)
    coef = rng.standard_normal((batch, n_fields) + grid.modal_shape) * amp
    nodal = torch.einsum("im,...mj->...ij", torch.as_tensor(grid.spherical_harmonics.basis.f),
                         torch.einsum("mjl,...ml->...mj", torch.as_tensor(grid.spherical_harmonics.basis.p),
                                      torch.as_tensor(coef))).numpy()
    std = nodal.std(axis=(-2, -1), keepdims=True) + 1e-12
    return nodal / std


def rotational_winds(grid: Grid, n_fields: int, lmax: int, rng: np.random.Generator, batch: int = 1,
                     speed: float = 10.0, divergent_fraction: float = 0.1) -> tuple[np.ndarray, np.ndarray]:
    """Band-limited (u, v) that are mostly rotational, like the real atmosphere.

    Vorticity and divergence are drawn in spectral space (support
    ``1 ≤ l ≤ lmax``, divergence ``divergent_fraction`` as large), turned into
    winds through the stream function and velocity potential, and scaled so
    each level's wind components have standard deviation ``speed``.
    Independent u and v noise would carry as much divergence as vorticity,
    which excites gravity waves far beyond observed amplitudes.
    """
    from tornado_gcm_b200.core.spherical_harmonic import get_cos_lat_vector

    g = grid.with_precision("highest")
    m, l = g.modal_mesh
    amp = np.where(g.mask & (l <= lmax) & (l > 0), 1.0, 0.0)
    zeta = torch.as_tensor(rng.standard_normal((batch, n_fields) + g.modal_shape) * amp)
    delta = torch.as_tensor(rng.standard_normal((batch, n_fields) + g.modal_shape) * amp * divergent_fraction)
    uc, vc = get_cos_lat_vector(zeta, delta, g, clip=False)
    cos = torch.as_tensor(np.cos(g.latitudes))
    u = (g.to_nodal(uc) / cos).numpy()
    v = (g.to_nodal(vc) / cos).numpy()
    rms = np.sqrt(0.5 * (u ** 2 + v ** 2).mean(axis=(-2, -1), keepdims=True)) + 1e-12
    return speed * u / rms, speed * v / rms


@dataclasses.dataclass
class SyntheticReanalysis:
    """Generator of pressure-level data and forcings on a grid."""

    grid: Grid
    levels: np.ndarray = dataclasses.field(default_factory=lambda: PRESSURE_LEVELS_37.copy())
    lmax: int = 21
    seed: int = 0
    # one horizontal anomaly pattern for every level of T, z and the winds
    # (False: an independent pattern per level, statically unstable columns)
    coherent: bool = True

    def _profiles(self):
        p = self.levels / 1000.0
        t_mean = 200.0 + 100.0 * p ** 0.35
        q_mean = 0.02 * p ** 3
        z_mean = 4.8e5 * (1.0 - np.log(self.levels) / np.log(1000.0)) * 0.999
        cl = 1e-4 * np.exp(-((np.log(p) - np.log(0.8)) ** 2) / 0.3)
        ci = 1e-4 * np.exp(-((np.log(p) - np.log(0.3)) ** 2) / 0.3)
        return t_mean, q_mean, z_mean, cl, ci

    def sample(self, batch: int, step: int = 0) -> dict:
        rng = np.random.default_rng([self.seed, step + 1000])
        nl = len(self.levels)
        t_mean, q_mean, z_mean, cl_mean, ci_mean = self._profiles()
        noise = lambda: band_limited_noise(self.grid, nl, self.lmax, rng, batch)
        sh = (1, nl, 1, 1)
        if self.coherent:
            shared = lambda: np.broadcast_to(band_limited_noise(self.grid, 1, self.lmax, rng, batch),
                                             (batch, nl) + self.grid.nodal_shape)
            u1, v1 = rotational_winds(self.grid, 1, self.lmax, rng, batch, speed=10.0, divergent_fraction=0.1)
            # wind anomaly amplitude from 0.6 (1000 hPa) to 1.4 (top), mean ≈ 1
            prof = (0.6 + 0.8 * (1.0 - self.levels / 1000.0)).reshape(sh)
            u, v = u1 * prof, v1 * prof
            t_noise, z_noise = shared(), shared()
        else:
            u, v = rotational_winds(self.grid, nl, self.lmax, rng, batch, speed=10.0, divergent_fraction=0.1)
            t_noise, z_noise = noise(), noise()
        out = {
            "u": u,
            "v": v,
            "t": np.clip(t_mean.reshape(sh) + 5.0 * t_noise, 180.0, 320.0),
            "q": np.minimum(q_mean.reshape(sh) * np.exp(0.3 * noise()), 0.02),
            "z": z_mean.reshape(sh) + 2.0e3 * z_noise,
            "clwc": np.minimum(cl_mean.reshape(sh) * np.exp(0.5 * noise()), 1e-4),
            "ciwc": np.minimum(ci_mean.reshape(sh) * np.exp(0.5 * noise()), 1e-4),
        }
        return {k: torch.as_tensor(v, dtype=torch.float32) for k, v in out.items()}

    def forcings(self, batch: int = 1) -> dict:
        rng = np.random.default_rng(self.seed + 17)
        lat = self.grid.latitudes
        n1 = lambda: band_limited_noise(self.grid, 1, 10, rng, 1)[:, 0]
        sst = 271.0 + 34.0 * np.cos(lat)[None, None, :] ** 2 + 0.0 * n1()
        ice = np.clip(0.5 + 0.5 * n1(), 0.0, 1.0)
        relief = n1()
        # continents where the relief field exceeds 0.3.  Height rises smoothly from the coast
        # (softplus ramp of width 0.2) and saturates smoothly below 3.5 km: a clipped linear ramp
        # (0 at the coast, flat-topped at 5 km) put 1-1.5 km steps between neighbouring grid
        # points at 1.4°, and the dry core's sigma-coordinate flow over those kinks drove
        # near-surface temperatures away without bound after ~100 physics steps
        x = (relief - 0.3) / 0.2
        ramp = 0.2 * np.logaddexp(0.0, x)
        oro = 3.5e3 * np.tanh(1.2e3 * ramp / 3.5e3)
        land = (relief > 0.3).astype(np.float64)
        f = {"sea_surface_temperature": sst, "sea_ice_cover": ice, "orography": oro, "land_sea_mask": land}
        return {k: torch.as_tensor(np.broadcast_to(v, (batch,) + self.grid.nodal_shape).copy(), dtype=torch.float32)
                for k, v in f.items()}

    def stats(self) -> dict:
        """Per-field, per-level mean/std used for normalisation."""
        x = self.sample(2, step=-1)
        out = {}
        for k, v in x.items():
            mean = v.mean(dim=(0, 2, 3))
            std = v.std(dim=(0, 2, 3))
            floor = 0.05 * float(std.mean()) + 0.01 * float(mean.abs().mean()) + 1e-12
            out[k] = (mean, torch.clamp(std, min=floor))
        return out


def pressure_to_sigma_matrix(pressure_levels_hpa: np.ndarray, sigma_centers: np.ndarray,
                             surface_pressure_hpa: float = 1000.0) -> np.ndarray:
    """Linear-in-log-p interpolation matrix (n_sigma × n_pressure) at fixed ps."""
    lp = np.log(pressure_levels_hpa)
    target = np.log(np.clip(sigma_centers * surface_pressure_hpa, pressure_levels_hpa[0], pressure_levels_hpa[-1]))
    m = np.zeros((len(sigma_centers), len(pressure_levels_hpa)))
    for i, t in enumerate(target):
        k = np.searchsorted(lp, t)
        k = min(max(k, 1), len(lp) - 1)
        w = (t - lp[k - 1]) / (lp[k] - lp[k - 1])
        m[i, k - 1] = 1.0 - w
        m[i, k] = w
    return m


def sigma_to_pressure_matrix(pressure_levels_hpa: np.ndarray, sigma_centers: np.ndarray,
                             surface_pressure_hpa: float = 1000.0) -> np.ndarray:
    """Linear-in-log-p interpolation matrix (n_pressure × n_sigma) at fixed ps (clamped ends)."""
    ls = np.log(sigma_centers * surface_pressure_hpa)
    target = np.clip(np.log(pressure_levels_hpa), ls[0], ls[-1])
    m = np.zeros((len(pressure_levels_hpa), len(sigma_centers)))
    for i, t in enumerate(target):
        k = np.searchsorted(ls, t)
        k = min(max(k, 1), len(ls) - 1)
        w = (t - ls[k - 1]) / (ls[k] - ls[k - 1])
        m[i, k - 1] = 1.0 - w
        m[i, k] = w
    return m
