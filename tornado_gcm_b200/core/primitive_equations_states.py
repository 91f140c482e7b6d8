"""Dycore test-case initial states (reference ``core/primitive_equations_states.py:29-290``).

Same constructors and returned states as the reference: isothermal rest
atmosphere (Held–Suarez start), the Jablonowski–Williamson steady state in
the reference's formulation (analytic vorticity of u = u0 cos^{3/2}(η_v)
sin²(2φ), zero T', flat ln ps), its localized vorticity perturbation, and
a Gaussian scalar blob.
"""

from __future__ import annotations

from typing import Callable, Optional

import numpy as np
import torch

from tornado_gcm_b200.core import primitive_equations

OROGRAPHY = "orography"
REF_TEMP_KEY = "reference_temperature"
GEOPOTENTIAL = "geopotential"


def _great_circle(lat0: float, lon0: float, lat: np.ndarray, lon: np.ndarray) -> np.ndarray:
    c = np.sin(lat0) * np.sin(lat) + np.cos(lat0) * np.cos(lat) * np.cos(lon - lon0)
    return np.arccos(np.clip(c, -1.0, 1.0))


def _surface_lnps(grid, p0: float, device) -> torch.Tensor:
    nod = torch.full(tuple(grid.nodal_shape), float(np.log(p0)), dtype=torch.float32, device=device)
    return grid.to_modal(nod).unsqueeze(0)


def isothermal_rest_atmosphere(coords, physics_specs, tref: float = 288.0, p0: float = 1e5, p1: float = 0.0,
                               surface_height: Optional[torch.Tensor] = None, device="cpu"):
    grid = coords.horizontal
    n = coords.vertical.layers
    if surface_height is not None:
        orography = primitive_equations.truncated_modal_orography(surface_height, coords)
    else:
        orography = torch.zeros(tuple(grid.modal_shape), device=device)
    ref_temp = np.full(n, tref, dtype=np.float64)

    def initial_state_fn(rng_key=None):
        shape = tuple(coords.modal_shape)
        lnps = torch.full(tuple(grid.nodal_shape), float(np.log(p0)), dtype=torch.float32, device=device)
        if p1 > 0 and rng_key is not None:
            lon, sin_lat = grid.nodal_mesh
            lon_t = torch.as_tensor(lon, dtype=torch.float32, device=device)
            lat_t = torch.as_tensor(np.arcsin(sin_lat), dtype=torch.float32, device=device)
            lnps = torch.log(torch.exp(lnps) + p1 * torch.sin(5 * lon_t) * torch.exp(-10 * lat_t ** 2))
        lsp = grid.to_modal(lnps).unsqueeze(0)
        z = lambda: torch.zeros(shape, device=device)
        return primitive_equations.State(z(), z(), z(), lsp)

    return initial_state_fn, {OROGRAPHY: orography, REF_TEMP_KEY: ref_temp}


def steady_state_jw(coords, physics_specs, u0: float = 35.0, p0: float = 1e5, t0: float = 288.0,
                    delta_t: float = 4.8e5, gamma: float = 0.005, eta_tropo: float = 0.2, eta0: float = 0.252,
                    device="cpu"):
    grid = coords.horizontal
    eta = coords.vertical.centers
    R, g, a = physics_specs.R, physics_specs.g, physics_specs.radius
    lat = np.arcsin(grid.nodal_axes[1])

    def t_ref(e):
        t = t0 * e ** (R * gamma / g)
        return t + delta_t * (eta_tropo - e) ** 5 if e > eta_tropo else t

    ref_temp = np.array([t_ref(e) for e in eta], dtype=np.float64)
    ev = (eta - eta0) * np.pi / 2.0

    def initial_state_fn(rng_key=None):
        shape = tuple(coords.modal_shape)
        prof = -4.0 * u0 / a * np.cos(ev) ** 1.5  # (n,)
        lat_part = np.sin(lat) * np.cos(lat) * (2.0 - 5.0 * np.sin(lat) ** 2)  # (J,)
        vort_nodal = np.broadcast_to(prof[:, None, None] * lat_part[None, None, :],
                                     (len(eta),) + tuple(grid.nodal_shape))
        vort = grid.to_modal(torch.as_tensor(np.ascontiguousarray(vort_nodal), dtype=torch.float32, device=device))
        z = lambda: torch.zeros(shape, device=device)
        return primitive_equations.State(vort, z(), z(), _surface_lnps(grid, p0, device))

    return initial_state_fn, {OROGRAPHY: torch.zeros(tuple(grid.modal_shape), device=device),
                              REF_TEMP_KEY: ref_temp}


def baroclinic_perturbation_jw(coords, physics_specs, u_perturb: float = 1.0, lon_location: float = np.pi / 9,
                               lat_location: float = 2 * np.pi / 9, perturbation_radius: float = 0.1, device="cpu"):
    grid = coords.horizontal
    lon, sin_lat = grid.nodal_mesh
    r = _great_circle(lat_location, lon_location, np.arcsin(sin_lat), lon)
    env = np.exp(-(r / perturbation_radius) ** 2) * u_perturb / physics_specs.radius
    n = coords.vertical.layers
    vort = grid.to_modal(torch.as_tensor(np.broadcast_to(env, (n,) + env.shape).copy(), dtype=torch.float32,
                                         device=device))
    shape = tuple(coords.modal_shape)
    return primitive_equations.State(vort, torch.zeros(shape, device=device), torch.zeros(shape, device=device),
                                     torch.zeros(tuple(coords.surface_modal_shape), device=device))


def gaussian_scalar(coords, lon_location: float = np.pi / 9, lat_location: float = 2 * np.pi / 9,
                    perturbation_radius: float = 0.2, amplitude: float = 1.0, device="cpu") -> torch.Tensor:
    grid = coords.horizontal
    lon, sin_lat = grid.nodal_mesh
    r = _great_circle(lat_location, lon_location, np.arcsin(sin_lat), lon)
    nod = amplitude * np.exp(-(r / perturbation_radius) ** 2)
    return grid.to_modal(torch.as_tensor(nod, dtype=torch.float32, device=device))
