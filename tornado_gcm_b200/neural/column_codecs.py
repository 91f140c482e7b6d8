"""Column encoder / decoder between pressure-level data and the sigma-level model state.

Encoder: normalised pressure-level fields (u, v, t, q, z, clwc, ciwc on P
levels) + forcings → physical prior (log-pressure interpolation to σ
levels at a reference surface pressure) + learned per-column correction
(MLP) → nodal σ-level u, v, T, q, cloud liquid/ice, ln ps → modal State
(u, v → vorticity/divergence, T' = T − T_ref).

Decoder: modal State → nodal σ-level fields → prior (σ→p interpolation,
hydrostatic geopotential) + learned correction → normalised pressure-level
fields.  Both MLPs run on the tcgen05 BF16 kernels on CUDA.

The same roles are played in the reference by the WeatherBench-to-
primitive encoders and learned decoders (``neural/encoders_decoders.py:32-495``).
"""

from __future__ import annotations

from typing import Sequence

import numpy as np
import torch
import torch.nn as nn

from tornado_gcm_b200.core import primitive_equations as pe
from tornado_gcm_b200.core import spherical_harmonic as sh
from tornado_gcm_b200.neural.standard_layers import Mlp, gelu_tanh
from tornado_gcm_b200.neural.towers import ForwardTower
from tornado_gcm_b200.training.synthetic import (DATA_FIELDS, pressure_to_sigma_matrix,
                                                 sigma_to_pressure_matrix)

VELOCITY_SCALE = 6.37122e6 * 2 * 7.292e-5  # m/s per model velocity unit (radius · 2Ω)
_G_SI = 9.80616
_RD_SI = 1004.0 * 2.0 / 7.0
TRACERS = ("specific_cloud_ice_water_content", "specific_cloud_liquid_water_content", "specific_humidity")
_TRACER_OF_FIELD = {"q": "specific_humidity", "clwc": "specific_cloud_liquid_water_content",
                    "ciwc": "specific_cloud_ice_water_content"}


def _scale_last_layer(mlp: Mlp, factor: float):
    with torch.no_grad():
        mlp.layers[-1].weight.mul_(factor)


class ColumnEncoder(nn.Module):
    def __init__(self, coords, reference_temperature: np.ndarray, pressure_levels: np.ndarray,
                 data_stats: dict, forcing_keys: Sequence[str], hidden: int = 256, depth: int = 3,
                 correction_scale: float = 0.1, orography_key: str | None = None,
                 orography_unit_m: float = 1.0):
        super().__init__()
        self.coords = coords
        self.orography_key = orography_key
        self.orography_unit_m = float(orography_unit_m)
        self.grid = coords.horizontal
        n = coords.vertical.layers
        npl = len(pressure_levels)
        self.n, self.npl = n, npl
        self.forcing_keys = tuple(forcing_keys)
        p2s = pressure_to_sigma_matrix(pressure_levels, coords.vertical.centers)
        self.register_buffer("p2s", torch.tensor(p2s, dtype=torch.float32))
        self.register_buffer("t_ref", torch.tensor(reference_temperature, dtype=torch.float32).reshape(-1, 1, 1))
        for k in DATA_FIELDS:
            m, s = data_stats[k]
            self.register_buffer(f"mean_{k}", m.float().reshape(-1, 1, 1).clone())
            self.register_buffer(f"std_{k}", s.float().reshape(-1, 1, 1).clone())
        n_in = len(DATA_FIELDS) * npl + len(self.forcing_keys)
        n_out = 6 * n + 1
        self.net = ForwardTower(Mlp.uniform(n_in, n_out, hidden_size=hidden, hidden_layers=depth,
                                            activation=gelu_tanh))
        _scale_last_layer(self.net.neural_net, correction_scale)
        # per-output physical scale of the learned correction (u, v m/s; T K; q, clouds kg/kg; ln ps)
        scales = np.concatenate([np.full(n, 1.0), np.full(n, 1.0), np.full(n, 1.0), np.full(n, 1e-4),
                                 np.full(n, 1e-6), np.full(n, 1e-6), [1e-3]])
        self.register_buffer("out_scale", torch.tensor(scales, dtype=torch.float32).reshape(-1, 1, 1))

    def _phys(self, data: dict, k: str) -> torch.Tensor:
        return data[k] * getattr(self, f"std_{k}") + getattr(self, f"mean_{k}")

    def forward(self, data: dict, forcings: dict | None = None) -> pe.State:
        ref = data["u"]
        lead = ref.shape[:-3]
        feats = [data[k] for k in DATA_FIELDS]
        if self.forcing_keys:
            for k in self.forcing_keys:
                f = forcings[k].to(ref.dtype)
                while f.dim() < ref.dim():
                    f = f.unsqueeze(-3)
                feats.append(f.expand(*lead, 1, *ref.shape[-2:]) if f.shape[-3] == 1 else f)
        x = torch.cat(feats, dim=-3)
        corr = self.net(x).float() * self.out_scale  # (…, 6n+1, I, J)
        n = self.n
        interp = lambda t: torch.einsum("sp,...pij->...sij", self.p2s, t)
        u = interp(self._phys(data, "u")) + corr[..., :n, :, :]
        v = interp(self._phys(data, "v")) + corr[..., n:2 * n, :, :]
        T = interp(self._phys(data, "t")) + corr[..., 2 * n:3 * n, :, :]
        q = torch.clamp(interp(self._phys(data, "q")) + corr[..., 3 * n:4 * n, :, :], min=0.0)
        cl = torch.clamp(interp(self._phys(data, "clwc")) + corr[..., 4 * n:5 * n, :, :], min=0.0)
        ci = torch.clamp(interp(self._phys(data, "ciwc")) + corr[..., 5 * n:6 * n, :, :], min=0.0)
        lnps = corr[..., 6 * n:, :, :]
        if self.orography_key is not None and forcings is not None and self.orography_key in forcings:
            # hypsometric prior: ln(ps / p0) = −g z_s / (R_d T_s) with T_s the lowest-level temperature
            zs = forcings[self.orography_key].to(T.dtype) * self.orography_unit_m
            while zs.dim() < T.dim():
                zs = zs.unsqueeze(-3)
            lnps = lnps - _G_SI * zs / (_RD_SI * T[..., -1:, :, :])
        g = self.grid
        vort, div = sh.uv_nodal_to_vor_div_modal(g, u / VELOCITY_SCALE, v / VELOCITY_SCALE)
        modal = g.to_modal(torch.cat([T - self.t_ref, q, cl, ci, lnps], dim=-3))
        temp, qm, clm, cim, lsp = torch.split(modal, [n, n, n, n, 1], dim=-3)
        tracers = {"specific_humidity": qm, "specific_cloud_liquid_water_content": clm,
                   "specific_cloud_ice_water_content": cim}
        return pe.State(vort, div, temp, lsp, tracers, sim_time=0.0)


class ColumnDecoder(nn.Module):
    def __init__(self, coords, reference_temperature: np.ndarray, pressure_levels: np.ndarray,
                 data_stats: dict, ideal_gas_constant_si: float = 1004.0 * 2 / 7, hidden: int = 256,
                 depth: int = 3, correction_scale: float = 0.1):
        super().__init__()
        self.coords = coords
        self.grid = coords.horizontal
        n = coords.vertical.layers
        npl = len(pressure_levels)
        self.n, self.npl = n, npl
        s2p = sigma_to_pressure_matrix(pressure_levels, coords.vertical.centers)
        self.register_buffer("s2p", torch.tensor(s2p, dtype=torch.float32))
        self.register_buffer("t_ref", torch.tensor(reference_temperature, dtype=torch.float32).reshape(-1, 1, 1))
        g = pe.get_geopotential_weights_sigma(coords.vertical, ideal_gas_constant_si)
        self.register_buffer("geo", torch.tensor(g, dtype=torch.float32))
        for k in DATA_FIELDS:
            m, s = data_stats[k]
            self.register_buffer(f"mean_{k}", m.float().reshape(-1, 1, 1).clone())
            self.register_buffer(f"std_{k}", s.float().reshape(-1, 1, 1).clone())
        n_in = 6 * n + 1
        n_out = len(DATA_FIELDS) * npl
        self.net = ForwardTower(Mlp.uniform(n_in, n_out, hidden_size=hidden, hidden_layers=depth,
                                            activation=gelu_tanh))
        _scale_last_layer(self.net.neural_net, correction_scale)
        in_scale = np.concatenate([np.full(n, 0.1), np.full(n, 0.1), np.full(n, 0.2), np.full(n, 1e3),
                                   np.full(n, 1e5), np.full(n, 1e5), [10.0]])
        self.register_buffer("in_scale", torch.tensor(in_scale, dtype=torch.float32).reshape(-1, 1, 1))

    def forward(self, state: pe.State, forcings: dict | None = None) -> dict:
        g = self.grid
        n = self.n
        uc, vc = sh.get_cos_lat_vector(state.vorticity, state.divergence, g, clip=False)
        tr = state.tracers
        stack = torch.cat([uc, vc, state.temperature_variation, tr["specific_humidity"],
                           tr["specific_cloud_liquid_water_content"], tr["specific_cloud_ice_water_content"],
                           state.log_surface_pressure], dim=-3)
        nodal = g.to_nodal(stack)
        sec = 1.0 / g.const("cos_lat", nodal.device, nodal.dtype)
        u = nodal[..., :n, :, :] * sec * VELOCITY_SCALE
        v = nodal[..., n:2 * n, :, :] * sec * VELOCITY_SCALE
        T = nodal[..., 2 * n:3 * n, :, :] + self.t_ref
        q, cl, ci = nodal[..., 3 * n:4 * n, :, :], nodal[..., 4 * n:5 * n, :, :], nodal[..., 5 * n:6 * n, :, :]
        lnps = nodal[..., 6 * n:, :, :]
        z = torch.einsum("gh,...hij->...gij", self.geo, T)
        sigma_fields = {"u": u, "v": v, "t": T, "q": q, "z": z, "clwc": cl, "ciwc": ci}
        feats = torch.cat([u / VELOCITY_SCALE, v / VELOCITY_SCALE, nodal[..., 2 * n:3 * n, :, :], q, cl, ci, lnps],
                          dim=-3) * self.in_scale
        corr = self.net(feats).float()
        out = {}
        for i, k in enumerate(DATA_FIELDS):
            prior = torch.einsum("ps,...sij->...pij", self.s2p, sigma_fields[k])
            prior_n = (prior - getattr(self, f"mean_{k}")) / getattr(self, f"std_{k}")
            out[k] = prior_n + corr[..., i * self.npl:(i + 1) * self.npl, :, :]
        return out
