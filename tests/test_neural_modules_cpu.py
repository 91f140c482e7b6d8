"""Feature, transform, attention, encoder/decoder, equation and helper modules (CPU, FP64 oracles)."""

import math

import numpy as np
import pytest
import torch

from tornado_gcm_b200.core import coordinate_systems, sigma_coordinates
from tornado_gcm_b200.core import primitive_equations as pe
from tornado_gcm_b200.core import spherical_harmonic as shm
from tornado_gcm_b200.utils.typing import KeyWithCosLatFactor


@pytest.fixture(scope="module")
def grid():
    return shm.Grid.T21()


def _smooth_modal(grid, n, scale=1.0, seed=0, dtype=torch.float64):
    gen = torch.Generator().manual_seed(seed)
    l = torch.arange(grid.modal_shape[1], dtype=dtype)
    x = torch.randn(n, *grid.modal_shape, generator=gen, dtype=dtype) * torch.as_tensor(grid.mask) * torch.exp(-l / 3)
    return x * scale


# ───────────────────────── attention ─────────────────────────


def test_attention_matches_explicit_softmax():
    from tornado_gcm_b200.neural.transformer_layers import MultiHeadAttention

    torch.manual_seed(0)
    mha = MultiHeadAttention(4, 16, normalize_qk=True).double()
    x = torch.randn(3, 7, 16, dtype=torch.float64)
    mask = torch.rand(3, 7, 7) > 0.3
    mask[..., 0] = True
    out = mha(x, mask=mask)
    q, k, v = mha.q_proj(x), mha.k_proj(x), mha.v_proj(x)
    sh = lambda t: t.view(3, 7, 4, 4).transpose(1, 2)
    q, k, v = mha.q_ln(sh(q)), mha.k_ln(sh(k)), sh(v)
    s = q @ k.transpose(-1, -2) / 2.0
    s = s.masked_fill(~mask[:, None], float("-inf"))
    ref = mha.out_proj((torch.softmax(s, -1) @ v).transpose(1, 2).reshape(3, 7, 16))
    torch.testing.assert_close(out, ref)


def test_transformer_stacks_and_column_tower():
    from tornado_gcm_b200.neural.towers import ColumnTransformerTower
    from tornado_gcm_b200.neural.transformer_layers import (ColumnTransformer, SinusoidalPositionalEncoding,
                                                             TransformerDecoder, TransformerEncoder)

    enc = TransformerEncoder(16, 4, 2)
    dec = TransformerDecoder(16, 4, 2, d_cross=8)
    x = torch.randn(2, 5, 16)
    assert enc(x).shape == x.shape
    assert dec(x, torch.randn(2, 3, 8)).shape == x.shape
    pe_ = SinusoidalPositionalEncoding(16)
    assert torch.allclose(pe_(torch.zeros(1, 4, 16))[0, 0, 1::2], torch.ones(8))
    tower = ColumnTransformerTower(ColumnTransformer(3, 2, d_model=16, num_heads=4, num_layers=1))
    y = tower(torch.randn(2, 6, 3, 4, 5))        # (batch, levels, features, lon, lat)
    assert y.shape == (2, 6, 2, 4, 5)


# ───────────────────────── transforms ─────────────────────────


def test_softclip_and_normalisation():
    from tornado_gcm_b200.neural.transforms import InverseShiftAndNormalize, ShiftAndNormalize, SoftClip

    sc = SoftClip(4.0, 0.5)
    x = torch.linspace(-8, 8, 1001, dtype=torch.float64)
    y = sc.clip(x)
    assert y.abs().max() < 4.0 and torch.all(y[1:] > y[:-1])
    assert float(sc.clip(torch.tensor(1e4, dtype=torch.float64))) <= 4.0
    assert abs(float(sc.clip(torch.tensor(0.0, dtype=torch.float64)))) < 1e-3
    d = {"a": torch.randn(3), "b": torch.randn(3)}
    fwd = ShiftAndNormalize({"a": 2.0}, {"a": 3.0}, global_scale=2.0)
    back = InverseShiftAndNormalize({"a": 2.0}, {"a": 3.0}, global_scale=2.0)
    r = back(fwd(d))
    torch.testing.assert_close(r["a"], d["a"])
    assert r["b"] is d["b"]


def test_diff_operators_and_batched_transforms(grid):
    from tornado_gcm_b200.neural.transforms import ToModalDiffOperators, batched_to_modal, batched_to_nodal

    a, b = _smooth_modal(grid, 3), _smooth_modal(grid, 1, seed=1)
    out = ToModalDiffOperators(grid)({KeyWithCosLatFactor("a", 0): a, ("b", 1): b})
    dlon, dlat = grid.cos_lat_grad(a, clip=False)
    torch.testing.assert_close(out[KeyWithCosLatFactor("a_dlon", 1)], dlon)
    torch.testing.assert_close(out[KeyWithCosLatFactor("a_dlat", 1)], dlat)
    torch.testing.assert_close(out[("b_del2", 1)], grid.laplacian(b))
    nod = batched_to_nodal(grid, {"a": a, "b": b[0]})
    torch.testing.assert_close(nod["a"], grid.to_nodal(a))
    torch.testing.assert_close(nod["b"], grid.to_nodal(b[0]))
    mod = batched_to_modal(grid, nod)
    torch.testing.assert_close(mod["a"], grid.to_modal(nod["a"]))


def test_to_modal_with_div_curl_inverts_velocity(grid):
    from tornado_gcm_b200.neural.transforms import ToModalWithDivCurl

    vor = grid.clip_wavenumbers(_smooth_modal(grid, 2, seed=2))
    div = grid.clip_wavenumbers(_smooth_modal(grid, 2, seed=3))
    vor[..., 0, 0] = 0
    div[..., 0, 0] = 0
    u, v = shm.vor_div_to_uv_nodal(grid, vor, div)
    out = ToModalWithDivCurl(grid)({"u_component_of_wind": u, "v_component_of_wind": v})
    err_v = grid.clip_wavenumbers(out["vorticity"]) - vor
    err_d = grid.clip_wavenumbers(out["divergence"]) - div
    assert float(err_v.abs().max()) < 1e-3 * float(vor.abs().max())
    assert float(err_d.abs().max()) < 1e-3 * float(div.abs().max())


# ───────────────────────── features ─────────────────────────


def _inputs(grid, n=4, seed=0):
    return {"vorticity": _smooth_modal(grid, n, seed=seed), "divergence": _smooth_modal(grid, n, seed=seed + 1),
            "temperature_variation": _smooth_modal(grid, n, seed=seed + 2),
            "log_surface_pressure": _smooth_modal(grid, 1, 0.01, seed=seed + 3),
            "tracers": {"specific_humidity": _smooth_modal(grid, n, 1e-3, seed=seed + 4)},
            "sim_time": torch.tensor(5.0)}


def test_velocity_and_prognostics(grid):
    from tornado_gcm_b200.neural.features import MemoryVelocityAndValues, VelocityAndPrognostics
    from tornado_gcm_b200.neural.transforms import ToModalDiffOperators

    inp = _inputs(grid)
    f = VelocityAndPrognostics(grid, compute_gradients_fn=ToModalDiffOperators(grid))(inp)
    u, v = shm.vor_div_to_uv_nodal(grid, inp["vorticity"], inp["divergence"], clip=False)
    torch.testing.assert_close(f["u"], u)
    torch.testing.assert_close(f["v"], v)
    torch.testing.assert_close(f["temperature_variation_del2"], grid.to_nodal(grid.laplacian(inp["temperature_variation"])))
    sec = torch.as_tensor(1.0 / grid.cos_lat)
    dlon, _ = grid.cos_lat_grad(inp["temperature_variation"], clip=False)
    torch.testing.assert_close(f["temperature_variation_dlon"], grid.to_nodal(dlon) * sec)
    m = MemoryVelocityAndValues(grid, fields_to_include=["temperature_variation"])({}, memory=inp)
    assert set(m) == {"memory_u", "memory_v", "memory_temperature_variation"}


def test_other_features(grid):
    from tornado_gcm_b200.neural import features as F

    inp = _inputs(grid)
    rad = F.RadiationFeatures(grid)(inp)["radiation"]
    assert rad.shape == (1, *grid.nodal_shape) and float(rad.min()) >= 0 and float(rad.max()) <= 1
    no_t = F.RadiationFeatures(grid)({k: v for k, v in inp.items() if k != "sim_time"})["radiation"]
    torch.testing.assert_close(no_t[0, 0], torch.as_tensor(grid.cos_lat, dtype=torch.float32))
    lat = F.LatitudeFeatures(grid)(inp)
    torch.testing.assert_close(lat["sin_latitude"] ** 2 + lat["cos_latitude"] ** 2, torch.ones(1, *grid.nodal_shape))
    pres = F.PressureFeatures(grid, np.array([0.25, 0.75]))(inp)["pressure"]
    torch.testing.assert_close(pres[1] / pres[0], torch.full(grid.nodal_shape, 3.0, dtype=pres.dtype))
    comb = F.CombinedFeatures([F.LatitudeFeatures(grid), F.LatitudeFeatures(grid)])
    with pytest.raises(ValueError):
        comb(inp)
    packed = F.pack_features({"b": torch.ones(2, 3, 4), "a": torch.zeros(3, 4)})
    assert packed.shape == (3, 3, 4) and float(packed[0].abs().sum()) == 0.0
    cov = F.FloatDataFeatures(grid, {"z": grid.to_nodal(_smooth_modal(grid, 1, seed=9))},
                              compute_gradients_fn=__import__("tornado_gcm_b200.neural.transforms",
                                                              fromlist=["x"]).ToModalDiffOperators(grid))(inp)
    assert {"z", "z_dlon", "z_dlat", "z_del2"} <= set(cov)


def test_embedding_features(grid):
    from tornado_gcm_b200.neural import features as F

    inp = _inputs(grid, n=3)

    class Conv(torch.nn.Module):
        def forward(self, x):                 # (channels, levels, lon, lat) → 2 outputs
            return torch.stack([x.sum(0), x.mean(0)])

    vol = F.EmbeddingVolumeFeatures(grid, Conv(), np.array([0.2, 0.5, 0.8]), n_output=2)(inp)
    assert set(vol) == {"CNN1D_0", "CNN1D_1"} and vol["CNN1D_0"].shape == (3, *grid.nodal_shape)

    class Const(torch.nn.Module):
        def __init__(self, c):
            super().__init__()
            self.c = c

        def forward(self, x):
            return torch.full((2,) + tuple(x.shape[1:]), self.c, dtype=x.dtype)

    mask = torch.zeros(grid.nodal_shape, dtype=torch.float64)
    mask[:10] = 1.0
    surf = F.EmbeddingSurfaceFeatures(grid, Const(1.0), Const(2.0), Const(3.0), mask, ({}, {}), ({}, {}), ({}, {}),
                                      output_size=2)
    ice = torch.zeros(grid.nodal_shape, dtype=torch.float64)
    ice[10:20] = 1.0
    emb = surf(inp, forcing={"sea_ice_cover": ice,
                             "sea_surface_temperature": torch.zeros(grid.nodal_shape, dtype=torch.float64)})
    e = emb["surface_embedding"]
    assert float(e[:, :10].min()) == 1.0 and float(e[:, 10:20].min()) == 3.0 and float(e[:, 20:].max()) == 2.0


# ───────────────────── encoders / decoders ─────────────────────


class _SI:
    g, R, R_vapor, kappa = 9.81, 287.0, 461.0, 2.0 / 7.0


def test_decoder_encoder_round_trip(grid):
    from tornado_gcm_b200.neural.encoders_decoders import PrimitiveToWeatherbenchDecoder, WeatherbenchToPrimitiveEncoder

    vert = sigma_coordinates.SigmaCoordinates.equidistant(8)
    coords = coordinate_systems.CoordinateSystem(grid, vert)
    tref = np.full(8, 250.0)
    plev = np.linspace(100, 900, 17) * 100.0
    vor = grid.clip_wavenumbers(_smooth_modal(grid, 1, 1e-5, seed=4)).expand(8, -1, -1).clone()
    div = grid.clip_wavenumbers(_smooth_modal(grid, 1, 1e-6, seed=5)).expand(8, -1, -1).clone()
    vor[..., 0, 0] = 0
    div[..., 0, 0] = 0
    lnps = grid.to_modal(torch.full((1, *grid.nodal_shape), math.log(1e5), dtype=torch.float64))
    st = pe.State(vor, div, torch.zeros_like(vor), lnps, {})
    wb = PrimitiveToWeatherbenchDecoder(coords, _SI, tref, plev)(st)
    assert wb["temperature"].shape == (17, *grid.nodal_shape)
    wb.pop("surface_pressure")
    back = WeatherbenchToPrimitiveEncoder(coords, _SI, tref, plev)(wb)
    err = grid.clip_wavenumbers(back.vorticity) - vor
    assert float(err[1:-1].abs().max()) < 1e-3 * float(vor.abs().max())
    dps = (grid.to_nodal(back.log_surface_pressure) - grid.to_nodal(lnps)).abs().max()
    assert float(dps) < 0.02


# ───────────────────────── equations ─────────────────────────


def test_equations_dict_api_and_held_suarez(grid):
    from tornado_gcm_b200.neural.coordinates import SigmaLevels
    from tornado_gcm_b200.neural.equations import (HeldSuarezForcing, MoistPrimitiveEquationsWithCloudMoisture,
                                                   PrimitiveEquations, get_reference_temperature)
    from tornado_gcm_b200.utils.units import SimUnits

    vert = sigma_coordinates.SigmaCoordinates.equidistant(6)
    coords = coordinate_systems.CoordinateSystem(grid, vert)
    units = SimUnits.from_si()
    tref = get_reference_temperature(SigmaLevels(vert))
    assert np.all(np.diff(tref[2:]) > 0)  # warmer towards the surface in the troposphere
    oro = torch.zeros(1, *grid.modal_shape, dtype=torch.float64)
    eq = PrimitiveEquations(coords, units, tref, oro)
    st = pe.State(_smooth_modal(grid, 6, 1e-3), _smooth_modal(grid, 6, 1e-3, seed=1),
                  _smooth_modal(grid, 6, seed=2), _smooth_modal(grid, 1, 1e-3, seed=3), {})
    t_abs = st.temperature_variation + torch.as_tensor(tref).reshape(-1, 1, 1) * 0  # modal: only l=0 shifts
    d = {"vorticity": st.vorticity, "divergence": st.divergence, "temperature_variation": st.temperature_variation,
         "log_surface_pressure": st.log_surface_pressure}
    ex_d, ex_s = eq.explicit_terms(d), eq.explicit_terms(st)
    torch.testing.assert_close(ex_d["vorticity"], ex_s.vorticity)
    assert t_abs.shape == st.temperature_variation.shape
    MoistPrimitiveEquationsWithCloudMoisture(coords, units, tref, oro)
    hs = HeldSuarezForcing(coords, units, tref)
    teq = hs.equilibrium_temperature()
    assert teq.min() >= 200.0 - 1e-9 and teq.shape == (6, 1, grid.nodal_shape[1])
    out = hs.explicit_terms(st)
    kv = torch.as_tensor(hs._kv).reshape(-1, 1, 1)
    torch.testing.assert_close(out.vorticity, -kv * st.vorticity)


def test_neural_equations_and_jax_aligned_parameterization(grid):
    from tornado_gcm_b200.neural.features import CombinedFeatures, VelocityAndPrognostics
    from tornado_gcm_b200.neural.neural_equations import DirectNeuralEquations
    from tornado_gcm_b200.neural.parameterizations import JaxAlignedDivCurlParameterization
    from tornado_gcm_b200.neural.transforms import IdentityTransform

    n = 3
    st = pe.State(_smooth_modal(grid, n), _smooth_modal(grid, n, seed=1), _smooth_modal(grid, n, seed=2),
                  _smooth_modal(grid, 1, seed=3), {"specific_humidity": _smooth_modal(grid, n, seed=4)}, 1.0)
    feats = CombinedFeatures([VelocityAndPrognostics(grid)])

    class Map(torch.nn.Module):
        def forward(self, f):
            return {"temperature_variation": 2.0 * f["temperature_variation"]}

    eqn = DirectNeuralEquations(grid, feats, Map())
    out = eqn.explicit_terms(st)
    torch.testing.assert_close(out.temperature_variation, grid.to_modal(grid.to_nodal(2 * st.temperature_variation)))
    assert float(out.vorticity.abs().max()) == 0.0

    class Net(torch.nn.Module):
        def forward(self, x):
            return torch.zeros((6 * n,) + tuple(x.shape[1:]), dtype=x.dtype)

    p = JaxAlignedDivCurlParameterization(grid, Net(), feats, IdentityTransform(), n_levels=n)
    t = p(st)
    assert t.vorticity.shape == st.vorticity.shape and float(t.temperature_variation.abs().max()) == 0.0


# ───────────────────────── helpers ─────────────────────────


def test_interpolators_and_helpers(grid):
    from tornado_gcm_b200.neural import field_utils as fu
    from tornado_gcm_b200.neural.coordinates import PressureLevels, SigmaLevels
    from tornado_gcm_b200.neural.interpolators import ConservativeOnPressure, LinearOnPressure
    from tornado_gcm_b200.neural.mappings import NodalMapping
    from tornado_gcm_b200.neural.normalizations import StreamNorm
    from tornado_gcm_b200.neural.spatial_filters import ComposedFilter, ExponentialModalFilter, HorizontalDiffusionFilter

    sig = SigmaLevels.equidistant(8)
    pl = PressureLevels.from_list(np.linspace(100, 1000, 10) * 100)
    ps = 1e5 + 1e3 * torch.rand(1, 4, 3, dtype=torch.float64)
    f = 2.0 * torch.as_tensor(sig.centers).reshape(-1, 1, 1) * ps + 3.0
    out = LinearOnPressure(pl).interpolate_field(f, sig, ps)
    torch.testing.assert_close(out, (2.0 * torch.as_tensor(pl.levels).reshape(-1, 1, 1) + 3.0).expand_as(out))
    x = torch.rand(8, 4, 3, dtype=torch.float64)
    same = ConservativeOnPressure(sig).regrid_field(x, sig, ps)
    torch.testing.assert_close(same, x)
    ref = torch.tensor([1.0, 2.0, 3.0])
    y = torch.randn(2, 3, 4, 5)
    torch.testing.assert_close(fu.extract_1d_field_perturbation(fu.reconstruct_1d_field_from_ref_values(y, ref), ref), y)
    assert fu.pad_along_axis(y, 1, 2).shape == (2, 6, 4, 5)
    assert fu.repeat_surface_to_volume(torch.randn(2, 4, 5), 3).shape == (2, 3, 4, 5)
    m = NodalMapping(torch.nn.Identity(), ["p", "q"], [2, 1])({"a": torch.randn(2, 4, 5), "b": torch.randn(4, 5)})
    assert m["p"].shape == (2, 4, 5) and m["q"].shape == (1, 4, 5)
    sn = StreamNorm(3, momentum=1.0)
    z = torch.randn(100, 3) * 5 + 2
    torch.testing.assert_close(sn.unnormalize(sn(z)), z, atol=1e-4, rtol=1e-4)
    filt = ComposedFilter(ExponentialModalFilter(grid), HorizontalDiffusionFilter(grid, tau=1e-4))
    s = filt(torch.ones(*grid.modal_shape))
    assert float(s[0, 0]) == 1.0 and float(s[0, -1]) < 1.0


def test_stochastic_physics_step(grid):
    from tornado_gcm_b200.neural.stochastic import (Corrector, GaussianRandomField, Perturbation,
                                                    StochasticPhysicsParameterizationStep)

    st = pe.State(_smooth_modal(grid, 2, dtype=torch.float32), _smooth_modal(grid, 2, seed=1, dtype=torch.float32),
                  _smooth_modal(grid, 2, seed=2, dtype=torch.float32), _smooth_modal(grid, 1, seed=3,
                                                                                      dtype=torch.float32),
                  {"specific_humidity": _smooth_modal(grid, 2, seed=4, dtype=torch.float32)})

    class Zero(torch.nn.Module):
        def forward(self, s):
            return s.tree_map(torch.zeros_like)

    step = StochasticPhysicsParameterizationStep(Zero(), Corrector(0.1), GaussianRandomField(grid, 2.0, 0.2),
                                                 Perturbation(), num_substeps=3)
    r0 = step.initialize_randomness(generator=torch.Generator().manual_seed(0))
    s1, r1 = step(st, randomness=r0)
    torch.testing.assert_close(s1.vorticity, st.vorticity)
    assert r1.prng_step == 3


def test_reference_diagnostics_api():
    from tornado_gcm_b200.core.primitive_equations import State
    from tornado_gcm_b200.neural import diagnostics as d
    from tornado_gcm_b200.utils.typing import ModelState

    def mk(q, t):
        z = torch.zeros(4, 5, 6)
        return State(vorticity=z + 1, divergence=z, temperature_variation=z + t,
                     log_surface_pressure=torch.zeros(1, 5, 6), tracers={"specific_humidity": torch.full((4, 5, 6), q)})

    traj = [mk(1.0, 2.0), mk(0.5, 2.0), mk(0.75, 3.0)]
    assert d.extract_energies(traj, mk(1.0, 2.0)).shape[0] == 4 and d.extract_masses(traj, mk(1.0, 2.0)).shape[0] == 4
    p, e = d.extract_precipitation_evaporation(traj)
    torch.testing.assert_close(p, torch.tensor([0.0, 2.0, 0.0], dtype=torch.float64))   # column q 4 -> 2 -> 3
    torch.testing.assert_close(e, torch.tensor([0.0, 0.0, -1.0], dtype=torch.float64))
    assert float(d.precipitation_rate_diagnostic(traj[1], traj[0])) == 2.0
    assert float(d.heating_rate_diagnostic(traj[2], traj[1])) == 4.0                     # 4 levels x (+1)
    out = d.CombinedStepDiagnostics()(ModelState(state=traj[2], memory=traj[1]))
    assert set(out) == {"P_minus_E_rate", "heating_rate", "total_energy", "dry_air_mass"}
    assert float(out["P_minus_E_rate"]) == -1.0


def test_conv_layers_accept_the_reference_vocabulary():
    from tornado_gcm_b200.neural.standard_layers import CnnLevel, ConvLonLat
    from tornado_gcm_b200.neural.towers import Conv2DTower, VerticalConvTower

    torch.manual_seed(0)
    t = VerticalConvTower(input_channels=3, output_channels=2, hidden_channels=[4, 4], kernel_size=3,
                          checkpoint_tower=True)
    x = torch.randn(3, 8, 5, 4, requires_grad=True)
    y = t(x)
    assert y.shape == (2, 8, 5, 4)
    y.sum().backward()
    assert x.grad is not None and all(p.grad is not None for p in t.parameters())
    c2 = Conv2DTower(input_channels=3, output_channels=2, num_hidden_units=5, num_hidden_layers=3, use_bias=False)
    assert len(c2.layers) == 4 and c2.layers[0].conv.bias is None
    assert c2(torch.randn(3, 6, 4)).shape == (2, 6, 4)
    assert ConvLonLat(input_channels=2, output_channels=3).conv.out_channels == 3
    cnn = CnnLevel(2, 3, channels=[4], kernel_sizes=[3, 5], dilations=[1, 2])
    assert cnn.layers[1].conv.kernel_size == (5,) and cnn.layers[1].conv.dilation == (2,)
    assert cnn(torch.randn(7, 2, 16)).shape == (7, 3, 16)
