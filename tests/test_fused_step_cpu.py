"""The fused SIL3 substep (column kernel + implicit kernels, CPU twins) against
the reference-semantics IMEX stepper, values and gradients."""

import numpy as np
import pytest
import torch

from tornado_gcm_b200.ops import _ext
from tornado_gcm_b200.ops import dycore as dyops
from tornado_gcm_b200.core import spherical_harmonic as sh, sigma_coordinates as sc, filtering
from tornado_gcm_b200.core import coordinate_systems as cs, primitive_equations as pe, time_integration as ti
from tornado_gcm_b200.utils.units import SimUnits

pytestmark = pytest.mark.skipif(not _ext.available(), reason="extension not built")


def _setup(n=5):
    g = sh.Grid.T21(precision="float32")
    coords = cs.CoordinateSystem(g, sc.SigmaCoordinates.equidistant(n))
    rng = np.random.default_rng(3)
    m, l = g.modal_mesh
    amp = np.where(g.mask, (1.0 + l) ** -1.5, 0.0)
    mk = lambda lv, s: torch.tensor(rng.standard_normal((2, lv) + g.modal_shape) * amp * s, dtype=torch.float32)
    oro = torch.tensor(rng.standard_normal(g.modal_shape) * amp * 1e-3, dtype=torch.float32)
    eq = pe.PrimitiveEquationsSigma(np.linspace(210, 290, n), oro, coords, SimUnits.from_si(),
                                    humidity_key="specific_humidity")
    st = pe.State(mk(n, 1e-1), mk(n, 1e-2), mk(n, 1.0), mk(1, 1e-2), {"specific_humidity": mk(n, 1e-3)}, 0.0)
    phys = st.tree_map(lambda x: 1e-3 * torch.randn_like(x))
    return eq, st, phys


def _reference_step(eq, st, phys, dt, filt):
    class Comb(ti.ImplicitExplicitODE):
        def explicit_terms(self, x):
            return eq.explicit_terms_reference(x) + phys

        def implicit_terms(self, x):
            return eq.implicit_terms(x)

        def implicit_inverse(self, x, s):
            return eq.implicit_inverse(x, s)

    out = ti.imex_rk_sil3(Comb(), dt)(st)
    return out.tree_map(filt)


def test_fused_sil3_matches_reference():
    eq, st, phys = _setup()
    dt = 0.02
    f = filtering.exponential_filter(eq.grid, 16.0, 18, 0.0)
    stepper = dyops.FusedSIL3(eq, dt, f.scaling)
    out = stepper.step(st, phys)
    ref = _reference_step(eq, st, phys, dt, f)
    for a, b in zip(out.tensors(), ref.tensors()):
        torch.testing.assert_close(a, b, rtol=1e-3, atol=1e-6)


def test_fused_sil3_gradients_match():
    eq, st, phys = _setup()
    dt = 0.02
    f = filtering.exponential_filter(eq.grid, 16.0, 18, 0.0)
    stepper = dyops.FusedSIL3(eq, dt, f.scaling)
    w = [torch.randn_like(t) for t in st.tensors()]

    def loss(fn):
        x = st.tree_map(lambda t: t.clone().requires_grad_(True))
        out = fn(x)
        val = sum((a * b).sum() for a, b in zip(out.tensors(), w))
        grads = torch.autograd.grad(val, x.tensors())
        return grads

    g_fused = loss(lambda x: stepper.step(x, phys))
    g_ref = loss(lambda x: _reference_step(eq, x, phys, dt, f))
    for a, b in zip(g_fused, g_ref):
        torch.testing.assert_close(a, b, rtol=2e-3, atol=1e-5)


def _packed_setup():
    eq, st, phys = _setup()
    keys = tuple(sorted(st.tracers))
    return eq, st, phys, keys


def test_spectral_recipes_match_torch_pre_post():
    from tornado_gcm_b200.ops import spectral

    eq, st, phys, keys = _packed_setup()
    y = spectral.pack_state(st, keys)
    pre = spectral.explicit_pre_recipe(eq, keys)
    ref_pre = eq.modal_pre_stack(st)
    torch.testing.assert_close(pre.apply(y), ref_pre, rtol=1e-5, atol=1e-7)
    post = spectral.explicit_post_recipe(eq, keys)
    rng = np.random.default_rng(5)
    modal = torch.tensor(rng.standard_normal((2, post.c_in) + eq.grid.modal_shape), dtype=torch.float32)
    ref_post = eq.modal_post(modal, st)
    out = post.apply(modal)
    oro = eq.grid.clip_wavenumbers(eq.orography_tendency(modal.device, modal.dtype))
    ref_packed = spectral.pack_state(ref_post, keys)
    ref_packed[:, eq.vertical.layers:2 * eq.vertical.layers] -= oro
    torch.testing.assert_close(out, ref_packed, rtol=1e-4, atol=1e-5)
    # transposes: <A x, y> == <x, A^T y>
    for r in (pre, post):
        x = torch.randn(2, r.c_in, *eq.grid.modal_shape, dtype=torch.float32)
        z = torch.randn(2, r.c_out, *eq.grid.modal_shape, dtype=torch.float32)
        lhs = (r.apply(x).double() * z.double()).sum()
        rhs = (x.double() * r.transpose().apply(z).double()).sum()
        assert abs(float(lhs - rhs)) <= 1e-4 * max(1.0, abs(float(lhs)))


def test_packed_sil3_matches_fused_values_and_grads():
    from tornado_gcm_b200.ops import spectral

    eq, st, phys, keys = _packed_setup()
    dt = 0.02
    f = filtering.exponential_filter(eq.grid, 16.0, 18, 0.0)
    ref_stepper = dyops.FusedSIL3(eq, dt, f.scaling)
    stepper = dyops.PackedSIL3(eq, dt, f.scaling, keys)
    n = eq.vertical.layers
    P = spectral.pack_state(phys, keys) + stepper.orography_packed(torch.device("cpu"))
    y0 = spectral.pack_state(st, keys).requires_grad_(True)
    out = stepper.step_packed(y0, P)
    st_ref = st.tree_map(lambda t: t.clone().requires_grad_(True))
    ref = spectral.pack_state(ref_stepper.step(st_ref, phys), keys)
    torch.testing.assert_close(out, ref, rtol=1e-3, atol=1e-6)
    w = torch.randn_like(out)
    (gy,) = torch.autograd.grad((out * w).sum(), y0)
    g_ref = torch.autograd.grad((ref * w).sum(), st_ref.tensors())
    g_ref_packed = torch.cat([g_ref[0], g_ref[1], g_ref[2], g_ref[3]] + list(g_ref[4:]), dim=-3)
    torch.testing.assert_close(gy, g_ref_packed, rtol=3e-3, atol=1e-5)


def test_packed_parameterization_matches_state_path():
    from tornado_gcm_b200.neural.parameterizations import NodalColumnParameterization
    from tornado_gcm_b200.neural.standard_layers import MlpUniform
    from tornado_gcm_b200.neural.towers import ForwardTower
    from tornado_gcm_b200.ops import spectral

    eq, st, _ = _setup()
    g, n = eq.grid, 5
    st.tracers["specific_cloud_ice_water_content"] = st.tracers["specific_humidity"] * 0.1
    keys = tuple(sorted(st.tracers))
    pkeys = ("specific_humidity",)  # the network sees a subset of the state tracers
    fk = ("orography", "sea_surface_temperature")
    torch.manual_seed(0)
    n_in = n * (3 + len(pkeys)) + 1 + len(fk)
    n_out = n * (3 + len(pkeys)) + 1
    tower = ForwardTower(MlpUniform(n_in, n_out, hidden_size=16, n_hidden_layers=2))
    p = NodalColumnParameterization(g, n, pkeys, tower, forcing_keys=fk, output_scale=torch.rand(n_out),
                                    input_scale=torch.rand(n_in), compute_dtype=torch.float32)
    forc = {k: torch.randn(2, *g.nodal_shape) for k in fk}
    ref = spectral.pack_state(p(st, forcings=forc), keys)
    y = spectral.pack_state(st, keys).requires_grad_(True)
    out = p.forward_packed(y, keys, forc)
    torch.testing.assert_close(out, ref, rtol=2e-4, atol=1e-7)
    w = torch.randn_like(out)
    (gy,) = torch.autograd.grad((out * w).sum(), y)
    st_leaves = [t.detach().clone().requires_grad_(True) for t in (st.vorticity, st.divergence,
                                                                    st.temperature_variation,
                                                                    st.log_surface_pressure)]
    trs = {k: st.tracers[k].detach().clone().requires_grad_(True) for k in keys}
    st2 = pe.State(*st_leaves, trs, 0.0)
    ref2 = spectral.pack_state(p(st2, forcings=forc), keys)
    gref = torch.autograd.grad((ref2 * w).sum(), st_leaves + [trs[k] for k in keys], allow_unused=True)
    gref = torch.cat([x if x is not None else torch.zeros_like(t)
                      for x, t in zip(gref, st_leaves + [trs[k] for k in keys])], dim=-3)
    torch.testing.assert_close(gy, gref, rtol=2e-3, atol=1e-6)


def test_bounds_checked_recipe_skips_out_of_range_terms_on_cpu():
    import copy

    from tornado_gcm_b200.ops import _ext, spectral

    if not _ext.available():
        pytest.skip("extension not built")
    eq, _, _ = _setup(4)
    rec = spectral.explicit_pre_recipe(eq, ("specific_humidity",))
    bad = copy.copy(rec)
    bad.terms = [copy.copy(t) for t in rec.terms]
    bad._dev, bad._transpose = {}, None
    bad.terms[0].pre = 99  # no such diagonal
    clean = copy.copy(rec)
    clean.terms = rec.terms[1:]
    clean._dev, clean._transpose = {}, None
    x = torch.randn(1, rec.c_in, *eq.grid.modal_shape)
    ops = _ext.require("bounds checks")
    ops.set_bounds_check(True)
    try:
        y = bad.apply(x)
    finally:
        ops.set_bounds_check(False)
    torch.testing.assert_close(y, clean.apply(x), rtol=0, atol=0)


def test_pack_of_unpacked_state_is_the_packed_tensor():
    """Re-packing an unpacked state returns the packed tensor itself (no copy, and backward
    needs no per-slice zero-fill and additions); a replaced field falls back to concatenation."""
    import dataclasses

    from tornado_gcm_b200.ops import spectral

    keys = ("a", "b")
    n = 3
    y = torch.randn(2, (3 + len(keys)) * n + 1, 5, 4, requires_grad=True)
    st = spectral.unpack_state(y * 1.0, n, keys, 0.0)
    assert spectral.pack_state(st, keys) is st._packed_src[0]
    st2 = spectral.carry_packed(st, dataclasses.replace(st, sim_time=1.0))
    assert spectral.pack_state(st2, keys) is st._packed_src[0]
    w = torch.randn_like(y)
    (g,) = torch.autograd.grad((spectral.pack_state(st2, keys) * w).sum(), y)
    torch.testing.assert_close(g, w)
    st3 = dataclasses.replace(st, vorticity=st.vorticity * 2.0)
    out = spectral.pack_state(st3, keys)
    assert out is not st._packed_src[0]
    torch.testing.assert_close(out[:, :n], 2.0 * (y[:, :n] * 1.0))
    assert spectral.pack_state(st, ("b", "a")) is not st._packed_src[0]


def test_hyperdiffusion_damps_the_truncation_wavenumber():
    """The model's hyperdiffusion filter decays every wavenumber (scaling ≤ 1, exp(-dt/τ) at the
    truncation), and the step-filter helper builds the same damping."""
    from tornado_gcm_b200.core import time_integration as ti
    from tornado_gcm_b200.models.builders import build_hybrid_gcm

    gcm, _ = build_hybrid_gcm("5.6deg", "cpu", seed=0)
    m = gcm.model
    s = np.asarray(m.hyperdiffusion_filter.scaling)
    cfg = m.config
    assert s[0] == 1.0 and np.all(s <= 1.0) and np.all(np.diff(s) <= 0)
    np.testing.assert_allclose(s[-1], np.exp(-m._inner_dt / cfg.hyperdiffusion_tau), rtol=1e-6)
    g = cfg.coords.horizontal
    f = ti.horizontal_diffusion_step_filter(g, m._inner_dt, cfg.hyperdiffusion_tau, cfg.hyperdiffusion_order)
    x = torch.ones(1, *g.modal_shape, dtype=torch.float64)
    y = f(x, x)
    assert float(y.abs().max()) <= 1.0 + 1e-12
