"""The dycore column kernel and implicit operators (CPU twin of the CUDA code)
against the torch implementation and torch autograd."""

import numpy as np
import pytest
import torch

from tornado_gcm_b200.ops import _ext
from tornado_gcm_b200.ops import dycore as dyops
from tornado_gcm_b200.core import spherical_harmonic as sh, sigma_coordinates as sc
from tornado_gcm_b200.core import coordinate_systems as cs, primitive_equations as pe
from tornado_gcm_b200.utils.units import SimUnits

pytestmark = pytest.mark.skipif(not _ext.available(), reason="extension not built")


def _eq(humidity=True, clouds=True, n=6, nt=3):
    g = sh.Grid.T21(precision="highest")
    coords = cs.CoordinateSystem(g, sc.SigmaCoordinates.equidistant(n))
    oro = torch.zeros(g.modal_shape)
    hk = "specific_humidity" if humidity else None
    ck = ("specific_cloud_ice_water_content", "specific_cloud_liquid_water_content") if clouds else None
    return pe.PrimitiveEquationsSigma(np.linspace(210, 290, n), oro, coords, SimUnits.from_si(),
                                      humidity_key=hk, cloud_keys=ck)


def _inputs(eq, B, tracer_keys, rng):
    n = eq.vertical.layers
    I, J = eq.grid.nodal_shape
    inp = {k: torch.tensor(rng.standard_normal((B, n, I, J)) * s) for k, s in
           [("vort", 1e-1), ("div", 1e-2), ("temp", 1.0), ("u", 0.5), ("v", 0.5)]}
    inp["tracers"] = {k: torch.tensor(np.abs(rng.standard_normal((B, n, I, J))) * 1e-3) for k in tracer_keys}
    inp["gx"] = torch.tensor(rng.standard_normal((B, 1, I, J)) * 1e-2)
    inp["gy"] = torch.tensor(rng.standard_normal((B, 1, I, J)) * 1e-2)
    if eq.humidity:
        inp["qx"] = torch.tensor(rng.standard_normal((B, n, I, J)) * 1e-4)
        inp["qy"] = torch.tensor(rng.standard_normal((B, n, I, J)) * 1e-4)
        inp["lap_lnps"] = torch.tensor(rng.standard_normal((B, 1, I, J)) * 1e-2)
    return inp


@pytest.mark.parametrize("humidity,clouds", [(False, False), (True, False), (True, True)])
def test_column_forward_and_vjp(humidity, clouds):
    rng = np.random.default_rng(1)
    eq = _eq(humidity, clouds)
    keys = ["specific_cloud_ice_water_content", "specific_cloud_liquid_water_content", "specific_humidity"] if clouds \
        else (["specific_humidity"] if humidity else ["tracer_a"])
    B = 2
    inp = _inputs(eq, B, keys, rng)
    spec = dyops.ColumnSpec.from_equation(eq, keys)
    stacked = spec.stack_inputs(inp)
    # reference in float64 with autograd
    ref_in = {k: (v.clone().requires_grad_(True) if torch.is_tensor(v) else
                  {kk: vv.clone().requires_grad_(True) for kk, vv in v.items()}) for k, v in inp.items()}
    ref_out = pe.nodal_explicit_tendencies(ref_in, eq.column_constants, eq.humidity_key, eq.cloud_keys or ())
    ref_stacked = spec.stack_outputs(ref_out)
    out = dyops.column_forward_raw(spec, stacked.float(), B)
    torch.testing.assert_close(out.double(), ref_stacked.detach(), rtol=2e-4, atol=2e-5)
    gout = torch.tensor(rng.standard_normal(tuple(out.shape)))
    (ref_stacked * gout).sum().backward()
    gin = dyops.column_vjp_raw(spec, stacked.float(), gout.float(), B)
    ref_gin = spec.stack_inputs({k: (v.grad if torch.is_tensor(v) else {kk: vv.grad for kk, vv in v.items()})
                                 for k, v in ref_in.items()})
    torch.testing.assert_close(gin.double(), ref_gin, rtol=2e-3, atol=2e-4)


@pytest.mark.parametrize("mode", [0, 2])
def test_implicit_ops_and_transposes(mode):
    rng = np.random.default_rng(2)
    eq = _eq(True, False)
    n = eq.vertical.layers
    M2, L = eq.grid.modal_shape
    B = 2
    mk = lambda lv: torch.tensor(rng.standard_normal((B, lv, M2, L)), dtype=torch.float64)
    d, t, p = mk(n), mk(n), mk(1)
    eta = 0.013
    st = pe.State(torch.zeros_like(d), d, t, p, {}, None)
    if mode == 0:
        ref = eq.implicit_inverse(st, eta)
    else:
        ref = eq.implicit_terms(st)
    od, ot, op = dyops.implicit_apply(eq, d.float(), t.float(), p.float(), eta, mode)
    torch.testing.assert_close(od.double(), ref.divergence, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(ot.double(), ref.temperature_variation, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(op.double(), ref.log_surface_pressure, rtol=1e-4, atol=1e-5)
    # transpose: <A x, y> == <x, A^T y>
    yd, yt, yp = mk(n), mk(n), mk(1)
    td, tt, tp = dyops.implicit_apply(eq, yd.float(), yt.float(), yp.float(), eta, mode + 1)
    lhs = (od.double() * yd).sum() + (ot.double() * yt).sum() + (op.double() * yp).sum()
    rhs = (d * td.double()).sum() + (t * tt.double()).sum() + (p * tp.double()).sum()
    assert abs(float(lhs - rhs)) <= 1e-4 * max(1.0, abs(float(lhs)))
