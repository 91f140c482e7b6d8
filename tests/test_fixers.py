"""Conservation fixers: the FP64-accumulating fixer kernel (CPU twin) against
the torch restatement and the reference ``LiteConservationFixer``; values and
gradients."""

import numpy as np
import pytest
import torch

from tornado_gcm_b200.core import primitive_equations as pe
from tornado_gcm_b200.neural import fixers
from tornado_gcm_b200.ops import _ext

needs_ext = pytest.mark.skipif(not _ext.available(), reason="extension not built")


def _state(seed, B=3, n=4, M2=11, L=6, t00=50.0):
    g = torch.Generator().manual_seed(seed)
    mk = lambda c, s: torch.randn(B, c, M2, L, generator=g, dtype=torch.float64) * s
    temp = mk(n, 1.0)
    temp[..., 0, 0] += t00
    return pe.State(mk(n, 0.1), mk(n, 0.05), temp, mk(1, 0.01), {"q": mk(n, 1e-3)}, 0.0)


def _torch_lite(st, before, fm=True, fe=True):
    f = fixers.LiteConservationFixer(fm, fe)
    if fm:
        st = fixers._mass_fix(st, before)
    if fe:
        deficit = fixers.compute_total_energy_lite(before) - fixers.compute_total_energy_lite(st)
        st = fixers._energy_fix(st, deficit)
    return st


@needs_ext
@pytest.mark.parametrize("fm,fe", [(True, True), (True, False), (False, True)])
def test_packed_fix_matches_torch(fm, fe):
    from tornado_gcm_b200.ops import fixers as fops

    st = _state(0).tree_map(lambda t: t.float())
    before = _state(1).tree_map(lambda t: t.float())
    out = fops.lite_fix(st, before, fm, fe)
    ref = _torch_lite(st, before, fm, fe)
    for a, b in zip(out.tensors(), ref.tensors()):
        torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-6)


@needs_ext
def test_packed_fix_skips_when_discriminant_negative():
    from tornado_gcm_b200.ops import fixers as fops

    st = _state(0, t00=0.5).tree_map(lambda t: t.float())
    before = st.tree_map(lambda t: t * 0.1)  # big energy loss → negative discriminant
    out = fops.lite_fix(st, before, False, True)
    torch.testing.assert_close(out.temperature_variation, st.temperature_variation)


@needs_ext
def test_packed_fix_gradients_match_torch_autograd():
    from tornado_gcm_b200.ops import fixers as fops
    from tornado_gcm_b200.ops import spectral

    n = 4
    st = _state(2).tree_map(lambda t: t.float())
    before = _state(3).tree_map(lambda t: t.float())
    keys = ("q",)
    y = spectral.pack_state(st, keys).requires_grad_(True)
    yb = spectral.pack_state(before, keys).requires_grad_(True)
    out = fops.packed_fix(y, yb, n)
    w = torch.randn_like(out)
    gy, gyb = torch.autograd.grad((out * w).sum(), [y, yb])

    y64 = y.detach().double().requires_grad_(True)
    yb64 = yb.detach().double().requires_grad_(True)
    ref = spectral.pack_state(_torch_lite(spectral.unpack_state(y64, n, keys), spectral.unpack_state(yb64, n, keys)),
                              keys)
    ry, ryb = torch.autograd.grad((ref * w.double()).sum(), [y64, yb64])
    torch.testing.assert_close(gy.double(), ry, rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(gyb.double(), ryb, rtol=1e-4, atol=1e-6)


@pytest.mark.oracle
@needs_ext
def test_lite_fixer_matches_reference(ref):
    """Single sample (the reference sums over everything; one sample is its case)."""
    from tornado_gcm_b200.ops import fixers as fops

    rfix = ref.import_module("tornado_gcm.neural.fixers")
    rpe = ref.import_module("tornado_gcm.core.primitive_equations")
    st = _state(4, B=1).tree_map(lambda t: t[0].float())
    before = _state(5, B=1).tree_map(lambda t: t[0].float())
    mk = lambda s: rpe.State(vorticity=s.vorticity, divergence=s.divergence, temperature_variation=s.temperature_variation,
                             log_surface_pressure=s.log_surface_pressure, tracers=s.tracers, sim_time=s.sim_time)
    r = rfix.LiteConservationFixer()(mk(st), mk(before))
    out = fops.lite_fix(st.tree_map(lambda t: t[None]), before.tree_map(lambda t: t[None]), energy_split="reference")
    torch.testing.assert_close(out.temperature_variation[0], r.temperature_variation, rtol=1e-6, atol=1e-5)
    torch.testing.assert_close(out.log_surface_pressure[0], r.log_surface_pressure, rtol=1e-6, atol=1e-7)


@needs_ext
@pytest.mark.parametrize("n", [4, 32])
def test_energy_split_restores_the_proxy_exactly(n):
    """Splitting the deficit over the levels restores E exactly; the reference formula adds (n-1)·D too much."""
    from tornado_gcm_b200.ops import fixers as fops

    st = _state(6, n=n).tree_map(lambda t: t.float())
    before = pe.State(st.vorticity * 3.0, st.divergence, st.temperature_variation, st.log_surface_pressure,
                      st.tracers, 0.0)  # the step lost vorticity energy: deficit > 0
    e = lambda s: fixers.compute_total_energy_lite(s)
    D = e(before) - e(st)
    assert bool((D > 0).all())
    split = fops.lite_fix(st, before, False, True, "levels")
    torch.testing.assert_close(e(split), e(before), rtol=1e-6, atol=0)
    refm = fops.lite_fix(st, before, False, True, "reference")
    torch.testing.assert_close(e(refm) - e(before), (n - 1) * D, rtol=1e-4, atol=0)

