"""Parity of the training utilities with the reference implementation (schedules and losses)."""

import pytest
import torch

pytestmark = pytest.mark.oracle


def _traj(seed, k=3):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(2, 4, 5, generator=g, dtype=torch.float64) for _ in range(k)]


def _states(seed, mod, k=2):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    return [mod.State(r(3, 5, 4), r(3, 5, 4), r(3, 5, 4), r(1, 5, 4), {"specific_humidity": r(3, 5, 4)})
            for _ in range(k)]


def test_learning_rate_schedules_match(ref):
    from tornado_gcm_b200.training import schedules as ours

    rs = ref.import_module("tornado_gcm.training.schedules")
    cases = [
        ("CosineDecaySchedule", dict(base_lr=1e-3, warmup_steps=10, total_steps=100, min_lr=1e-5)),
        ("ExponentialDecaySchedule", dict(init_value=1e-3, transition_steps=20, decay_rate=0.5, transition_begin=5,
                                          staircase=True, end_value=1e-5)),
        ("WarmupExponentialDecaySchedule", dict(init_value=0.0, peak_value=1e-3, warmup_steps=10,
                                                transition_steps=30, decay_rate=0.3)),
        ("DelayedConstantSchedule", None),
    ]
    for name, kw in cases:
        if kw is None:
            continue
        a, b = getattr(ours, name)(**kw), getattr(rs, name)(**kw)
        for step in (0, 1, 5, 9, 10, 11, 37, 99, 100, 250):
            assert a(step) == pytest.approx(b(step), rel=1e-12, abs=1e-15), (name, step)
    pr_a = ours.ProgressiveRolloutSchedule(total_steps=1000)
    pr_b = rs.ProgressiveRolloutSchedule(total_steps=1000)
    for step in (0, 199, 200, 499, 500, 799, 800, 999):
        assert pr_a.get_rollout(step) == pr_b.get_rollout(step)
        assert pr_a.get_rollout(step, max_available=6) == pr_b.get_rollout(step, max_available=6)


def test_trajectory_losses_match(ref):
    from tornado_gcm_b200.training import losses as ours

    rl = ref.import_module("tornado_gcm.training.losses")
    p, t = _traj(0), _traj(1)
    for name in ("TrajectoryMSE", "TrajectoryMAE"):
        a, b = getattr(ours, name)()(p, t), getattr(rl, name)()(p, t)
        torch.testing.assert_close(a, b, rtol=1e-12, atol=1e-14, msg=name)
    from tornado_gcm_b200.core import primitive_equations as pe

    rpe = ref.import_module("tornado_gcm.core.primitive_equations")
    ps, ts = _states(2, pe), _states(3, pe)
    rps, rts = _states(2, rpe), _states(3, rpe)
    torch.testing.assert_close(ours.TrajectoryMSE()(ps, ts), rl.TrajectoryMSE()(rps, rts), rtol=1e-12, atol=1e-14)
    e = torch.tensor([1.0, 1.01, 0.98, 1.02], dtype=torch.float64)
    # FP64 math on both sides; the reference returns float32 always, this framework the input's dtype
    for name in ("EnergyConservationLoss", "MassConservationLoss"):
        a, b = getattr(ours, name)()(e), getattr(rl, name)()(e)
        assert a.dtype == torch.float64
        torch.testing.assert_close(a.float(), b, rtol=1e-6, atol=1e-12, msg=name)
    pr = torch.tensor([0.1, -0.2, 0.3], dtype=torch.float64)
    ev = torch.tensor([-0.1, 0.05, -0.3], dtype=torch.float64)
    torch.testing.assert_close(ours.HydrologicalClosureLoss()(pr, ev), rl.HydrologicalClosureLoss()(pr, ev))
    phys_a = ours.PhysicsConstrainedLoss(warmup_steps=1)
    phys_b = rl.PhysicsConstrainedLoss(warmup_steps=1)
    for step in (0, 5):
        a = phys_a(predictions=p, targets=t, energies=e, masses=e, precipitation=pr, evaporation=ev, step=step)
        b = phys_b(predictions=p, targets=t, energies=e, masses=e, precipitation=pr, evaporation=ev, step=step)
        torch.testing.assert_close(a["total"].double(), b["total"].double(), rtol=1e-6, atol=1e-12)


def test_ensemble_and_bias_losses_match(ref):
    from tornado_gcm_b200.training import losses as ours

    rl = ref.import_module("tornado_gcm.training.losses")
    g = torch.Generator().manual_seed(5)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    ens = [{"a": r(4, 3, 6), "b": r(4, 2, 6)} for _ in range(2)]
    tgt = [{"a": r(3, 6), "b": r(2, 6)} for _ in range(2)]
    w = {"a": 2.0}
    torch.testing.assert_close(ours.CRPSLoss(variable_weights=w)(ens, tgt), rl.CRPSLoss(variable_weights=w)(ens, tgt))
    preds = [{"a": r(3, 6), "b": r(2, 6)} for _ in range(2)]
    for name in ("SpectralNormMatchingLoss", "BatchMeanBiasLoss"):
        a = getattr(ours, name)(variable_weights=w)(preds, tgt)
        b = getattr(rl, name)(variable_weights=w)(preds, tgt)
        torch.testing.assert_close(a, b, rtol=1e-10, atol=1e-12, msg=name)


def test_spectral_filters_match(ref):
    import numpy as np

    from tornado_gcm_b200.core import filtering, spherical_harmonic as sh

    rf = ref.import_module("tornado_gcm.core.filtering")
    g, rg = sh.Grid.T21(), ref.spherical_harmonic.Grid.T21()
    x = torch.randn(3, *g.modal_shape, dtype=torch.float64)
    for args in ((16.0, 18, 0.0), (4.0, 3, 0.4)):
        a = filtering.exponential_filter(g, *args)(x)
        b = rf.exponential_filter(rg, *args)(x)
        torch.testing.assert_close(a, b, rtol=1e-12, atol=1e-14)
    a = filtering.horizontal_diffusion_filter(g, -0.01, 2)(x)
    b = rf.horizontal_diffusion_filter(rg, -0.01, 2)(x)
    torch.testing.assert_close(a, b, rtol=1e-12, atol=1e-14)
    assert np.isfinite(a.numpy()).all()


def test_vertical_interpolation_and_soft_clip_match(ref):
    import numpy as np

    from tornado_gcm_b200.core import sigma_coordinates as sc, vertical_interpolation as vi
    from tornado_gcm_b200.neural.transforms import SoftClip
    from tornado_gcm_b200.utils.units import SimUnits

    rvi = ref.import_module("tornado_gcm.core.vertical_interpolation")
    rsc = ref.sigma_coordinates
    rtr = ref.import_module("tornado_gcm.neural.transforms")
    levels = np.array([100.0, 200.0, 300.0, 500.0, 700.0, 850.0, 925.0, 1000.0]) * 100.0
    pc, rpc = vi.PressureCoordinates(levels), rvi.PressureCoordinates(levels)
    s, rs = sc.SigmaCoordinates.equidistant(6), rsc.SigmaCoordinates.equidistant(6)
    g = torch.Generator().manual_seed(3)
    field = torch.randn(8, 5, 4, generator=g, dtype=torch.float64)
    ps = 9.0e4 + 1.2e4 * torch.rand(5, 4, generator=g, dtype=torch.float64)
    # pressure -> sigma: the reference flattens (levels, lon, lat) as (columns, levels) with
    # ``x.reshape(-1, n_pressure)`` and so interpolates scrambled columns
    # (``core/vertical_interpolation.py:139``); this framework is checked column by column
    # against numpy instead (constant extrapolation outside the pressure range, as there).
    a = vi.interp_pressure_to_sigma({"x": field}, pc, s, ps)["x"]
    sig = np.asarray(s.centers)
    for i in range(5):
        for j in range(4):
            want = np.interp(sig * float(ps[i, j]), levels, field[:, i, j].numpy())
            np.testing.assert_allclose(a[:, i, j].numpy(), want, rtol=1e-12, atol=1e-12)
    on_sigma = torch.randn(6, 5, 4, generator=g, dtype=torch.float64)
    a = vi.interp_sigma_to_pressure({"x": on_sigma}, pc, s, ps)["x"]
    b = rvi.interp_sigma_to_pressure({"x": on_sigma}, rpc, rs, ps)["x"]
    torch.testing.assert_close(a, b, rtol=1e-12, atol=1e-12)
    src = torch.tensor([0.0, 0.2, 0.5, 1.0], dtype=torch.float64)
    dst = torch.tensor([0.0, 0.1, 0.6, 0.9, 1.0], dtype=torch.float64)
    torch.testing.assert_close(vi.conservative_regrid_weights(src, dst), rvi.conservative_regrid_weights(src, dst))
    z = torch.linspace(-40.0, 40.0, 101, dtype=torch.float64)
    torch.testing.assert_close(SoftClip(8.0, 0.5)({"z": z})["z"], rtr.SoftClip(8.0, 0.5)({"z": z})["z"],
                               rtol=1e-12, atol=1e-12)
    units = SimUnits.from_si()
    geo = 9.80616 * torch.linspace(16000.0, 100.0, 8, dtype=torch.float64)[:, None, None].expand(8, 5, 4)
    oro = torch.full((1, 5, 4), 250.0, dtype=torch.float64)
    a = vi.get_surface_pressure(pc, geo, oro, units.g if hasattr(units, "g") else 9.80616)
    b = rvi.get_surface_pressure(rpc, geo, oro, units.g if hasattr(units, "g") else 9.80616)
    torch.testing.assert_close(a, b, rtol=1e-12, atol=1e-10)


def test_feature_transforms_match(ref):
    from tornado_gcm_b200.neural import transforms as ours

    rt = ref.import_module("tornado_gcm.neural.transforms")
    g = torch.Generator().manual_seed(9)
    x = {"a": torch.randn(4, 6, 5, generator=g, dtype=torch.float64) * 3,
         "b": torch.randn(1, 6, 5, generator=g, dtype=torch.float64)}
    shifts, scales = {"a": 0.5, "b": -1.0}, {"a": 2.0, "b": 0.25}

    def same(a, b, what):
        assert set(a) == set(b), what
        for k in a:
            torch.testing.assert_close(a[k].double(), b[k].double(), rtol=1e-6, atol=1e-9, msg=f"{what}.{k}")

    for name in ("ShiftAndNormalize", "InverseShiftAndNormalize"):
        for gs in (None, 3.0):
            same(getattr(ours, name)(shifts, scales, gs)(x), getattr(rt, name)(shifts, scales, gs)(x), name)
    same(ours.InverseLevelScale(["a"], [1.0, 2.0, 4.0, 8.0])(x), rt.InverseLevelScale(["a"], [1.0, 2.0, 4.0, 8.0])(x),
         "InverseLevelScale")
    same(ours.HardClip(-1.0, 2.0)(x), rt.HardClip(-1.0, 2.0)(x), "HardClip")
    ls = {"a": torch.tensor([1.0, 0.5, 2.0, 4.0], dtype=torch.float64)}
    tt_a = ours.TendencyTransform(ls, clip_min={"a": -2.0}, clip_max={"b": 0.5})
    tt_b = rt.TendencyTransform(ls, clip_min={"a": -2.0}, clip_max={"b": 0.5})
    same(tt_a(x), tt_b(x), "TendencyTransform")


def test_physics_features_match(ref):
    """Radiation (solar geometry), pressure, latitude and velocity/prognostic features."""
    from tornado_gcm_b200.core import spherical_harmonic as sh
    from tornado_gcm_b200.neural import features as ours

    rfe = ref.import_module("tornado_gcm.neural.features")
    g = sh.Grid.T21(precision="highest")
    rg = ref.spherical_harmonic.Grid.T21()
    gen = torch.Generator().manual_seed(4)
    mask = torch.as_tensor(g.mask)
    m = lambda n: torch.randn(n, *g.modal_shape, generator=gen, dtype=torch.float64) * mask * 1e-2  # noqa: E731
    inputs = {"vorticity": m(3), "divergence": m(3), "temperature_variation": m(3),
              "log_surface_pressure": m(1),
              "sim_time": torch.tensor(1234.5, dtype=torch.float64)}

    def same(a, b, what, tol=1e-5):
        assert set(a) == set(b), (what, sorted(a), sorted(b))
        for k in a:
            x, y = torch.as_tensor(a[k]).double(), torch.as_tensor(b[k]).double()
            torch.testing.assert_close(x, y, rtol=tol, atol=tol * (float(y.abs().max()) + 1e-30), msg=f"{what}.{k}")

    for t in (0.0, 1234.5):
        inp = dict(inputs, sim_time=torch.tensor(t, dtype=torch.float64))
        same(ours.RadiationFeatures(g, 738000.0, 1.0)(inp), rfe.RadiationFeatures(rg, 738000.0, 1.0)(inp),
             "radiation")
    same(ours.LatitudeFeatures(g)(inputs), rfe.LatitudeFeatures(rg)(inputs), "latitude")
    sig = [0.1, 0.5, 0.9]
    same(ours.PressureFeatures(g, sig)(inputs), rfe.PressureFeatures(rg, sig)(inputs), "pressure")
    same(ours.VelocityAndPrognostics(g)(inputs), rfe.VelocityAndPrognostics(rg)(inputs), "velocity", tol=1e-4)


def test_storage_files_interchange_with_the_reference(ref, tmp_path):
    """Files written by either side read back on the other (exact and lossy BF16 records)."""
    from tornado_gcm_b200.precision.sda import StorageConfig as OurCfg
    from tornado_gcm_b200.precision.storage import SDAStorageManager as Ours

    rsda = ref.import_module("tornado_gcm.precision.sda")
    rman = ref.import_module("tornado_gcm.precision.storage.manager")
    g = torch.Generator().manual_seed(2)
    vars_ = {"temperature": torch.randn(3, 8, 4, generator=g), "u": torch.randn(3, 8, 4, generator=g)}
    ours = Ours(OurCfg(mode="mixed", critical_variables=["temperature"], non_critical_variables=["u"],
                       compressor="none"))
    theirs = rman.SDAStorageManager(rsda.StorageConfig(mode="exact", critical_variables=["temperature", "u"],
                                                       compressor="none"))
    ours.write(vars_, str(tmp_path / "a"), step=3)
    back = theirs.read(str(tmp_path / "a"), step=3)
    torch.testing.assert_close(back["temperature"], vars_["temperature"])
    torch.testing.assert_close(back["u"], vars_["u"].to(torch.bfloat16).float())
    theirs.write(vars_, str(tmp_path / "b"))
    back = ours.read(str(tmp_path / "b"))
    for k in vars_:
        torch.testing.assert_close(back[k], vars_[k])


def test_training_checkpoints_interchange_with_the_reference(ref, tmp_path):
    """A reference checkpoint (model, optimizer, training state, EMA) loads here and back."""
    from tornado_gcm_b200.training import checkpointing as ours

    rck = ref.import_module("tornado_gcm.training.checkpointing")
    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Linear(4, 6), torch.nn.GELU(), torch.nn.Linear(6, 2))
    opt = torch.optim.AdamW(net.parameters(), lr=1e-3)
    net(torch.randn(3, 4)).sum().backward()
    opt.step()
    ema = {n: p.detach().clone() * 0.5 for n, p in net.named_parameters()}
    rck.save_checkpoint(tmp_path / "r.pt", net, opt, rck.TrainingState(step=7, phase=2, best_val_loss=0.25), ema)
    net2 = torch.nn.Sequential(torch.nn.Linear(4, 6), torch.nn.GELU(), torch.nn.Linear(6, 2))
    opt2 = torch.optim.AdamW(net2.parameters(), lr=1e-3)
    st = ours.load_checkpoint(tmp_path / "r.pt", net2, opt2)
    assert (st.step, st.phase, st.best_val_loss) == (7, 2, 0.25)
    for a, b in zip(net.parameters(), net2.parameters()):
        torch.testing.assert_close(a, b)
    assert opt2.state_dict()["state"][0]["step"] == opt.state_dict()["state"][0]["step"]
    for k, v in ours.load_ema(tmp_path / "r.pt").items():
        torch.testing.assert_close(v, ema[k])
    ours.save_checkpoint(tmp_path / "o.pt", net2, opt2, ours.TrainingState(step=8, phase=3), ema)
    net3 = torch.nn.Sequential(torch.nn.Linear(4, 6), torch.nn.GELU(), torch.nn.Linear(6, 2))
    st3 = rck.load_checkpoint(tmp_path / "o.pt", net3)
    assert st3.step == 8 and st3.phase == 3
    for a, b in zip(net.parameters(), net3.parameters()):
        torch.testing.assert_close(a, b)


def test_reference_sda_configs_load_alike(ref):
    """Every SDA YAML of the reference parses here into the same policy, profiler, scheduler,
    accelerator, storage and sparse settings as in the reference."""
    import glob
    import os

    from tornado_gcm_b200.precision.sda import SDAConfig

    rsda = ref.import_module("tornado_gcm.precision.sda")
    root = os.path.dirname(os.path.dirname(ref.import_module("tornado_gcm.precision.sda").__file__))
    files = sorted(glob.glob(os.path.join(root, "configs", "*.yaml")))
    assert files
    for path in files:
        a, b = SDAConfig.from_yaml(path).to_dict(), rsda.SDAConfig.from_yaml(path).to_dict()
        for section in ("policy", "profiler", "scheduler", "accelerator", "storage", "sparse"):
            if section not in b:
                continue
            for k, v in b[section].items():
                if k in a.get(section, {}):
                    assert str(a[section][k]) == str(v), (os.path.basename(path), section, k, a[section][k], v)


def test_random_field_spectrum_matches_the_reference_shape(ref):
    """Same AR(1) coefficient and the same spectral shape exp(-κ l(l+1)/2); the normalisation
    differs by design (here: the nodal area-mean variance equals ``variance``)."""
    import numpy as np

    from tornado_gcm_b200.core import spherical_harmonic as sh
    from tornado_gcm_b200.neural.stochastic import GaussianRandomField

    rst = ref.import_module("tornado_gcm.neural.stochastic")
    g, rg = sh.Grid.T21(), ref.spherical_harmonic.Grid.T21()
    a = GaussianRandomField(g, correlation_time=3.0, correlation_length=0.2, variance=2.0)
    b = rst.GaussianRandomField(rg, correlation_time=3.0, correlation_length=0.2, variance=2.0)
    assert a._phi == pytest.approx(b._phi, rel=1e-15)
    ratio = (a._sigma[0] / b._sigma_n).numpy()
    np.testing.assert_allclose(ratio, ratio[0], rtol=1e-5)
    gen = torch.Generator().manual_seed(0)
    draws = torch.stack([g.to_nodal(a.sample_modal((), gen).double()) for _ in range(400)])
    w = torch.as_tensor(g.spherical_harmonics.basis.w, dtype=torch.float64)
    area_var = float((draws ** 2).mean(0).mean(0) @ w / w.sum())
    assert area_var == pytest.approx(2.0, rel=0.1)


def test_data_windows_and_forecast_starts_match(ref):
    import numpy as np

    from tornado_gcm_b200.training import data_loading as dl, evaluation as ev

    rdl = ref.import_module("tornado_gcm.training.data_loading")
    rev = ref.import_module("tornado_gcm.training.evaluation")
    t = np.concatenate([np.arange(0, 40), np.arange(43, 60), np.arange(70, 75), np.arange(90, 120)]) * 6.0
    assert dl.find_contiguous_segments(t) == rdl.find_contiguous_segments(t)
    for w, r in ((8, 0.05), (12, 0.2), (20, 0.05)):
        a = dl.gap_tolerant_sampling(t, w, r)
        b = rdl.gap_tolerant_sampling(t, w, r)
        key = lambda x: (x.start_idx, x.length, x.weight) if hasattr(x, "start_idx") else tuple(vars(x).values())  # noqa: E731
        assert a and [key(x) for x in a] == [key(x) for x in b], (w, r)
    first, last = np.datetime64("2020-01-01T00"), np.datetime64("2020-12-31T00")
    for alt in (True, False):
        np.testing.assert_array_equal(ev.get_forecast_starts_equispaced(10, first, last, alt),
                                      rev.get_forecast_starts_equispaced(10, first, last, alt))
    cands = np.arange(np.datetime64("2020-01-01T00"), np.datetime64("2020-03-01T00"), np.timedelta64(6, "h"))
    for bal in (True, False):
        np.testing.assert_array_equal(ev.get_forecast_starts_balanced(12, cands, bal),
                                      rev.get_forecast_starts_balanced(12, cands, bal))


def test_data_pipeline_helpers_match(ref):
    import numpy as np

    from tornado_gcm_b200.training import data_pipeline as dp

    rdp = ref.import_module("tornado_gcm.training.data_pipeline")
    t0 = np.datetime64("2020-01-01T00")
    times = t0 + np.arange(0, 96, 6).astype("timedelta64[h]")
    for scale in (1.0, 6.0):
        s_a = dp.datetime64_to_sim_time(times, t0, scale)
        np.testing.assert_array_equal(s_a, rdp.datetime64_to_sim_time(times, t0, scale))
        np.testing.assert_array_equal(dp.sim_time_to_datetime64(s_a, t0, scale),
                                      rdp.sim_time_to_datetime64(s_a, t0, scale))
    src_lon, src_lat = np.linspace(0, 357.5, 144), np.linspace(-90, 90, 73)
    tgt_lon, tgt_lat = np.linspace(0, 354.375, 64), np.linspace(-87.2, 87.2, 32)
    field = np.random.default_rng(1).standard_normal((3, 144, 73))
    a = dp.BilinearRegridder(src_lon, src_lat, tgt_lon, tgt_lat)
    b = rdp.BilinearRegridder(src_lon, src_lat, tgt_lon, tgt_lat)
    np.testing.assert_allclose(np.asarray(a(field)), np.asarray(b(field)), rtol=1e-10, atol=1e-12)
    lon, lat = np.linspace(0, 350, 36), np.linspace(-85, 85, 18)
    holes = np.random.default_rng(2).standard_normal((36, 18))
    holes[5:9, 3:6] = np.nan
    fa, fb = dp.NearestNaNFiller(lon, lat), rdp.NearestNaNFiller(lon, lat)
    ca, cb = fa.fill(holes), fb.fill(holes)
    assert not np.isnan(ca).any()
    np.testing.assert_allclose(np.asarray(ca), np.asarray(cb))


def test_verification_metrics_match(ref):
    """RMSE, ACC (with and without climatology) and bias per variable and lead time, on
    dict and State trajectories."""
    from tornado_gcm_b200.core import primitive_equations as pe
    from tornado_gcm_b200.training import evaluation as ev

    rev = ref.import_module("tornado_gcm.training.evaluation")
    rpe = ref.import_module("tornado_gcm.core.primitive_equations")
    g = torch.Generator().manual_seed(8)
    r = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    preds = [{"t": r(3, 6, 5), "z": r(1, 6, 5)} for _ in range(3)]
    tgts = [{"t": r(3, 6, 5), "z": r(1, 6, 5)} for _ in range(3)]
    clim = {"t": r(3, 6, 5), "z": r(1, 6, 5)}

    def same(a, b, what):
        assert set(a) == set(b), what
        for k in a:
            assert a[k] == pytest.approx(b[k], rel=1e-6, abs=1e-9), (what, k)  # fp32 metric tables here

    same(ev.compute_rmse(preds, tgts), rev.compute_rmse(preds, tgts), "rmse")
    same(ev.compute_bias(preds, tgts), rev.compute_bias(preds, tgts), "bias")
    same(ev.compute_anomaly_correlation(preds, tgts), rev.compute_anomaly_correlation(preds, tgts), "acc")
    same(ev.compute_anomaly_correlation(preds, tgts, clim), rev.compute_anomaly_correlation(preds, tgts, clim),
         "acc-clim")
    same(ev.compute_rmse(preds, tgts, ["t"]), rev.compute_rmse(preds, tgts, ["t"]), "rmse-filter")
    gen_state = torch.Generator().manual_seed(11)
    rr = lambda *s: torch.randn(*s, generator=gen_state, dtype=torch.float64)  # noqa: E731
    raw = [(rr(2, 4, 3), rr(2, 4, 3), rr(2, 4, 3), rr(1, 4, 3)) for _ in range(4)]
    ours_s = [pe.State(*x, {}) for x in raw]
    ref_s = [rpe.State(*x, {}) for x in raw]
    same(ev.compute_rmse(ours_s[:2], ours_s[2:]), rev.compute_rmse(ref_s[:2], ref_s[2:]), "rmse-state")


def test_precision_monitor_and_zone_casts_match(ref):
    from tornado_gcm_b200.precision import monitor as mon, zone_cast as zc
    from tornado_gcm_b200.precision.policy import PrecisionPolicy, PrecisionZone

    rmon = ref.import_module("tornado_gcm.precision.monitor")
    rzc = ref.import_module("tornado_gcm.precision.zone_cast")
    rpol = ref.import_module("tornado_gcm.precision.policy")
    g = torch.Generator().manual_seed(6)
    x = torch.randn(4, 8, 5, generator=g, dtype=torch.float64) * 10
    x[0, 0, 0] = float("nan")
    a, b = mon.PrecisionMonitor(), rmon.PrecisionMonitor()
    for m in (a, b):
        m.audit_zone_transfer("Z1_to_Z3", x, x.to(torch.bfloat16))
        m.step()
        m.audit_conservation(torch.tensor(1.0), torch.tensor(1.0 + 3e-7), torch.tensor(2.0), torch.tensor(2.0 - 1e-6))
    sa, sb = a.summary(), b.summary()
    assert set(sb) <= set(sa)
    for k in sb:
        assert sa[k] == pytest.approx(sb[k], rel=1e-5, abs=1e-12, nan_ok=True), k
    ops = (torch.randn(3, 4, generator=g), torch.randn(4, 5, generator=g, dtype=torch.float64))
    torch.testing.assert_close(zc.einsum_highest("ij,jk->ik", *ops), rzc.einsum_highest("ij,jk->ik", *ops))
    y = torch.randn(6, generator=g)
    for src, dst in ((PrecisionZone.Z1_DYNAMICS_CORE, PrecisionZone.Z3_NEURAL_NETWORK),
                     (PrecisionZone.Z3_NEURAL_NETWORK, PrecisionZone.Z2_CONSERVATION_FIXER)):
        rs, rd = getattr(rpol.PrecisionZone, src.name), getattr(rpol.PrecisionZone, dst.name)
        oa = zc.zone_cast(y, src, dst, PrecisionPolicy())
        ob = rzc.zone_cast(y, rs, rd, rpol.PrecisionPolicy())
        assert oa.dtype == ob.dtype
        torch.testing.assert_close(oa, ob)


def test_multi_adam_groups_and_gradient_cuts_match(ref):
    from tornado_gcm_b200.training import optimization as ours

    ro = ref.import_module("tornado_gcm.training.optimization")
    torch.manual_seed(0)
    model = torch.nn.ModuleDict({"encoder": torch.nn.Linear(3, 4), "physics_net": torch.nn.Linear(4, 4),
                                 "decoder": torch.nn.Linear(4, 2)})
    keys, lrs = ("encoder", "REGEX_^phys"), (1e-3, 3e-4)
    a = ours.multi_adam(model, keys, lrs, default_learning_rate=5e-5, weight_decay=0.1)
    b = ro.multi_adam(model, keys, lrs, default_learning_rate=5e-5, weight_decay=0.1)
    ga = sorted((g["lr"], g.get("weight_decay"), tuple(sorted(id(p) for p in g["params"]))) for g in a.param_groups)
    gb = sorted((g["lr"], g.get("weight_decay"), tuple(sorted(id(p) for p in g["params"]))) for g in b.param_groups)
    assert ga == gb
    with pytest.raises(Exception):
        ours.multi_adam(model, ("nothing",), (1e-3,))
    w = torch.nn.Parameter(torch.tensor(1.3))
    step = lambda s: s * w + 0.1  # noqa: E731
    x0 = torch.tensor(0.5)
    ta = ours.StopGradientTrajectory([2]).rollout(step, x0, 4)
    tb = ro.StopGradientTrajectory([2]).rollout(step, x0, 4)
    ga_, = torch.autograd.grad(sum(ta), [w])
    gb_, = torch.autograd.grad(sum(tb), [w])
    torch.testing.assert_close(ga_, gb_)
    torch.testing.assert_close(torch.stack(list(ta)), torch.stack(list(tb)))


def test_network_state_dicts_interchange_with_the_reference(ref):
    """Reference layers' weights load into this framework's layers with strict key matching and
    give the same outputs (the towers of a reference checkpoint keep working here)."""
    import torch.nn.functional as F

    from tornado_gcm_b200.neural import standard_layers as ours
    from tornado_gcm_b200.neural import towers as our_towers

    rsl = ref.import_module("tornado_gcm.neural.standard_layers")
    rtw = ref.import_module("tornado_gcm.neural.towers")
    torch.manual_seed(3)
    pairs = [
        (rsl.Mlp(7, 3, intermediate_sizes=[5, 6], activation=F.gelu),
         ours.Mlp(7, 3, intermediate_sizes=[5, 6], activation=F.gelu), (4, 7)),
        (rsl.ConvLevel(3, 5, kernel_size=3), ours.ConvLevel(3, 5, kernel_size=3), (2, 3, 8)),
        (rsl.ConvLonLat(3, 4, (3, 3)), ours.ConvLonLat(3, 4, (3, 3)), (3, 8, 6)),
        (rtw.VerticalConvTower(3, 2, [4, 4], kernel_size=3), our_towers.VerticalConvTower(3, 2, [4, 4], kernel_size=3),
         (3, 8, 5, 4)),
    ]
    for theirs, mine, shape in pairs:
        mine.load_state_dict(theirs.state_dict(), strict=True)
        x = torch.randn(*shape)
        with torch.no_grad():
            torch.testing.assert_close(mine(x), theirs(x), msg=type(mine).__name__)


def test_modal_div_curl_parameterization_matches(ref):
    """The modal parameterization of the reference benchmark arm: reference weights in this
    framework's module, same tendencies (forcings appended, div/curl back to modal)."""
    import torch.nn.functional as F

    from tornado_gcm_b200.core import primitive_equations as pe, spherical_harmonic as sh
    from tornado_gcm_b200.neural.parameterizations import ModalNeuralDivCurlParameterization
    from tornado_gcm_b200.neural.standard_layers import Mlp
    from tornado_gcm_b200.neural.towers import ForwardTower

    rsl = ref.import_module("tornado_gcm.neural.standard_layers")
    rtw = ref.import_module("tornado_gcm.neural.towers")
    rpa = ref.import_module("tornado_gcm.neural.parameterizations")
    rpe = ref.import_module("tornado_gcm.core.primitive_equations")
    n = 3
    g, rg = sh.Grid.T21(precision="highest"), _ref_grid_fp64_like(ref)
    c_in, c_out = 3 * n + 1 + 2, 3 * n + 1
    torch.manual_seed(0)
    rnet = rtw.ForwardTower(rsl.Mlp(c_in, c_out, intermediate_sizes=[16], activation=F.gelu))
    net = ForwardTower(Mlp(c_in, c_out, intermediate_sizes=[16], activation=F.gelu))
    net.load_state_dict(rnet.state_dict(), strict=True)
    a = ModalNeuralDivCurlParameterization(g, net, n, fwd_dtype=torch.float32)
    b = rpa.ModalNeuralDivCurlParameterization(rg, rnet, n, fwd_dtype=torch.float32)
    gen = torch.Generator().manual_seed(1)
    mask = torch.as_tensor(g.mask)
    m = lambda k: (torch.randn(k, *g.modal_shape, generator=gen) * mask * 1e-2).double()  # noqa: E731
    vals = (m(n), m(n), m(n), m(1))
    forc = {"sst": torch.rand(*g.nodal_shape, generator=gen).double(), "ice": torch.rand(1, *g.nodal_shape,
                                                                                         generator=gen).double()}
    with torch.no_grad():
        ta = a(pe.State(*vals, {}), forcings=forc)
        tb = b(rpe.State(*vals, {}), forcings=forc)
    for f in ("vorticity", "divergence", "temperature_variation", "log_surface_pressure"):
        x, y = getattr(ta, f).double(), getattr(tb, f).double()
        assert float(y.abs().max()) > 0, f
        torch.testing.assert_close(x, y, rtol=1e-4, atol=1e-4 * float(y.abs().max()), msg=f)


def _ref_grid_fp64_like(ref):
    rg = ref.spherical_harmonic.Grid.T21()
    rsh = ref.spherical_harmonic.RealSphericalHarmonics(
        longitude_wavenumbers=rg.longitude_wavenumbers, total_wavenumbers=rg.total_wavenumbers,
        longitude_nodes=rg.longitude_nodes, latitude_nodes=rg.latitude_nodes,
        latitude_spacing=rg.latitude_spacing, einsum_fn=ref.spherical_harmonic.einsum_highest)
    rg.__dict__["spherical_harmonics"] = rsh
    return rg


def test_field_utilities_match(ref):
    from tornado_gcm_b200.neural import field_utils as fu

    rfu = ref.import_module("tornado_gcm.neural.field_utils")
    g = torch.Generator().manual_seed(21)
    x = torch.randn(2, 5, 6, 4, generator=g, dtype=torch.float64)
    refv = torch.linspace(200.0, 290.0, 5, dtype=torch.float64)
    w = torch.rand(5, generator=g, dtype=torch.float64)
    cases = [
        ("reconstruct_1d_field_from_ref_values", (x, refv)),
        ("extract_1d_field_perturbation", (x, refv)),
        ("slice_along_axis", (x, 1, 3)),
        ("pad_along_axis", (x, 1, 2)),
        ("weighted_vertical_mean", (x, w)),
        ("repeat_surface_to_volume", (x[:, :1], 4)),
        ("vertical_flip", (x,)),
    ]
    for name, args in cases:
        torch.testing.assert_close(getattr(fu, name)(*args), getattr(rfu, name)(*args), msg=name)


def test_stream_norm_and_modal_filter_modules_match(ref):
    from tornado_gcm_b200.core import spherical_harmonic as sh
    from tornado_gcm_b200.neural.normalizations import StreamNorm
    from tornado_gcm_b200.neural.spatial_filters import ComposedFilter, ExponentialModalFilter, \
        HorizontalDiffusionFilter

    rn = ref.import_module("tornado_gcm.neural.normalizations")
    rsf = ref.import_module("tornado_gcm.neural.spatial_filters")
    g = torch.Generator().manual_seed(13)
    a, b = StreamNorm(6, momentum=0.1), rn.StreamNorm(6, momentum=0.1)
    for _ in range(3):
        x = torch.randn(5, 4, 6, generator=g) * 2 + 1
        torch.testing.assert_close(a(x), b(x))
    a.eval(), b.eval()
    x = torch.randn(3, 6, generator=g)
    torch.testing.assert_close(a(x), b(x))
    torch.testing.assert_close(a.running_var, b.running_var)
    grid, rgrid = sh.Grid.T21(), ref.spherical_harmonic.Grid.T21()
    m = torch.randn(2, *grid.modal_shape, generator=g)
    fa = ComposedFilter(ExponentialModalFilter(grid, 8.0, 6, 0.3), HorizontalDiffusionFilter(grid, 0.02, 2))
    fb = rsf.ComposedFilter(rsf.ExponentialModalFilter(rgrid, 8.0, 6, 0.3), rsf.HorizontalDiffusionFilter(rgrid, 0.02, 2))
    torch.testing.assert_close(fa(m), fb(m))
