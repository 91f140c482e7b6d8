"""Forecast evaluation metrics/runners and the reanalysis preprocessing helpers (CPU)."""

import numpy as np
import pytest
import torch


def test_forecast_start_sampling():
    from tornado_gcm_b200.training.evaluation import get_forecast_starts_balanced, get_forecast_starts_equispaced

    s = get_forecast_starts_equispaced(4, np.datetime64("2020-01-01"), np.datetime64("2020-01-08"))
    assert len(s) == 4 and (s[1] - s[1].astype("datetime64[D]")).astype("timedelta64[h]").astype(int) == 12
    cand = np.arange(np.datetime64("2020-01-01T00"), np.datetime64("2020-02-01T00"), np.timedelta64(6, "h"))
    b = get_forecast_starts_balanced(8, cand)
    hours = ((b - b.astype("datetime64[D]")).astype("timedelta64[h]").astype(int))
    assert sorted(np.unique(hours, return_counts=True)[1].tolist()) == [2, 2, 2, 2]


def test_metrics_against_numpy():
    from tornado_gcm_b200.training.evaluation import compute_anomaly_correlation, compute_bias, compute_rmse

    g = torch.Generator().manual_seed(0)
    preds = [{"a": torch.randn(3, 8, 4, generator=g)} for _ in range(2)]
    tgts = [{"a": torch.randn(3, 8, 4, generator=g)} for _ in range(2)]
    r = compute_rmse(preds, tgts)["a"]
    b = compute_bias(preds, tgts)["a"]
    acc = compute_anomaly_correlation(preds, tgts)["a"]
    for k in range(2):
        p, t = preds[k]["a"].double().numpy(), tgts[k]["a"].double().numpy()
        assert r[k] == pytest.approx(np.sqrt(((p - t) ** 2).mean()))
        assert b[k] == pytest.approx((p - t).mean())
        c = t.mean()
        assert acc[k] == pytest.approx(((p - c) * (t - c)).sum() / np.sqrt(((p - c) ** 2).sum() * ((t - c) ** 2).sum()))
    w = torch.tensor([0.0, 0.0, 1.0, 1.0])
    rw = compute_rmse(preds, tgts, lat_weights=w)["a"][0]
    p, t = preds[0]["a"].double().numpy(), tgts[0]["a"].double().numpy()
    assert rw == pytest.approx(np.sqrt(((p - t)[..., 2:] ** 2).mean()))


class _Decay(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.c = torch.nn.Parameter(torch.tensor(0.5))

    def step(self, s, forcings=None):
        return {k: v * self.c for k, v in s.items()}


def test_evaluation_runner_and_benchmark():
    from tornado_gcm_b200.training.evaluation import (EvalConfig, EvaluationRunner, WeatherBenchmarkConfig,
                                                      WeatherBenchmarkRunner)

    states = [{"x": torch.full((2, 3), 0.5 ** i)} for i in range(30)]
    model = _Decay()
    runner = EvaluationRunner(model, EvalConfig(eval_cadence=2, n_eval_samples=3, rollout_steps=4))
    runner.set_eval_data(states)
    assert not runner.should_evaluate(0) and runner.should_evaluate(1)
    res = runner.evaluate()
    assert res.n_samples == 3 and max(res.rmse["x"]) < 1e-7
    runner.update_ema_params({"c": torch.tensor(0.25)})
    res_ema = runner.evaluate(use_ema=True)
    assert res_ema.rmse["x"][0] > 0 and float(model.c) == 0.5   # EMA swapped in then restored
    assert "rmse/x/t+1" in res.summary()
    bench = WeatherBenchmarkRunner(model, WeatherBenchmarkConfig(eval_cadence=1, n_eval_samples=2, forecast_hours=72,
                                                                 dt_hours=6.0))
    bench.set_eval_data(states)
    out = bench.evaluate(use_ema=False)
    assert "x" in out.day3_rmse and out.n_samples == 2


def test_time_and_forcing_helpers():
    from tornado_gcm_b200.training import data_pipeline as dp

    t = np.arange(np.datetime64("2020-01-01T00"), np.datetime64("2020-01-03T00"), np.timedelta64(6, "h"))
    st = dp.datetime64_to_sim_time(t, t[0], 6.0)
    assert st.tolist() == list(range(len(t)))
    assert (dp.sim_time_to_datetime64(st, t[0], 6.0) == t).all()
    d = dp.with_sim_time({"a": np.zeros((len(t), 1, 4, 3))}, t)
    assert d["sim_time"].shape == (len(t), 1, 1, 1)
    f = dp.DynamicDataForcing(np.arange(4.0), {"sst": np.arange(4.0)[:, None] * np.ones((4, 5))}, dt_tolerance=0.4)
    assert float(f(2.2)["sst"][0]) == 2.0 and torch.isnan(f(2.5)["sst"]).all()
    clim = dp.Climatology({"ice": np.linspace(0, 1, 365)[:, None] * np.ones((365, 3))})
    ap = dp.AnomalyPersistence({"ice": np.full(3, 0.9)}, clim, initial_dayofyear=1, clip_variables=("ice",))
    assert float(ap(365)["ice"].max()) == 1.0
    sh = dp.selective_temporal_shift({"a": np.arange(5), "b": np.arange(5)}, ["a"], 2)
    assert sh["a"].tolist() == [0, 1, 2] and sh["b"].tolist() == [2, 3, 4]


def test_bilinear_regridder_and_nan_filler():
    from tornado_gcm_b200.training.data_pipeline import BilinearRegridder, NearestNaNFiller

    slon, slat = np.arange(0, 360, 10.0), np.linspace(-85, 85, 18)
    tlon, tlat = np.arange(5, 360, 20.0), np.linspace(-80, 80, 9)
    LON, LAT = np.meshgrid(slon, slat, indexing="ij")
    f = 3.0 * LAT + 2.0                                    # linear in latitude: reproduced exactly
    out = BilinearRegridder(slon, slat, tlon, tlat)(f)
    TL = np.meshgrid(tlon, tlat, indexing="ij")[1]
    np.testing.assert_allclose(out, 3.0 * TL + 2.0, atol=1e-9)
    g = np.cos(np.deg2rad(LON))                             # periodic seam: 355° between 350° and 0°
    seam = BilinearRegridder(slon, slat, np.array([355.0]), slat)(g)
    np.testing.assert_allclose(seam[0], 0.5 * (np.cos(np.deg2rad(350)) + 1.0), atol=1e-12)
    tt = BilinearRegridder(slon, slat, tlon, tlat)(torch.as_tensor(f))
    assert torch.is_tensor(tt)
    h = LAT.copy()
    h[3, 4] = np.nan
    filled = NearestNaNFiller(slon, slat).fill(h)
    assert not np.isnan(filled).any() and abs(filled[3, 4] - LAT[3, 4]) <= 10.0
