"""HPS level 1 (sensitivity profiling) and level 2 (zone discovery) on CPU."""

import math

import numpy as np
import pytest
import torch

from tornado_gcm_b200.precision.sensitivity import (ModuleSensitivity, SensitivityMap, SensitivityProfiler,
                                                    default_conservation_validator)
from tornado_gcm_b200.precision.zone_discovery import (DiscoveryResult, ModuleGraph, ZoneDiscovery,
                                                       compare_with_pzha, detect_monotonicity_violations,
                                                       lattice_prune)


class _Toy(torch.nn.Module):
    """Linear 'model' on a State-like object: step(x) = A x with a sensitive and a tolerant part."""

    def __init__(self):
        super().__init__()
        self.sensitive = torch.nn.Linear(8, 8, bias=False, dtype=torch.float64)
        self.tolerant = torch.nn.Linear(8, 8, bias=False, dtype=torch.float64)
        with torch.no_grad():
            self.sensitive.weight.copy_(torch.eye(8, dtype=torch.float64) * (1 + 1.0 / 3.0))
            self.tolerant.weight.zero_()
            self.tolerant.weight[0, 0] = 1.0  # exactly representable in bf16

    def step(self, s, forcings=None):
        from tornado_gcm_b200.core.primitive_equations import State

        f = lambda t: self.sensitive(t) * 0.75 + self.tolerant(t) * 1e-3
        return State(f(s.vorticity), f(s.divergence), s.temperature_variation, s.log_surface_pressure, {})


def _state():
    from tornado_gcm_b200.core.primitive_equations import State

    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, 8, generator=g, dtype=torch.float64)
    return State(x, x.clone(), x.clone(), torch.ones(1, 8, dtype=torch.float64), {})


def test_sensitivity_profiler_ranks_modules():
    model = _Toy()
    prof = SensitivityProfiler(model)
    smap = prof.run_hierarchical(_state(), n_steps=20, refine_threshold=10.0)
    assert set(smap.modules) == {"sensitive", "tolerant"}
    assert smap.sensitivity_ranking[0][0] == "sensitive"
    assert smap.modules["tolerant"].drift < 1e-12 < smap.modules["sensitive"].drift
    rec = smap.get_zone_recommendation()
    assert rec["tolerant"] == "tolerant"
    # parameters restored exactly after profiling
    assert float(model.sensitive.weight[0, 0]) == 1 + 1.0 / 3.0
    curve = prof.profile_module_multi_dtype("sensitive", [torch.bfloat16, torch.float16, torch.float32], _state(),
                                            smap.baseline_metrics, 20)
    assert curve[0].drift > curve[2].drift
    assert "Ranking" in smap.summary_str()


def test_zone_perturbation_on_hybrid_model():
    from tornado_gcm_b200.models.builders import build_hybrid_gcm

    gcm, data = build_hybrid_gcm("5.6deg", "cpu")
    model = gcm.model
    enc = gcm.encoder
    x0 = {k: (v - getattr(enc, f"mean_{k}")) / getattr(enc, f"std_{k}") for k, v in data.sample(1, 0).items()}
    forc = gcm.normalize_forcings(data.forcings(1))
    with torch.no_grad():
        st = enc(x0, forc)
    prof = SensitivityProfiler(model)
    smap = prof.run_zone_perturbation(st, n_steps=2, forcings=forc)
    assert set(smap.modules) == {"zone:Z1_dynamics", "zone:Z2_fixer", "zone:Z3_neural"}
    assert all(math.isfinite(ms.drift) for ms in smap.modules.values())
    assert next(model.parameters()).dtype == torch.float32  # restored


def _map(drifts):
    m = SensitivityMap(n_steps=1)
    for k, v in drifts.items():
        m.modules[k] = ModuleSensitivity(k, v)
    return m


def test_zone_discovery_separates_decades():
    smap = _map({"a": 1e-6, "b": 2e-6, "c": 1e-5, "d": 0.5, "e": 0.7, "f": 3e-3, "g": 5e-3})
    res = ZoneDiscovery(smap, ModuleGraph.from_execution_order(list("abcdefg"))).discover(max_zones=4)
    zone = res.module_zone_map
    assert zone["d"] == zone["e"] and zone["a"] == zone["b"] and zone["d"] != zone["a"]
    by = {z.zone_id: z for z in res.zones}
    assert by[zone["d"]].recommended_precision == "FP64"
    assert by[zone["a"]].recommended_precision == "BF16"
    assert res.estimated_cast_cost >= 1
    pol = DiscoveryResult(res.zones, res.k, module_zone_map=zone).to_policy()
    assert pol.z0_dtype == torch.float64
    assert "Zone" in res.summary_str()


def test_pzha_comparison_monotonicity_and_lattice():
    smap = _map({"parameterization": 1e-5, "dycore": 5e-3, "conservation_fixer": 0.3, "filters": 0.2})
    res = ZoneDiscovery(smap, ModuleGraph.for_neuralgcm()).discover()
    text = compare_with_pzha(res, smap)
    assert "Agreement with PZHA" in text
    bf, f32, f64 = "torch.bfloat16", "torch.float32", "torch.float64"
    runs = [{"config_id": "lo", "zone_dtypes": [bf, bf], "drift": 1.0},
            {"config_id": "hi", "zone_dtypes": [f32, bf], "drift": 2.0},
            {"config_id": "ok", "zone_dtypes": [bf, f32], "drift": 0.5}]
    v = detect_monotonicity_violations(runs)
    assert len(v) == 1 and v[0]["config_high"] == "hi" and v[0]["zone_changed"] == 0
    configs = [(a, b) for a in (bf, f32, f64) for b in (bf, f32, f64)]
    kept = lattice_prune(configs, {(f32, f32): 5.0, (f64, f64): 0.1}, threshold=1.0)
    assert (bf, bf) not in kept and (bf, f32) not in kept and (f64, f64) in kept and (f64, bf) in kept


def test_hps_plots_are_written(tmp_path):
    from tornado_gcm_b200.precision.hps_visualization import plot_hps_results

    smap = _map({"a": 1e-6, "b": 1e-2, "c": 0.5, "d": float("inf")})
    res = ZoneDiscovery(smap).discover()
    paths = plot_hps_results(smap, res, tmp_path, {"T21": (22, 2), "TL63": (64, 3)})
    assert len(paths) == 4
    for p in paths:
        assert p.suffix == ".svg" and p.read_text().startswith("<svg")
