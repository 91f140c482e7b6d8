"""Trace ranges, throughput log, fault-injection parsing, poison-mode switch and packaged configs (CPU)."""

import json
import pathlib

import pytest
import torch


def test_zone_range_and_throughput_log(tmp_path):
    from tornado_gcm_b200.utils.tracing import ThroughputLog, device_time_max_over_ranks, zone_range

    with torch.profiler.profile() as prof:
        with zone_range("Z1_dycore"):
            torch.ones(4).sum()
    assert any(e.name == "Z1_dycore" for e in prof.events())
    log = ThroughputLog(str(tmp_path / "tp.jsonl"))
    rec = log.record(3, 250.0, samples=4, n_gpus=1)
    assert rec["samples_per_s"] == pytest.approx(16.0)
    line = json.loads((tmp_path / "tp.jsonl").read_text().strip())
    assert line["step"] == 3 and line["n_gpus"] == 1
    assert device_time_max_over_ranks(1.5) == 1.5


def test_fault_spec_parsing():
    from tornado_gcm_b200.parallel.elastic import InjectedFault, maybe_inject_fault, parse_fault_spec

    assert parse_fault_spec("1:5:raise") == (1, 5, "raise")
    assert parse_fault_spec("") is None
    with pytest.raises(ValueError):
        parse_fault_spec("1:5:gpu_trap")
    maybe_inject_fault(0, 5, "1:5:raise")          # other rank: nothing happens
    with pytest.raises(InjectedFault):
        maybe_inject_fault(1, 5, "1:5:raise")


def test_poison_switch_python_side():
    from tornado_gcm_b200.ops import _ext

    old = _ext.poison_enabled()
    try:
        _ext.set_poison_mode(True)
        assert torch.isnan(_ext.empty(3, dtype=torch.float32, device="cpu")).all()
        assert (_ext.empty(2, dtype=torch.int32, device="cpu") == -1).all()
    finally:
        _ext.set_poison_mode(old)


def test_packaged_configs_parse():
    from tornado_gcm_b200.precision.sda import SDAConfig

    cfg_dir = pathlib.Path(__file__).resolve().parents[1] / "tornado_gcm_b200" / "configs"
    names = sorted(p.name for p in cfg_dir.glob("*.yaml"))
    for n in ("sda_debug_fp32.yaml", "sda_neuralgcm_0.7deg.yaml", "sda_neuralgcm_1.4deg.yaml",
              "sda_neuralgcm_2.8deg_full.yaml"):
        assert n in names
    for n in names:
        c = SDAConfig.from_yaml(str(cfg_dir / n))
        assert c.model.resolution and c.training.batch_size >= 1
