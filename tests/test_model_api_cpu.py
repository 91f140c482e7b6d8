"""Model facade, JAX checkpoint mapping, dynamic forcing, inference engines and
the CLI on the CPU (T21-sized cases where a model is stepped)."""

import pickle

import numpy as np
import pytest
import torch

from tornado_gcm_b200.model import jax_checkpoint_loader as jl


def _haiku_dict(comps: jl.JaxNeuralComponents, rng) -> dict:
    """Nested Haiku-style params for every tower of the components (test fixture)."""
    root = {}

    def put(path, arr):
        d = root
        parts = path.split("/")
        for p in parts[:-1]:
            d = d.setdefault(p, {})
        d[parts[-1]] = arr

    def epd(prefix, epd_mod, surface=False):
        s = "surface_model_" if surface else ""
        for part in ("encode", "decode"):
            for i, lin in enumerate(getattr(epd_mod, part).layers):
                put(f"{prefix}/{s}{part}_tower/~/mlp_uniform/~/linear_{i}/w",
                    rng.standard_normal(tuple(lin.weight.shape[::-1])).astype(np.float32))
                if lin.bias is not None:
                    put(f"{prefix}/{s}{part}_tower/~/mlp_uniform/~/linear_{i}/b",
                        rng.standard_normal(lin.bias.shape).astype(np.float32))
        for bidx, blk in enumerate(epd_mod.process_blocks):
            suffix = "" if bidx == 0 else f"_{bidx}"
            for i, lin in enumerate(blk.layers):
                put(f"{prefix}/{s}process_tower{suffix}/~/mlp_uniform/~/linear_{i}/w",
                    rng.standard_normal(tuple(lin.weight.shape[::-1])).astype(np.float32))
                put(f"{prefix}/{s}process_tower{suffix}/~/mlp_uniform/~/linear_{i}/b",
                    rng.standard_normal(lin.bias.shape).astype(np.float32))

    r = "params/stochastic_modular_step_model/~/"
    epd(r + "dimensional_learned_weatherbench_to_primitive_with_memory_encoder/~/a_nodal_mapping/~/epd_tower",
        comps.encoder_epd[0])
    epd(r + "dimensional_learned_weatherbench_to_primitive_with_memory_encoder/~/b_nodal_mapping/~/epd_tower",
        comps.encoder_epd[1])
    epd(r + "dimensional_learned_primitive_to_weatherbench_decoder/nodal_mapping/~/epd_tower", comps.decoder_epd)
    epd(r + "stochastic_physics_parameterization_step/~/physics/~/epd_tower", comps.physics_epd)
    for k, name in enumerate(("land", "sea", "ice")):
        epd(r + f"stochastic_physics_parameterization_step/~/{name}_surface", comps.surface_epd[k], surface=True)
    for i, layer in enumerate(comps.volume_conv.layers):
        suffix = "" if i == 0 else f"_{i}"
        w = layer.conv.weight
        put(r + f"stochastic_physics_parameterization_step/~/volume/~/conv_level{suffix}/w",
            rng.standard_normal((w.shape[2], w.shape[1], w.shape[0])).astype(np.float32))
        put(r + f"stochastic_physics_parameterization_step/~/volume/~/conv_level{suffix}/b",
            rng.standard_normal((w.shape[0], 1)).astype(np.float32))
    return root


def test_jax_checkpoint_roundtrip(tmp_path):
    comps = jl.JaxNeuralComponents()
    rng = np.random.default_rng(0)
    nested = _haiku_dict(comps, rng)
    path = tmp_path / "ckpt.pkl"
    with open(path, "wb") as fh:
        pickle.dump(nested, fh)
    flat = jl.load_jax_checkpoint(path)
    target = jl.JaxNeuralComponents()
    rep = jl.load_jax_weights(target, flat, strict=False)
    assert not rep["skipped"] and not rep["unmatched"]
    mapping = jl.build_weight_mapping(flat)
    sd = target.state_dict()
    for p, (key, kind) in mapping.items():
        ref = torch.as_tensor(flat[p])
        if kind == "linear_w":
            ref = ref.t()
        elif kind == "conv_w":
            ref = ref.permute(2, 1, 0)
        torch.testing.assert_close(sd[key], ref.reshape(sd[key].shape))
    loaded = set(rep["loaded"])
    assert all(k in loaded for k in sd if "positional" not in k)


def test_dynamic_forcing_nearest_row_and_nan():
    from tornado_gcm_b200.model.dynamic_data_forcing import build_dynamic_data_forcing_torch

    data = {"sim_time": np.array([0.0, 1.0, 2.0]), "sst": np.arange(3 * 4, dtype=np.float32).reshape(3, 2, 2)}
    fn = build_dynamic_data_forcing_torch(data, dt_tolerance=0.25, device="cpu")
    out = fn({}, 1.1)
    torch.testing.assert_close(out["sst"], torch.tensor(data["sst"][1]))
    assert torch.isnan(fn({}, 1.5)["sst"]).all()


def _small():
    from tornado_gcm_b200.models.builders import build_hybrid_gcm

    gcm, data = build_hybrid_gcm("5.6deg", "cpu")
    enc = gcm.encoder
    norm = lambda d: {k: (v - getattr(enc, f"mean_{k}")) / getattr(enc, f"std_{k}") for k, v in d.items()}
    return gcm, data, norm


def test_mp_inference_rollout_and_streaming():
    from tornado_gcm_b200.inference import InferenceConfig, InferenceRunner, MPInference, NumpyWriter

    gcm, data, norm = _small()
    eng = MPInference(gcm, use_graph=False)
    x0 = norm(data.sample(1, 0))
    forc = data.forcings(1)
    out = eng.rollout(x0, steps=2, forcings=forc)
    assert len(out) == 2 and set(out[0]) >= {"u", "t"}
    assert all(torch.isfinite(v).all() for v in out[-1].values())
    s0 = gcm.encoder(x0, gcm.normalize_forcings(forc))
    final, saved = eng.run_streaming(s0, 3, inner_steps=1, forcings=forc, keep_steps={1, 3}, nan_guard=True,
                                     checkpoint_interval=1)
    assert [s for s, _ in saved] == [1, 3]
    ref = eng.run(s0, 3, inner_steps=1, forcings=forc)
    torch.testing.assert_close(saved[-1][1].vorticity, ref[-1].vorticity)
    runner = InferenceRunner(eng, InferenceConfig(outer_steps=3, inner_steps=1, chunk_size=2))
    w = NumpyWriter()
    traj = runner.run(s0, writer=w)
    assert len(traj) == 3 and w.finalize()["vorticity"].shape[0] == 3


def test_inference_checkpoint_roundtrip(tmp_path):
    from tornado_gcm_b200.inference import MPInference
    from tornado_gcm_b200.training.checkpointing import export_inference_checkpoint

    gcm, _, _ = _small()
    path = tmp_path / "m.pt"
    export_inference_checkpoint(gcm, path, meta={"resolution": "5.6deg"})
    eng = MPInference.from_state_dict(torch.load(path, weights_only=True), device="cpu", use_graph=False)
    a = dict(gcm.named_parameters())
    for k, v in eng.hybrid.named_parameters():
        torch.testing.assert_close(v, a[k].to(torch.bfloat16).float())
    for k, v in eng.hybrid.named_buffers():
        torch.testing.assert_close(v, dict(gcm.named_buffers())[k])


def test_sda_inference_adaptive_and_sparse():
    from tornado_gcm_b200.inference import SDAInference
    from tornado_gcm_b200.precision.sda import SDAConfig

    gcm, data, norm = _small()
    cfg = SDAConfig()
    cfg.profiler.spectral_audit = True
    eng = SDAInference(gcm, cfg, use_graph=False)
    s0 = gcm.encoder(norm(data.sample(1, 0)), gcm.normalize_forcings(data.forcings(1)))
    f = data.forcings(1)
    traj = eng.run_adaptive(s0, 2, inner_steps=1, quality_threshold=0.0, forcings=f)
    assert eng.escalated and len(traj) == 2
    traj, stats = eng.run_sparse(s0, 2, inner_steps=1, forcings=f)
    assert 0.0 < stats["memory_savings"] < 1.0


def test_sda_trainer_and_cli(tmp_path):
    from click.testing import CliRunner

    from tornado_gcm_b200.cli import main
    from tornado_gcm_b200.precision.sda import SDAConfig
    from tornado_gcm_b200.training.sda_trainer import SDATrainer

    gcm, _, _ = _small()
    cfg = SDAConfig()
    cfg.training.rollout_steps = 1
    cfg.training.batch_size = 1
    tr = SDATrainer(gcm, cfg, total_steps=2)
    hist = tr.fit(log_every=1)
    assert len(hist) == 2 and np.isfinite(hist[-1]["loss"])
    ck = tmp_path / "c.pt"
    tr.save_checkpoint(ck)
    tr.load_checkpoint(ck)
    yaml_path = tmp_path / "cfg.yaml"
    yaml_path.write_text("model:\n  resolution: '5.6deg'\ntraining:\n  total_steps: 1\n  batch_size: 1\n"
                         "  rollout_steps: 1\n")
    res = CliRunner().invoke(main, ["train", "-c", str(yaml_path), "-k", str(tmp_path / "k.pt"), "-d", "cpu"])
    assert res.exit_code == 0, res.output
    from tornado_gcm_b200.training.checkpointing import export_inference_checkpoint
    from tornado_gcm_b200.training.synthetic import SyntheticReanalysis

    export_inference_checkpoint(gcm, tmp_path / "inf.pt", meta={"resolution": "5.6deg"})
    src = SyntheticReanalysis(gcm.model.config.coords.horizontal)
    enc = gcm.encoder
    ic = {k: (v - getattr(enc, f"mean_{k}")) / getattr(enc, f"std_{k}") for k, v in src.sample(1, 0).items()}
    ic["forcings"] = src.forcings(1)
    torch.save(ic, tmp_path / "ic.pt")
    res = CliRunner().invoke(main, ["infer", "-c", str(yaml_path), "-k", str(tmp_path / "inf.pt"), "-i",
                                    str(tmp_path / "ic.pt"), "-o", str(tmp_path / "fc.npz"), "-s", "2", "-d", "cpu",
                                    "--no-sda"])
    assert res.exit_code == 0, res.output
    assert np.load(tmp_path / "fc.npz")["t"].shape[0] == 2


def test_checkpointed_outer_steps_give_the_same_gradients():
    gcm, data, norm = _small()
    x0 = norm(data.sample(2, 0))
    tg = [norm(data.sample(2, i + 1)) for i in range(2)]
    forc = data.forcings(2)
    params = [p for p in gcm.parameters() if p.requires_grad]

    def grads(ckpt: bool):
        gcm.checkpoint_outer_steps = ckpt
        gcm.model._step_count = 0
        for p in params:
            p.grad = None
        loss = gcm.loss(x0, tg, forc)
        loss.backward()
        return float(loss), [p.grad.clone() for p in params], gcm.model._step_count

    l0, g0, n0 = grads(False)
    l1, g1, n1 = grads(True)
    gcm.checkpoint_segment = 2  # segments of 2 and 1 physics steps per 3-step block
    l2, g2, n2 = grads(True)
    gcm.checkpoint_outer_steps = False
    gcm.checkpoint_segment = 0
    assert l0 == pytest.approx(l1, rel=1e-6) and l0 == pytest.approx(l2, rel=1e-6)
    assert n0 == n1 == n2 == 2 * gcm.physics_steps_per_output  # recompute leaves the fixer counter alone
    for a, b, c in zip(g0, g1, g2):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-7)
        torch.testing.assert_close(a, c, rtol=1e-5, atol=1e-7)


def test_physics_memory_check_needs_every_core_field_and_tracer():
    from tornado_gcm_b200.models.api import _physics_memory_ok_for_epd as ok

    class _S:
        def __init__(self, tracers):
            self.tracers = tracers

    core = {k: 0 for k in ("vorticity", "divergence", "temperature_variation", "log_surface_pressure")}
    assert not ok(None, _S({})) and not ok({}, _S({})) and not ok({"vorticity": 0}, _S({}))
    assert ok(core, _S({})) and ok(object(), _S({}))
    assert not ok(core, _S({"q": 0})) and not ok({**core, "tracers": [0]}, _S({"q": 0}))
    assert ok({**core, "tracers": {"q": 0, "c": 0}}, _S({"q": 0}))


def test_sda_trainer_backward_precision_hooks():
    from tornado_gcm_b200.precision.sda import SDAConfig
    from tornado_gcm_b200.training.sda_trainer import SDATrainer

    gcm, _, _ = _small()
    cfg = SDAConfig()
    cfg.training.rollout_steps = 1
    cfg.training.batch_size = 1
    tr = SDATrainer(gcm, cfg, total_steps=1)
    tr.configure_backward_precision(("decoder",))
    n = len(tr._backward_hooks)
    assert n > 0
    hist = tr.fit(log_every=1)
    assert np.isfinite(hist[-1]["loss"])
    tr.configure_backward_precision(("decoder",))      # re-configuring replaces, not stacks
    assert len(tr._backward_hooks) == n
    tr.remove_backward_hooks()
    assert not tr._backward_hooks


def test_inference_and_vectorized_wrappers_follow_the_reference_contract():
    from tornado_gcm_b200.models.api import InferenceModel, VectorizedModel

    gcm, data, norm = _small()
    gcm.eval()
    m = gcm.model
    forc = data.forcings(1)
    with torch.no_grad():
        s0 = gcm.encoder(norm(data.sample(1, 0)), forc)
        inf = InferenceModel(m, post_process_fn=lambda s: s.vorticity.norm())
        traj = inf(s0, 2, 1, forcings=forc)
        assert len(traj) == 2 and all(torch.isfinite(t) for t in traj)
        # assimilation without an encoder on the bare model: a model-space state, blended
        half = InferenceModel(m).assimilate(s0 * 2.0, state=s0, alpha=0.5)
        torch.testing.assert_close(half.vorticity, s0.vorticity * 1.5)
        assert VectorizedModel(m, use_vmap=False).mode == "loop" and VectorizedModel(m).mode == "batch"


def test_atmosphere_and_pressure_level_facades():
    import numpy as np

    from tornado_gcm_b200.core import coordinate_systems as cs, sigma_coordinates as sc, spherical_harmonic as sh
    from tornado_gcm_b200.core import primitive_equations_states as pes
    from tornado_gcm_b200.model.atmosphere import AtmosphereConfig, AtmosphericModel
    from tornado_gcm_b200.model.legacy import SHORT_TO_LONG, PressureLevelModel
    from tornado_gcm_b200.utils.units import SimUnits

    # dycore-only facade: two outer steps from an isothermal state at rest stay at rest
    coords = cs.CoordinateSystem(sh.Grid.T21(), sc.SigmaCoordinates.equidistant(4))
    units = SimUnits.from_si()
    cfg = AtmosphereConfig(coords=coords, physics_specs=units, dt=0.01, dycore_substeps=1,
                           reference_temperature=np.full(4, 288.0), orography=torch.zeros(coords.horizontal.modal_shape))
    atm = AtmosphericModel(cfg)
    init_fn, _ = pes.isothermal_rest_atmosphere(coords, units, tref=288.0)
    s0 = init_fn()
    s0.tracers = {"specific_humidity": torch.zeros_like(s0.temperature_variation)}
    final, traj = atm(s0, 2, forcings={})
    assert len(traj) == 2 and torch.isfinite(final.vorticity).all()
    half = atm.assimilate(None, state=s0, alpha=1.0) if atm.encoder is not None else s0
    assert half is s0

    # pressure-level wrapper on the hybrid model, with the reference's keyword names
    gcm, data, _ = _small()
    gcm.eval()
    plm = PressureLevelModel(atmosphere_model=gcm)
    raw = {SHORT_TO_LONG.get(k, k): v for k, v in data.sample(1, 0).items()}
    with torch.no_grad():
        out = plm.predict(raw, forcings=data.forcings(1), outer_steps=1)
    assert len(out) == 1 and set(out[0]) <= set(plm.output_variables) and out[0]
    assert all(torch.isfinite(v).all() for v in out[0].values())


def test_host_offload_rollout_gradients_match_plain_rollout():
    from tornado_gcm_b200.training.trainer import HostOffloadCheckpoint

    w = torch.nn.Parameter(torch.tensor([0.9, 1.1]))
    step = lambda s: torch.tanh(s * w) + 0.1  # noqa: E731
    x0 = torch.tensor([0.3, -0.2])
    final, traj = HostOffloadCheckpoint(max_offloaded=3).rollout(step, x0, 6, segment_length=2)
    assert len(traj) == 6
    (g1,) = torch.autograd.grad(sum(t.sum() for t in traj), [w])
    s, ref = x0, []
    for _ in range(6):
        s = step(s)
        ref.append(s)
    (g2,) = torch.autograd.grad(sum(t.sum() for t in ref), [w])
    torch.testing.assert_close(g1, g2)
    torch.testing.assert_close(final, s)


def test_sda_trainer_reference_keywords():
    from tornado_gcm_b200.precision.sda import SDAConfig
    from tornado_gcm_b200.training.sda_trainer import SDATrainer

    gcm, _, _ = _small()
    cfg = SDAConfig()
    cfg.training.rollout_steps = 1
    cfg.training.batch_size = 1
    opt = torch.optim.AdamW(gcm.parameters(), lr=3e-4, weight_decay=0.01)
    calls = []

    def loss_fn(predictions, targets):
        calls.append(len(predictions))
        return {"total": sum(((p["t"] - t["t"]) ** 2).mean() for p, t in zip(predictions, targets))}

    tr = SDATrainer(gcm, cfg, optimizer=opt, loss_fn=loss_fn, max_grad_norm=0.5, ema_num_steps=99)
    assert tr._trainer.optimizer.param_groups[0]["lr"] == 3e-4 and tr._trainer.max_grad_norm == 0.5
    seen = []
    hist = tr.fit(total_steps=2, callbacks=[lambda i, out: seen.append(i)], log_interval=1)
    assert len(hist) == 2 and seen == [0, 1] and calls and np.isfinite(hist[-1]["loss"])
    gcm.loss_fn = None
