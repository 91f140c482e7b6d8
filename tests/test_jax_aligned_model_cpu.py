"""NeuralGCM 2.8° model assembled from a Haiku-layout checkpoint (strict path map).

A synthetic checkpoint with the exact Haiku parameter paths and layouts of
the deterministic 2.8° checkpoint ((in, out) linear kernels, (kernel, in, out)
conv kernels, (out, 1) conv biases) is loaded strictly by this framework's
loader and by the reference's own loader; the towers of both then give the
same outputs, and the assembled model runs a forward step.
"""

import pickle

import numpy as np
import pytest
import torch

from tornado_gcm_b200.model import jax_checkpoint_loader as jcl

ROOT = "params/stochastic_modular_step_model/~/"
PHYS = ROOT + "stochastic_physics_parameterization_step/~/"
ENC = ROOT + "dimensional_learned_weatherbench_to_primitive_with_memory_encoder/~/"
DEC = ROOT + "dimensional_learned_primitive_to_weatherbench_decoder/"


def _epd_leaves(prefix, n_in, n_out, latent=384, blocks=5, surface=False, decode_hidden=0):
    """Haiku leaves of one EPD tower: encode (biased), residual process blocks of 4 biased
    linears, bias-free decode."""
    s = "surface_model_" if surface else ""
    out = {}
    out[f"{prefix}{s}encode_tower/~/mlp_uniform/~/linear_0/w"] = (n_in, latent)
    out[f"{prefix}{s}encode_tower/~/mlp_uniform/~/linear_0/b"] = (latent,)
    for blk in range(blocks):
        suffix = "" if blk == 0 else f"_{blk}"
        for i in range(4):
            out[f"{prefix}{s}process_tower{suffix}/~/mlp_uniform/~/linear_{i}/w"] = (latent, latent)
            out[f"{prefix}{s}process_tower{suffix}/~/mlp_uniform/~/linear_{i}/b"] = (latent,)
    dims = [latent] * (decode_hidden + 1) + [n_out]
    for i in range(decode_hidden + 1):
        out[f"{prefix}{s}decode_tower/~/mlp_uniform/~/linear_{i}/w"] = (dims[i], dims[i + 1])
    return out


def _synthetic_checkpoint(rng):
    shapes = {}
    shapes.update(_epd_leaves(PHYS + "div_curl_neural_parameterization/nodal_mapping/~/epd_tower/", 2365, 192))
    for k, n_in in enumerate((4, 1, 5)):
        suffix = "" if k == 0 else f"_{k}"
        shapes.update(_epd_leaves(
            PHYS + f"custom_coords_corrector/~/embedding_surface_features/~/modal_to_nodal_embedding{suffix}"
                   f"/nodal_mapping/~/epd_tower/", n_in, 8, latent=8, blocks=1, surface=True, decode_hidden=1))
    chans = [9, 64, 64, 64, 64, 32]
    for i in range(5):
        suffix = "" if i == 0 else f"_{i}"
        base = PHYS + f"custom_coords_corrector/~/embedding_volume_features/~/vertical_conv_tower/~/conv_level{suffix}/"
        shapes[base + "w"] = (5, chans[i], chans[i + 1])
        shapes[base + "b"] = (chans[i + 1], 1)
    shapes[PHYS + "div_curl_neural_parameterization/learned_positional_features/learned_positional_features"] = (8, 128, 64)
    shapes[PHYS + "custom_coords_corrector/~/learned_orography/orography"] = (4094,)
    for e, sfx in enumerate(("", "_1")):
        enc = ENC + f"learned_weatherbench_to_primitive_encoder{sfx}/"
        shapes.update(_epd_leaves(enc + "nodal_mapping/~/epd_tower/", 1052, 193))
        shapes[enc + "learned_positional_features/learned_positional_features"] = (8, 128, 64)
        shapes[enc + "learned_orography/orography"] = (4223,)
    shapes.update(_epd_leaves(DEC + "nodal_mapping/~/epd_tower/", 784, 259))
    shapes[DEC + "learned_positional_features/learned_positional_features"] = (8, 128, 64)
    flat = {k: (rng.standard_normal(s) * 0.05).astype(np.float32) for k, s in shapes.items()}
    nested: dict = {}
    for path, v in flat.items():
        node = nested
        parts = path.split("/")
        for p in parts[:-1]:
            node = node.setdefault(p, {})
        node[parts[-1]] = v
    return flat, nested


@pytest.fixture(scope="module")
def checkpoint(tmp_path_factory):
    rng = np.random.default_rng(0)
    flat, nested = _synthetic_checkpoint(rng)
    path = tmp_path_factory.mktemp("jax") / "ckpt.pkl"
    with open(path, "wb") as fh:
        pickle.dump(nested, fh)
    return path, flat


def test_strict_load_fills_every_parameter(checkpoint):
    path, flat = checkpoint
    comps = jcl.JaxNeuralComponents()
    report = jcl.load_jax_weights(comps, jcl.read_jax_checkpoint(path), strict=True)
    assert not report["missing"] and not report["skipped"]
    # the only leaves without a counterpart are the two learned orographies the model does not use
    assert all("orography" in p for p in report["unmatched"])
    w = flat[PHYS + "div_curl_neural_parameterization/nodal_mapping/~/epd_tower/encode_tower/~/mlp_uniform/~/linear_0/w"]
    torch.testing.assert_close(comps.physics_epd.encode.layers[0].weight, torch.as_tensor(w).t())


def test_strict_load_rejects_a_missing_leaf(checkpoint):
    path, flat = checkpoint
    broken = dict(jcl.read_jax_checkpoint(path))
    broken.pop(next(k for k in broken if "process_tower_3/~/mlp_uniform/~/linear_2/b" in k))
    with pytest.raises(RuntimeError):
        jcl.load_jax_weights(jcl.JaxNeuralComponents(), broken, strict=True)


@pytest.mark.oracle
def test_towers_match_reference_loader(checkpoint, ref, monkeypatch):
    import sys
    import types

    path, _ = checkpoint
    # the reference loader imports its pint-based unit module at load time but uses it only in its
    # model builder; pint is not installed, so an empty stand-in is put in place for this import
    monkeypatch.setitem(sys.modules, "tornado_gcm.scales", types.ModuleType("tornado_gcm.scales"))
    monkeypatch.delitem(sys.modules, "tornado_gcm.model.jax_checkpoint_loader", raising=False)
    rj = ref.import_module("tornado_gcm.model.jax_checkpoint_loader")
    theirs = rj.build_jax_neural_components()
    rj.load_jax_weights(theirs, path, strict=True)
    ours = jcl.JaxNeuralComponents()
    jcl.load_jax_weights(ours, jcl.read_jax_checkpoint(path), strict=True)
    torch.manual_seed(0)
    x = torch.randn(7, 2365)
    with torch.no_grad():
        torch.testing.assert_close(ours.physics_epd(x), theirs.physics_epd(x), rtol=1e-5, atol=1e-5)
        for k, n_in in enumerate((4, 1, 5)):
            xs = torch.randn(5, n_in)
            torch.testing.assert_close(ours.surface_epd[k](xs), theirs.physics_surface_embeds[k](xs),
                                       rtol=1e-5, atol=1e-5)
        xc = torch.randn(9, 32, 4, 2)  # (channels, levels, lon, lat)
        torch.testing.assert_close(ours.volume_conv(xc), theirs.physics_volume_embed(xc), rtol=1e-5, atol=1e-5)
        xe = torch.randn(4, 1052)
        torch.testing.assert_close(ours.encoder_epd[1](xe), theirs.encoder_1_epd(xe), rtol=1e-5, atol=1e-5)
        xd = torch.randn(4, 784)
        torch.testing.assert_close(ours.decoder_epd(xd), theirs.decoder_epd(xd), rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(ours.physics_positional, theirs.physics_positional)


def test_aligned_model_steps_from_checkpoint(checkpoint):
    from tornado_gcm_b200.core.primitive_equations import State

    path, _ = checkpoint
    model, comps, coords, config, report = jcl.build_jax_aligned_model(path)
    assert config["physics_features"] == 2365 and not report["missing"]
    g = coords.horizontal
    n = 32
    mask = torch.as_tensor(g.mask)
    torch.manual_seed(1)
    mk = lambda lv: torch.randn(lv, *g.modal_shape) * 1e-3 * mask
    tr = {k: mk(n) * 1e-3 for k in ("specific_humidity", "specific_cloud_liquid_water_content",
                                    "specific_cloud_ice_water_content")}
    st = State(mk(n), mk(n), mk(n), mk(1), tr, sim_time=0.0)
    I, J = g.nodal_shape
    forc = {"sea_surface_temperature": torch.full((1, I, J), 285.0), "sea_ice_cover": torch.zeros(1, I, J)}
    with torch.no_grad():
        tend = model.parameterization(st, forcings=forc, memory=st)
        nxt = model.step(st, forcings=forc)
    for t in (tend.vorticity, tend.temperature_variation, nxt.vorticity, nxt.log_surface_pressure):
        assert torch.isfinite(t).all()
    assert float(tend.vorticity.abs().max()) > 0.0


def test_reference_named_builders(checkpoint):
    path, _ = checkpoint
    comps, report = jcl.build_and_load_jax_model(path)
    assert not comps.training and not report["missing"]
    model, comps2, coords, config, report2 = jcl.build_jax_aligned_experiment_model(path)
    assert config["physics_features"] == 2365 and not report2["missing"]
    for a, b in zip(comps.parameters(), comps2.parameters()):
        torch.testing.assert_close(a, b)
