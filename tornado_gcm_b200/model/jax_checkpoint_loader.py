"""NeuralGCM JAX (Haiku) checkpoint → PyTorch — reference ``model/jax_checkpoint_loader.py:52-900``.

A NeuralGCM checkpoint is a pickled nested dict whose ``params`` leaves are
Haiku module paths such as
``params/stochastic_modular_step_model/~/<component>/~/.../epd_tower/process_tower_2/~/mlp_uniform/~/linear_1/w``.
This module

* flattens the pickle to ``"a/b/c" → ndarray`` (:func:`read_jax_checkpoint`);
* builds the networks of the 2.8° deterministic checkpoint
  (:class:`JaxNeuralComponents`: encoder / decoder / physics EPD towers,
  three surface EPDs, the vertical convolution tower, learned positional
  features) — the layer sizes are those of the checkpoint format;
* maps every Haiku leaf to a state-dict entry by a small set of path rules
  (:func:`build_weight_mapping`) and converts layouts: Haiku ``Linear`` ``w``
  is ``(in, out)`` → ``weight = w.T``; Haiku ``Conv1D`` ``w`` is
  ``(kernel, in, out)`` → ``weight = w.permute(2, 1, 0)``, ``b`` squeezed;
* loads the weights (:func:`load_jax_weights`) and reports unmatched leaves.

:func:`load_jax_checkpoint` returns the flat dict (the reference's name);
:func:`load_jax_hybrid` copies matching towers into this framework's hybrid
model (its column tower, encoder and decoder MLPs) by position and shape.
"""

from __future__ import annotations

import logging
import pickle
import re
from pathlib import Path
from typing import Any, Optional

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from tornado_gcm_b200.neural.standard_layers import Epd, Mlp
from tornado_gcm_b200.neural.towers import VerticalConvTower

logger = logging.getLogger(__name__)

# layer sizes of the deterministic 2.8° checkpoint (fixed by the checkpoint format)
LATENT_SIZE = 384
NUM_BLOCKS = 5
N_SIGMA_LAYERS = 32
PHYSICS_EPD_INPUT, PHYSICS_EPD_OUTPUT = 2365, 192
DECODER_EPD_INPUT, DECODER_EPD_OUTPUT = 784, 259
ENCODER_EPD_INPUT, ENCODER_EPD_OUTPUT = 1052, 193
SURFACE_EMBED_INPUTS = (4, 1, 5)  # land, sea, sea ice
SURFACE_LATENT = 8
VOLUME_CONV_IN, VOLUME_CONV_HIDDEN, VOLUME_CONV_OUT, VOLUME_CONV_KERNEL = 9, (64, 64, 64, 64), 32, 5
POSITIONAL_SHAPE = (8, 128, 64)

_ROOT = "params/stochastic_modular_step_model/~/"
_COMPONENTS = {
    "dimensional_learned_primitive_to_weatherbench_decoder/": "decoder",
    "dimensional_learned_weatherbench_to_primitive_with_memory_encoder/~/": "encoder",
    "stochastic_physics_parameterization_step/~/": "physics",
}


def _gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    return F.gelu(x, approximate="tanh")


def build_epd_tower(input_size: int, output_size: int, latent_size: int = LATENT_SIZE, num_blocks: int = NUM_BLOCKS,
                    process_hidden: int = 3, decode_hidden: int = 0, *, process_n_hidden: Optional[int] = None,
                    decode_n_hidden: Optional[int] = None, encode_bias: bool = True,
                    decode_bias: bool = False) -> Epd:
    """The checkpoint's EPD: encode = one linear (biased by default), ``num_blocks`` residual
    process MLPs of ``process_hidden + 1`` biased linears, decode = MLP (bias-free by
    default) with ``decode_hidden`` hidden layers; GELU (tanh form) between layers.
    ``process_n_hidden`` / ``decode_n_hidden`` are the reference's names of the two counts."""
    process_hidden = process_hidden if process_n_hidden is None else process_n_hidden
    decode_hidden = decode_hidden if decode_n_hidden is None else decode_n_hidden
    mlp = lambda i, o, hidden, bias: Mlp(i, o, intermediate_sizes=(latent_size,) * hidden, activation=_gelu_tanh,
                                         activate_final=False, use_bias=bias)
    return Epd(mlp(input_size, latent_size, 0, encode_bias), mlp(latent_size, output_size, decode_hidden, decode_bias),
               [mlp(latent_size, latent_size, process_hidden, True) for _ in range(num_blocks)])


def build_surface_epd(input_size: int, output_size: int = SURFACE_LATENT) -> Epd:
    return build_epd_tower(input_size, output_size, latent_size=SURFACE_LATENT, num_blocks=1, decode_hidden=1)


def build_volume_conv_tower() -> VerticalConvTower:
    return VerticalConvTower(VOLUME_CONV_IN, VOLUME_CONV_OUT, channels=VOLUME_CONV_HIDDEN,
                             kernel_size=VOLUME_CONV_KERNEL)


class JaxNeuralComponents(nn.Module):
    """The learnable networks of the NeuralGCM 2.8° deterministic checkpoint."""

    def __init__(self):
        super().__init__()
        self.encoder_epd = nn.ModuleList([build_epd_tower(ENCODER_EPD_INPUT, ENCODER_EPD_OUTPUT) for _ in range(2)])
        self.decoder_epd = build_epd_tower(DECODER_EPD_INPUT, DECODER_EPD_OUTPUT)
        self.physics_epd = build_epd_tower(PHYSICS_EPD_INPUT, PHYSICS_EPD_OUTPUT)
        self.surface_epd = nn.ModuleList([build_surface_epd(n) for n in SURFACE_EMBED_INPUTS])
        self.volume_conv = build_volume_conv_tower()
        self.encoder_positional = nn.ParameterList([nn.Parameter(torch.zeros(POSITIONAL_SHAPE)) for _ in range(2)])
        self.decoder_positional = nn.Parameter(torch.zeros(POSITIONAL_SHAPE))
        self.physics_positional = nn.Parameter(torch.zeros(POSITIONAL_SHAPE))

    def count_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters())


# ── reading and mapping ──────────────────────────────────────────────────────
def read_jax_checkpoint(path: str | Path) -> dict[str, Any]:
    """Unpickle a checkpoint and flatten it to ``"a/b/c" → leaf``."""
    path = Path(path)
    if not path.exists():
        raise FileNotFoundError(f"checkpoint not found: {path}")
    with open(path, "rb") as fh:
        data = pickle.load(fh)
    flat: dict[str, Any] = {}

    def walk(obj, prefix: str) -> None:
        if isinstance(obj, dict):
            for k, v in obj.items():
                walk(v, f"{prefix}{k}/")
        elif isinstance(obj, (list, tuple)):
            for i, v in enumerate(obj):
                walk(v, f"{prefix}[{i}]/")
        elif isinstance(obj, (np.ndarray, np.generic, int, float, str)) or hasattr(obj, "__array__"):
            flat[prefix.rstrip("/")] = np.asarray(obj) if hasattr(obj, "__array__") else obj

    walk(data, "")
    return flat


load_jax_checkpoint_flat = read_jax_checkpoint

_MLP_RE = re.compile(r"(surface_model_)?(encode|process|decode)_tower(?:_(\d+))?/~/mlp_uniform/~/linear_(\d+)/(w|b)$")
_CONV_RE = re.compile(r"conv_level(?:_(\d+))?/(w|b)$")


def _component(path: str) -> Optional[tuple[str, str]]:
    if not path.startswith(_ROOT):
        return None
    rest = path[len(_ROOT):]
    for prefix, name in _COMPONENTS.items():
        if rest.startswith(prefix):
            return name, rest[len(prefix):]
    return None


def build_weight_mapping(jax_params: dict) -> dict[str, tuple[str, str]]:
    """``{haiku path: (state-dict key, kind)}`` for :class:`JaxNeuralComponents`.

    kinds: ``linear_w``, ``linear_b``, ``conv_w``, ``conv_b``, ``positional``.
    Several towers of the same kind inside one component (the two encoder
    towers, the three surface towers) are numbered by the sorted order of
    their owner prefixes.
    """
    mapping: dict[str, tuple[str, str]] = {}
    owners: dict[tuple[str, str], list[str]] = {}
    parsed = []
    for path in jax_params:
        c = _component(path)
        if c is None:
            continue
        comp, sub = c
        m = _MLP_RE.search(sub)
        if m:
            owner = sub[:m.start()]
            surf = bool(m.group(1))
            owners.setdefault((comp, "surface" if surf else "epd"), [])
            if owner not in owners[(comp, "surface" if surf else "epd")]:
                owners[(comp, "surface" if surf else "epd")].append(owner)
            parsed.append((path, comp, owner, surf, m))
            continue
        m = _CONV_RE.search(sub)
        if m:
            idx = int(m.group(1)) if m.group(1) else 0
            kind = "conv_w" if m.group(2) == "w" else "conv_b"
            mapping[path] = (f"volume_conv.layers.{idx}.conv.{'weight' if kind == 'conv_w' else 'bias'}", kind)
            continue
        if "learned_positional" in sub or "positional_features" in sub:
            owners.setdefault((comp, "pos"), []).append(sub)
            parsed.append((path, comp, sub, None, None))
    for k in owners:
        owners[k] = sorted(set(owners[k]))
    # surface towers: order by their input width (land 4, sea 1, ice 5), not by name
    for key in [k for k in owners if k[1] == "surface"]:
        def width(owner, comp=key[0]):
            for path, c, o, surf, m in parsed:
                if m is not None and c == comp and o == owner and m.group(2) == "encode" and m.group(4) == "0" \
                        and m.group(5) == "w":
                    return int(np.asarray(jax_params[path]).shape[0])
            return -1
        ordered = sorted(owners[key], key=lambda o: SURFACE_EMBED_INPUTS.index(width(o))
                         if width(o) in SURFACE_EMBED_INPUTS else 99)
        owners[key] = ordered
    for path, comp, owner, surf, m in parsed:
        if m is None:  # positional features
            i = owners[(comp, "pos")].index(owner)
            key = {"encoder": f"encoder_positional.{i}", "decoder": "decoder_positional",
                   "physics": "physics_positional"}[comp]
            mapping[path] = (key, "positional")
            continue
        part, block, lin, wb = m.group(2), m.group(3), int(m.group(4)), m.group(5)
        i = owners[(comp, "surface" if surf else "epd")].index(owner)
        if surf:
            base = f"surface_epd.{i}"
        elif comp == "encoder":
            base = f"encoder_epd.{i}"
        else:
            base = f"{comp}_epd"
        if part == "process":
            sub_mod = f"process_blocks.{int(block) if block else 0}"
        else:
            sub_mod = part
        mapping[path] = (f"{base}.{sub_mod}.layers.{lin}.{'weight' if wb == 'w' else 'bias'}", f"linear_{wb}")
    return mapping


def _convert(value: np.ndarray, kind: str, target: torch.Tensor) -> torch.Tensor:
    t = torch.as_tensor(np.asarray(value, dtype=np.float32))
    if kind == "linear_w":
        t = t.t()
    elif kind == "conv_w":
        t = t.permute(2, 1, 0)
    elif kind in ("conv_b", "linear_b"):
        t = t.reshape(-1)
    if t.shape != target.shape:
        t = t.reshape(target.shape)
    return t.to(target.dtype)


def load_jax_weights(model: nn.Module, checkpoint_path, strict: bool = True) -> dict:
    """Copy mapped leaves into ``model``; returns a report of what was (not) loaded.

    ``checkpoint_path``: a pickled Haiku checkpoint (read with :func:`read_jax_checkpoint`,
    its ``params/`` leaves used) or an already flattened ``{path: array}`` dict."""
    if isinstance(checkpoint_path, (str, Path)):
        flat = read_jax_checkpoint(checkpoint_path)
        jax_params = {k: v for k, v in flat.items() if k.startswith("params/")}
    else:
        jax_params = checkpoint_path
    module = model
    mapping = build_weight_mapping(jax_params)
    sd = module.state_dict()
    loaded, skipped = [], []
    with torch.no_grad():
        for path, (key, kind) in mapping.items():
            if key not in sd:
                skipped.append(path)
                continue
            try:
                sd[key].copy_(_convert(jax_params[path], kind, sd[key]))
                loaded.append(key)
            except RuntimeError:
                skipped.append(path)
    missing = [k for k in sd if k not in set(loaded)]
    unmatched = [p for p in jax_params if p.startswith("params/") and p not in mapping]
    if strict and (missing or skipped):
        raise RuntimeError(f"JAX load incomplete: {len(missing)} missing, {len(skipped)} skipped")
    return {"loaded": loaded, "missing": missing, "skipped": skipped, "unmatched": unmatched}


def load_jax_checkpoint(checkpoint_path: str | Path, device: str | torch.device | None = None,
                        resolution: Optional[str] = None):
    """Without ``device``: the flat parameter dict (the reference's behaviour).

    With ``device``: a hybrid model of ``resolution`` whose column tower,
    encoder and decoder MLPs are initialised from the checkpoint's physics,
    encoder and decoder towers wherever the layer shapes agree.
    """
    flat = read_jax_checkpoint(checkpoint_path)
    if device is None:
        return flat
    return load_jax_hybrid(flat, device=device, resolution=resolution or "2.8deg")


def build_jax_neural_components() -> JaxNeuralComponents:
    return JaxNeuralComponents()


def load_jax_hybrid(flat: dict, device: str | torch.device = "cpu", resolution: str = "2.8deg"):
    """Hybrid model of this framework initialised from a checkpoint's towers by shape."""
    from tornado_gcm_b200.models.builders import build_hybrid_gcm

    comps = JaxNeuralComponents()
    report = load_jax_weights(comps, flat, strict=False)
    gcm, _ = build_hybrid_gcm(resolution, device)
    pairs = [(comps.physics_epd, gcm.model.parameterization.tower), (comps.encoder_epd[0], gcm.encoder.net),
             (comps.decoder_epd, gcm.decoder.net)]
    copied = 0
    with torch.no_grad():
        for src, dst in pairs:
            s_lin = [m for m in src.modules() if isinstance(m, nn.Linear)]
            d_lin = [m for m in dst.modules() if isinstance(m, nn.Linear)]
            for a, b in zip(s_lin, d_lin):
                if a.weight.shape == b.weight.shape:
                    b.weight.copy_(a.weight)
                    if a.bias is not None and b.bias is not None:
                        b.bias.copy_(a.bias)
                    copied += 1
    logger.info("JAX checkpoint: %d tensors loaded into the reference towers, %d linear layers copied into the "
                "%s hybrid model", len(report["loaded"]), copied, resolution)
    gcm.jax_load_report = {**report, "linear_layers_copied": copied}
    return gcm


# ── the runnable 2.8° NeuralGCM model ────────────────────────────────────────
# The checkpoint's physics step: TL63 (128 x 64 Gaussian grid), 32 equidistant
# sigma layers, dt = 0.525024 (one hour in the checkpoint's time unit), five
# dycore substeps, dycore filter tau 120 min order 3, stability filter
# tau 4 min order 10 cutoff 0.4 (also applied to the parameterization's
# tendencies), FP64 conservation fixer.  Features: surface embeddings (land /
# sea / sea-ice towers), the vertical conv tower's 32 CNN1D features,
# pressure, radiation, latitude, prognostics with their gradients and
# Laplacians, memory values, geopotential at the surface (with gradients),
# land-sea mask and the learned positional features -> ShiftAndNormalize ->
# InverseLevelScale (humidity) -> SoftClip(16), 2365 channels in sorted-key
# order into the physics EPD; its 192 outputs -> InverseShiftAndNormalize
# (global scale 0.02) -> humidity level scales -> (zeta, delta, T', tracers)
# tendencies.  Normalisation statistics: data/neuralgcm_2p8deg_normalization.json.
JAX_DT_NONDIM = 0.525024
JAX_DYCORE_SUBSTEPS = 5
_STATS_FILE = Path(__file__).resolve().parent.parent / "data" / "neuralgcm_2p8deg_normalization.json"


def jax_normalization_stats() -> dict:
    import json

    with open(_STATS_FILE, encoding="utf-8") as fh:
        st = json.load(fh)
    cnn = {f"CNN1D_{i}": st["cnn_feature_scale"] for i in range(st["n_cnn_features"])}
    cnn_shift = {f"CNN1D_{i}": st["cnn_feature_shift"] for i in range(st["n_cnn_features"])}
    st["advance_scales"] = {**cnn, **st["feature_scales"]}
    st["advance_shifts"] = {**cnn_shift, **st["feature_shifts"]}
    return st


def build_jax_aligned_model(checkpoint: str | Path | dict | None = None, device: str | torch.device = "cpu",
                            strict: bool = True, geopotential_at_surface: Optional[torch.Tensor] = None,
                            land_sea_mask: Optional[torch.Tensor] = None):
    """NeuralGCM 2.8° deterministic model wired to :class:`JaxNeuralComponents` — reference
    ``model/jax_checkpoint_loader.py:885-1241`` (``build_jax_aligned_experiment_model``).

    ``checkpoint``: a pickle path or an already flattened parameter dict; the
    weights are loaded with the strict path map (every leaf mapped, every
    parameter filled).  ``geopotential_at_surface`` / ``land_sea_mask``
    ``(1, lon, lat)`` come from the checkpoint's auxiliary data (zeros when
    absent).  Returns ``(model, components, coords, config, report)``.
    """
    from tornado_gcm_b200.core import coordinate_systems, filtering, sigma_coordinates, spherical_harmonic
    from tornado_gcm_b200.models.api import ModelConfig, NeuralGCMModel
    from tornado_gcm_b200.neural import features as ft
    from tornado_gcm_b200.neural import transforms as tr
    from tornado_gcm_b200.neural.fixers import F64ConservationFixer
    from tornado_gcm_b200.neural.parameterizations import JaxAlignedDivCurlParameterization
    from tornado_gcm_b200.neural.towers import ForwardTower
    from tornado_gcm_b200.precision.policy import PrecisionPolicy
    from tornado_gcm_b200.utils.units import SimUnits, minutes_to_nondim

    stats = jax_normalization_stats()
    grid = spherical_harmonic.Grid.TL63()
    vertical = sigma_coordinates.SigmaCoordinates.equidistant(N_SIGMA_LAYERS)
    coords = coordinate_systems.CoordinateSystem(grid, vertical)
    I, J = grid.nodal_shape
    geo = geopotential_at_surface if geopotential_at_surface is not None else torch.zeros(1, I, J)
    lsm = land_sea_mask if land_sea_mask is not None else torch.zeros(1, I, J)

    comps = JaxNeuralComponents()
    report = None
    if checkpoint is not None:
        flat = checkpoint if isinstance(checkpoint, dict) else read_jax_checkpoint(checkpoint)
        report = load_jax_weights(comps, {k: v for k, v in flat.items() if k.startswith("params/")}, strict=strict)

    scales, shifts = stats["advance_scales"], stats["advance_shifts"]
    fields = ["divergence", "vorticity", "u", "v", "temperature_variation", "log_surface_pressure",
              "specific_humidity", "specific_cloud_liquid_water_content", "specific_cloud_ice_water_content"]
    norm = (scales, shifts)
    surface = ft.EmbeddingSurfaceFeatures(
        grid, ForwardTower(comps.surface_epd[0], feature_axis=-3), ForwardTower(comps.surface_epd[1], feature_axis=-3),
        ForwardTower(comps.surface_epd[2], feature_axis=-3), lsm.clone(), norm, norm, norm)
    volume = ft.EmbeddingVolumeFeatures(grid, comps.volume_conv, vertical.centers, n_output=VOLUME_CONV_OUT,
                                        feature_name="CNN1D", embedding_scales=scales, embedding_shifts=shifts)
    extractor = ft.CombinedFeatures([
        surface, volume, ft.PressureFeatures(grid, vertical.centers), ft.RadiationFeatures(grid),
        ft.LatitudeFeatures(grid),
        ft.VelocityAndPrognostics(grid, fields_to_include=fields, compute_gradients_fn=tr.ToModalDiffOperators(grid)),
        ft.MemoryVelocityAndValues(grid, fields_to_include=fields, compute_gradients_fn=None),
        ft.FloatDataFeatures(grid, {"geopotential_at_surface": geo}, compute_gradients_fn=tr.ToModalDiffOperators(grid)),
        ft.FloatDataFeatures(grid, {"land_sea_mask": lsm}, compute_gradients_fn=None),
        ft.LearnedPositionalFeatures(comps.physics_positional),
    ])
    feature_transform = tr.SequentialTransform([
        tr.ShiftAndNormalize(shifts=shifts, scales=scales),
        tr.InverseLevelScale(["specific_humidity", "specific_humidity_del2", "specific_humidity_dlat",
                              "specific_humidity_dlon"], stats["humidity_inverse_level_scales"]),
        tr.SoftClip(max_value=16.0, hinge_softness=1.0),
    ])
    tendency_transform = tr.SequentialTransform([
        tr.InverseShiftAndNormalize(shifts=stats["tendency_shifts"], scales=stats["tendency_scales"],
                                    global_scale=stats["tendency_global_scale"]),
        tr.TendencyTransform(level_scales={"specific_humidity": torch.tensor(
            stats["tendency_humidity_level_scales"], dtype=torch.float32)}),
    ])
    dycore_att = JAX_DT_NONDIM / minutes_to_nondim(120.0)
    stab_att = JAX_DT_NONDIM / minutes_to_nondim(4.0)
    param = JaxAlignedDivCurlParameterization(grid, ForwardTower(comps.physics_epd, feature_axis=-3), extractor,
                                              feature_transform, tendency_transform, n_levels=N_SIGMA_LAYERS)
    param.filter_fn = filtering.exponential_filter(grid, attenuation=stab_att, order=10, cutoff=0.4)
    # orography from the surface geopotential (m^2/s^2 over the squared velocity scale)
    vel2 = (6371220.0 * 2 * 7.292e-5) ** 2
    orography = grid.to_modal(geo[0].double() / vel2).float()
    cfg = ModelConfig(coords=coords, dt=JAX_DT_NONDIM, dycore_substeps=JAX_DYCORE_SUBSTEPS,
                      physics_specs=SimUnits.from_si(), reference_temperature=np.asarray(
                          stats["reference_temperatures"]), orography=orography,
                      cloud_keys=("specific_cloud_liquid_water_content", "specific_cloud_ice_water_content"),
                      precision_policy=PrecisionPolicy(), filter_attenuation=dycore_att, filter_order=3,
                      filter_cutoff=0.0, stability_filter_attenuation=stab_att, stability_filter_order=10,
                      stability_filter_cutoff=0.4)
    model = NeuralGCMModel(cfg, param, F64ConservationFixer(energy_split="reference")).to(device)
    comps = comps.to(device)
    config = {"resolution": "2.8", "n_levels": N_SIGMA_LAYERS, "dt_hours": 1.0, "grid": "TL63",
              "latent_size": LATENT_SIZE, "num_blocks": NUM_BLOCKS, "physics_features": PHYSICS_EPD_INPUT}
    return model, comps, coords, config, report


def build_jax_aligned_experiment_model(checkpoint_path: str | Path | None = None, device: str | torch.device = "cpu"):
    """Reference-named entry point (``model/jax_checkpoint_loader.py:885``): the runnable
    2.8° NeuralGCM of :func:`build_jax_aligned_model`, weights loaded with the strict map.
    Returns ``(model, components, coords, config, report)``."""
    return build_jax_aligned_model(checkpoint_path, device=device, strict=True)


def build_and_load_jax_model(checkpoint_path: str | Path, device: str | torch.device = "cpu"):
    """The neural components alone with the checkpoint's weights (reference
    ``model/jax_checkpoint_loader.py:861``): ``(components in eval mode, load report)``.
    Leaves without a target are reported rather than refused, as in the reference."""
    comps = build_jax_neural_components()
    flat = read_jax_checkpoint(checkpoint_path)
    report = load_jax_weights(comps, {k: v for k, v in flat.items() if k.startswith("params/")}, strict=False)
    return comps.to(device).eval(), report
