"""Builders for the hybrid GCM at the benchmark resolutions.

=========  ======  ===========  ==============  ================  =========
name       grid    lon × lat    σ levels        dt (physics)      tower
=========  ======  ===========  ==============  ================  =========
2.8deg     TL63    128 × 64     32 equidistant  20 min            5 × 384
1.4deg     TL127   256 × 128    32              10 min            5 × 512
0.7deg     TL255   512 × 256    32              5 min             5 × 768
=========  ======  ===========  ==============  ================  =========

A 6-h model step is ``6 h / dt`` physics steps; the neural tendency is
called every physics step and each physics step is one IMEX-SIL3 dycore
substep followed by the dycore (τ = 120 min, order 3), stability
(τ = 4 min, order 10, cutoff 0.4) and hyperdiffusion (∇⁴, τ = 12 h at the
largest wavenumber; 3 h at 0.7°) spectral filters.  Data enter through a column
encoder (3 × 256) from 7 fields on 37 pressure levels and leave through
a column decoder back to the same fields; the Z2 fixer restores mass and
the energy proxy with FP64 accumulation every physics step.
"""

from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np
import torch
import torch.nn as nn
import torch.utils.checkpoint as torch_checkpoint

from tornado_gcm_b200.core import coordinate_systems, sigma_coordinates, spherical_harmonic
from tornado_gcm_b200.models.api import ModelConfig, NeuralGCMModel
from tornado_gcm_b200.neural.column_codecs import TRACERS, VELOCITY_SCALE, ColumnDecoder, ColumnEncoder
from tornado_gcm_b200.neural.fixers import F64ConservationFixer, LiteConservationFixer
from tornado_gcm_b200.neural.parameterizations import NodalColumnParameterization
from tornado_gcm_b200.neural.standard_layers import Mlp, gelu_tanh
from tornado_gcm_b200.neural.towers import ForwardTower
from tornado_gcm_b200.precision.policy import PrecisionPolicy
from tornado_gcm_b200.training.synthetic import DATA_FIELDS, FORCING_FIELDS, SyntheticReanalysis
from tornado_gcm_b200.utils.units import SimUnits, minutes_to_nondim


@dataclasses.dataclass(frozen=True)
class ResolutionSpec:
    name: str
    grid: str
    dt_minutes: float
    tower_width: int
    tower_hidden_layers: int = 5
    layers: int = 32
    outer_hours: float = 6.0
    encoder_width: int = 256
    encoder_hidden_layers: int = 3
    # ∇⁴ hyperdiffusion e-folding time at the truncation wavenumber
    hyperdiffusion_hours: float = 12.0
    # IMEX-SIL3 dycore substeps per physics step (the tower runs once per physics step)
    dycore_substeps: int = 1
    # orography smoothing: modal coefficients times exp(-(l / (f·L))^8) (None: unfiltered)
    orography_filter: Optional[float] = None

    @property
    def physics_steps_per_output(self) -> int:
        return int(round(self.outer_hours * 60.0 / self.dt_minutes))


RESOLUTIONS = {
    "2.8deg": ResolutionSpec("2.8deg", "TL63", 20.0, 384),
    "1.4deg": ResolutionSpec("1.4deg", "TL127", 10.0, 512),
    # TL255: a 3-h hyperdiffusion time scale at the truncation wavenumber
    "0.7deg": ResolutionSpec("0.7deg", "TL255", 5.0, 768, hyperdiffusion_hours=3.0),
    # small configuration for tests and CPU demonstrations: T21 (64 x 32 grid), 8 levels, dt 2 h
    "5.6deg": ResolutionSpec("5.6deg", "T21", 120.0, 32, tower_hidden_layers=2, layers=8, encoder_width=32,
                             encoder_hidden_layers=1),
}


def reference_temperature_profile(sigma_centers: np.ndarray) -> np.ndarray:
    return np.maximum(200.0, 288.0 * sigma_centers ** 0.19)


class HybridGCM(nn.Module):
    """Encoder → NeuralGCMModel rollout → decoder, with a training loss."""

    def __init__(self, model: NeuralGCMModel, encoder: ColumnEncoder, decoder: ColumnDecoder,
                 physics_steps_per_output: int, forcing_keys=FORCING_FIELDS, forcing_scale=None):
        super().__init__()
        self.model = model
        self.encoder = encoder
        self.decoder = decoder
        self.physics_steps_per_output = physics_steps_per_output
        self.forcing_keys = tuple(forcing_keys)
        self._forcing_scale = forcing_scale or {}
        # recompute each 6-h block of physics steps in backward instead of keeping its
        # activations (the reference's checkpoint_outer_steps, model/api.py:788)
        self.checkpoint_outer_steps = False
        # physics steps per recomputed segment (0: the whole 6-h block); at 0.7° one
        # physics step keeps ~2 GB of tower activations, so a 72-step block does not fit
        self.checkpoint_segment = 0
        # a model sharded over W ranks (parallel.spectral_shard.shard_hybrid_gcm) sees 1/W of
        # every field: its local mean squared error counts 1/W towards the global loss
        self.loss_scale = 1.0
        # optional trajectory loss ``fn(predictions=[...], targets=[...]) -> tensor or {"total": tensor}``
        # in place of the per-field MSE (the reference trainer's ``loss_fn`` protocol)
        self.loss_fn = None
        self.shard = None

    def normalize_forcings(self, forcings: dict) -> dict:
        out = {}
        for k, v in forcings.items():
            off, sc = self._forcing_scale.get(k, (0.0, 1.0))
            out[k] = (v - off) * sc
        return out

    def _segment(self, state, f, start: int, n: int):
        # The step counter drives the fixer cadence: a recompute in backward runs
        # with the counter the forward pass saw and leaves the current one alone.
        # (A recompute may also stop early, once the tensors it needs exist.)
        m = self.model
        before = m._step_count
        m._step_count = start
        try:
            for _ in range(n):
                state = m.step(state, f)
        finally:
            m._step_count = max(before, start + n)
        return state

    def rollout(self, data0: dict, forcings: dict, outer_steps: int, decode: bool = True,
                checkpoint_outer_steps: Optional[bool] = None):
        ckpt = self.checkpoint_outer_steps if checkpoint_outer_steps is None else checkpoint_outer_steps
        f = self.normalize_forcings(forcings)
        state = self.encoder(data0, f)
        outs = []
        for _ in range(outer_steps):
            if ckpt and torch.is_grad_enabled():
                # no RNG state capture: the step draws no random numbers, and reading the
                # generator state is not allowed inside CUDA-graph capture
                n_phys = self.physics_steps_per_output
                seg = self.checkpoint_segment if self.checkpoint_segment > 0 else n_phys
                done = 0
                while done < n_phys:
                    k = min(seg, n_phys - done)
                    state = torch_checkpoint.checkpoint(self._segment, state, f, self.model._step_count, k,
                                                        use_reentrant=False, preserve_rng_state=False)
                    done += k
            else:
                for _ in range(self.physics_steps_per_output):
                    state = self.model.step(state, f)
            outs.append(self.decoder(state, f) if decode else state)
        return state, outs

    def loss(self, data0: dict, targets: list, forcings: dict) -> torch.Tensor:
        _, preds = self.rollout(data0, forcings, len(targets))
        if self.loss_fn is not None:
            out = self.loss_fn(predictions=preds, targets=list(targets))
            return (out["total"] if isinstance(out, dict) else out) * self.loss_scale
        total = 0.0
        for pred, tgt in zip(preds, targets):
            total = total + sum(((pred[k] - tgt[k]) ** 2).mean() for k in DATA_FIELDS) / len(DATA_FIELDS)
        return total * (self.loss_scale / len(targets))

    def forward(self, data0: dict, forcings: dict, outer_steps: int):
        return self.rollout(data0, forcings, outer_steps)[1]


def resolve_resolution(name) -> str:
    """``2.8`` / ``"2.8"`` / ``"2.8deg"`` / ``"TL63"`` → the key of :data:`RESOLUTIONS`."""
    s = str(name).strip().lower().replace("°", "").replace("degrees", "").replace("deg", "")
    for key, spec in RESOLUTIONS.items():
        if s == key.replace("deg", "") or s == spec.grid.lower():
            return key
    raise KeyError(f"unknown resolution {name!r}; known: {sorted(RESOLUTIONS)}")


def make_fixer(section=None) -> Optional[nn.Module]:
    """Conservation fixer from a config ``fixer`` section (kind, fix_mass, fix_energy, energy_split).

    ``None`` gives the default: the FP64-accumulated packed fixer with the
    level-split energy correction.
    """
    if section is None:
        return LiteConservationFixer()
    kind = str(getattr(section, "kind", "lite")).lower()
    kw = dict(fix_mass=bool(section.fix_mass), fix_energy=bool(section.fix_energy),
              energy_split=str(getattr(section, "energy_split", "levels")))
    if kind == "none":
        return None
    if kind in ("f64", "fp64", "float64"):
        return F64ConservationFixer(**kw)
    if kind != "lite":
        raise ValueError(f"unknown fixer kind {kind!r} (lite | f64 | none)")
    return LiteConservationFixer(**kw)


def build_hybrid_gcm(resolution: str = "2.8deg", device: str | torch.device = "cpu",
                     policy: Optional[PrecisionPolicy] = None, seed: int = 0,
                     sht_precision: Optional[str] = None,
                     output_init_scale: float = 0.01, fixer=None,
                     **config_overrides) -> tuple[HybridGCM, SyntheticReanalysis]:
    """Random-init hybrid model of the given resolution plus its synthetic data source.

    ``fixer`` is a config ``fixer`` section (see :func:`make_fixer`); its
    ``cadence`` sets how often the fixer runs.

    ``output_init_scale`` multiplies the tower's last weight matrix: the random
    tendencies then stay small enough that multi-day rollouts of the random
    model remain stable at 1.4° and finer (with 0.1, one of two synthetic
    samples at 1.4° went unstable after ~22 simulated hours).
    """
    spec = RESOLUTIONS[resolve_resolution(resolution)]
    policy = policy or PrecisionPolicy.pzha_b200()
    torch.manual_seed(seed)
    grid0 = getattr(spherical_harmonic.Grid, spec.grid)()
    prec = sht_precision or policy.sht_precision(grid0.total_wavenumbers)
    grid = getattr(spherical_harmonic.Grid, spec.grid)(precision=prec)
    vertical = sigma_coordinates.SigmaCoordinates.equidistant(spec.layers)
    coords = coordinate_systems.CoordinateSystem(grid, vertical)
    units = SimUnits.from_si()
    t_ref = reference_temperature_profile(vertical.centers)
    data = SyntheticReanalysis(grid, seed=seed)
    forc = data.forcings(1)
    oro_nd = forc["orography"][0].double() / 6.37122e6
    oro_modal = grid.clip_wavenumbers(grid.with_precision("highest").to_modal(oro_nd))
    if spec.orography_filter is not None:
        _, l_tot = grid.modal_mesh
        L = grid.modal_shape[-1]
        oro_modal = oro_modal * torch.as_tensor(np.exp(-(np.asarray(l_tot) / (spec.orography_filter * L)) ** 8))
    oro_modal = oro_modal.float()

    dt = minutes_to_nondim(spec.dt_minutes)
    tau_dycore = minutes_to_nondim(120.0)
    tau_stab = minutes_to_nondim(4.0)
    cfg = ModelConfig(
        coords=coords, dt=dt, inner_steps=spec.physics_steps_per_output, dycore_substeps=spec.dycore_substeps,
        physics_specs=units, reference_temperature=t_ref, orography=oro_modal, precision_policy=policy,
        # the filters act once per dycore substep: attenuation per substep = substep dt / τ
        filter_attenuation=dt / spec.dycore_substeps / tau_dycore, filter_order=3, filter_cutoff=0.0,
        stability_filter_attenuation=dt / spec.dycore_substeps / tau_stab, stability_filter_order=10,
        stability_filter_cutoff=0.4,
        humidity_key="specific_humidity",
        cloud_keys=("specific_cloud_ice_water_content", "specific_cloud_liquid_water_content"),
        hyperdiffusion_order=2, hyperdiffusion_tau=minutes_to_nondim(spec.hyperdiffusion_hours * 60.0),
    )
    if config_overrides:  # e.g. hyperdiffusion_tau, filter settings
        cfg = dataclasses.replace(cfg, **config_overrides)
    n = spec.layers
    tracer_keys = tuple(sorted(TRACERS))
    n_in = n * (3 + len(tracer_keys)) + 1 + len(FORCING_FIELDS)
    n_out = n * (3 + len(tracer_keys)) + 1
    tower = ForwardTower(Mlp.uniform(n_in, n_out, hidden_size=spec.tower_width,
                                     hidden_layers=spec.tower_hidden_layers, activation=gelu_tanh))
    with torch.no_grad():
        tower.neural_net.layers[-1].weight.mul_(output_init_scale)
    # channel scales: [u, v (nondim), T', tracers (ice, liquid, humidity), ln ps, forcings]
    tr_in = {"specific_cloud_ice_water_content": 1e5, "specific_cloud_liquid_water_content": 1e5,
             "specific_humidity": 1e3}
    tr_out = {"specific_cloud_ice_water_content": 1e-8, "specific_cloud_liquid_water_content": 1e-8,
              "specific_humidity": 1e-6}
    in_scale = np.concatenate([np.full(2 * n, VELOCITY_SCALE / 10.0), np.full(n, 0.2)] +
                              [np.full(n, tr_in[k]) for k in tracer_keys] + [[10.0], np.ones(len(FORCING_FIELDS))])
    out_scale = np.concatenate([np.full(2 * n, 1e-5), np.full(n, 1e-3)] +
                               [np.full(n, tr_out[k]) for k in tracer_keys] + [[1e-5]])
    param = NodalColumnParameterization(grid, n, tracer_keys, tower, forcing_keys=FORCING_FIELDS,
                                        output_scale=out_scale, input_scale=in_scale)
    model = NeuralGCMModel(cfg, parameterization=param, conservation_fixer=make_fixer(fixer))
    if fixer is not None:
        model.set_fixer_cadence(int(getattr(fixer, "cadence", 1)))
    stats = data.stats()
    forcing_scale = {"sea_surface_temperature": (288.0, 0.1), "orography": (0.0, 1e-3)}
    enc = ColumnEncoder(coords, t_ref, data.levels, stats, FORCING_FIELDS, hidden=spec.encoder_width,
                        depth=spec.encoder_hidden_layers, orography_key="orography",
                        orography_unit_m=1.0 / forcing_scale["orography"][1])
    dec = ColumnDecoder(coords, t_ref, data.levels, stats, hidden=spec.encoder_width,
                        depth=spec.encoder_hidden_layers)
    gcm = HybridGCM(model, enc, dec, spec.physics_steps_per_output, FORCING_FIELDS, forcing_scale)
    return gcm.to(device), data
