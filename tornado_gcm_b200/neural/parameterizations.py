"""Neural physics parameterizations (Z3) — reference ``neural/parameterizations.py``.

* :class:`SimpleParameterization` / :class:`ModalNeuralDivCurlParameterization`
  keep the reference constructor signatures and state-dict keys; both accept
  leading batch dimensions.
* :class:`NodalColumnParameterization` is the per-column physics tower of the
  NeuralGCM design: nodal (u, v, T', tracers, ln ps) plus forcings →
  column network → nodal tendencies → modal (u, v mapped to ζ, δ by curl /
  divergence).  On CUDA the column network runs on the tcgen05 BF16 GEMMs.
"""

from __future__ import annotations

from typing import Callable, Optional, Sequence

import torch
import torch.nn as nn

from tornado_gcm_b200.core import primitive_equations, spherical_harmonic
from tornado_gcm_b200.core.spherical_harmonic import Grid

State = primitive_equations.State


def _forcing_channels(forcings: Optional[dict], like: torch.Tensor, lead: tuple, keys=None) -> list:
    """Nodal forcing fields as (…, 1, lon, lat) channels, sorted by key."""
    if not forcings:
        return []
    out = []
    for k in (keys if keys is not None else sorted(forcings)):
        if k not in forcings:
            continue
        v = forcings[k]
        if not isinstance(v, torch.Tensor):
            continue
        v = v.to(like.dtype)
        if v.shape[-2:] != like.shape[-2:]:
            continue
        while v.ndim < len(lead) + 3:
            v = v.unsqueeze(-3) if v.ndim == len(lead) + 2 else v.unsqueeze(0)
        out.append(v.expand(*lead, v.shape[-3], *like.shape[-2:]))
    return out


class SimpleParameterization(nn.Module):
    """MLP on the flattened modal state (test/debug parameterization)."""

    def __init__(self, modal_shape: tuple[int, int], n_levels: int, hidden_size: int = 64):
        super().__init__()
        self.modal_shape = tuple(modal_shape)
        self.n_levels = n_levels
        self.input_size = (3 * n_levels + 1) * modal_shape[0] * modal_shape[1]
        self.output_size = self.input_size
        self.net = nn.Sequential(
            nn.Linear(self.input_size, hidden_size), nn.GELU(),
            nn.Linear(hidden_size, hidden_size), nn.GELU(),
            nn.Linear(hidden_size, self.output_size),
        )
        nn.init.zeros_(self.net[-1].weight)
        nn.init.zeros_(self.net[-1].bias)

    def forward(self, state: State, forcings=None, memory=None) -> State:
        M, L = self.modal_shape
        nz = self.n_levels
        lead = state.vorticity.shape[:-3]
        flat = lambda t: t.reshape(*lead, -1)
        parts = [flat(state.vorticity), flat(state.divergence), flat(state.temperature_variation),
                 flat(state.log_surface_pressure)]
        if forcings:
            for k in sorted(forcings):
                f = forcings[k].to(parts[0].dtype)
                parts.append(f.reshape(*lead, -1) if f.shape[:len(lead)] == lead else
                             f.reshape(-1).expand(*lead, -1))
        x = torch.cat(parts, dim=-1)
        n_in = x.shape[-1]
        if n_in < self.input_size:
            x = torch.nn.functional.pad(x, (0, self.input_size - n_in))
        elif n_in > self.input_size:
            x = x[..., : self.input_size]
        y = self.net(x.to(self.net[0].weight.dtype))
        vol = nz * M * L
        vor = y[..., :vol].reshape(*lead, nz, M, L)
        div = y[..., vol:2 * vol].reshape(*lead, nz, M, L)
        tmp = y[..., 2 * vol:3 * vol].reshape(*lead, nz, M, L)
        lsp = y[..., 3 * vol:3 * vol + M * L].reshape(*lead, 1, M, L)
        return State(vor, div, tmp, lsp, {k: torch.zeros_like(v) for k, v in state.tracers.items()}, state.sim_time)


class ModalNeuralDivCurlParameterization(nn.Module):
    """Nodal features (ζ, δ, T', ln ps) → tower → nodal tendencies → modal (+filter)."""

    def __init__(self, grid: Grid, neural_net: nn.Module, n_levels: int,
                 filter_fn: Optional[Callable[[torch.Tensor], torch.Tensor]] = None,
                 use_mixed_precision_backward: bool = False, fwd_dtype: torch.dtype = torch.bfloat16):
        super().__init__()
        self.grid = grid
        self.neural_net = neural_net
        self.n_levels = n_levels
        self.filter_fn = filter_fn
        self.use_mixed_precision_backward = use_mixed_precision_backward
        self.fwd_dtype = fwd_dtype

    def _state_to_nodal_features(self, state: State) -> torch.Tensor:
        stacked = torch.cat([state.vorticity, state.divergence, state.temperature_variation,
                             state.log_surface_pressure], dim=-3)
        return self.grid.to_nodal(stacked)

    def _nodal_output_to_state(self, y: torch.Tensor, state: State) -> State:
        nz = self.n_levels
        modal = self.grid.to_modal(y[..., : 3 * nz + 1, :, :])
        vor, div, tmp, sp = torch.split(modal, [nz, nz, nz, 1], dim=-3)
        if self.filter_fn is not None:
            vor, div, tmp, sp = (self.filter_fn(t) for t in (vor, div, tmp, sp))
        return State(vor, div, tmp, sp, {k: torch.zeros_like(v) for k, v in state.tracers.items()}, state.sim_time)

    def forward(self, state: State, forcings=None, memory=None) -> State:
        x = self._state_to_nodal_features(state)
        extra = _forcing_channels(forcings, x, tuple(x.shape[:-3]))
        if extra:
            x = torch.cat([x] + extra, dim=-3)
        if self.use_mixed_precision_backward and self.training:
            from tornado_gcm_b200.training.optimization import MixedPrecisionBackward

            y = MixedPrecisionBackward.apply(self.neural_net, x, self.fwd_dtype)
        else:
            y = self.neural_net(x)
        return self._nodal_output_to_state(y.to(state.vorticity.dtype), state)


class NodalColumnParameterization(nn.Module):
    """Column physics: nodal (u, v, T', tracers, ln ps, forcings) → nodal tendencies.

    Input channels per column: ``2n (u, v) + n (T') + n·len(tracers) + 1
    (ln ps) + len(forcing_keys)``.  Output channels: the same prognostic
    set (without forcings).  Velocity tendencies are converted to vorticity
    / divergence tendencies with the spectral curl / divergence of
    ``(u, v)/cosθ`` as in NeuralGCM's div-curl parameterizations.
    """

    def __init__(self, grid: Grid, n_levels: int, tracer_keys: Sequence[str], neural_net: nn.Module,
                 forcing_keys: Sequence[str] = (), output_scale=1.0, input_scale=None,
                 filter_fn: Optional[Callable[[torch.Tensor], torch.Tensor]] = None,
                 compute_dtype: torch.dtype = torch.bfloat16):
        super().__init__()
        self.grid = grid
        self.n_levels = n_levels
        self.tracer_keys = tuple(tracer_keys)
        self.forcing_keys = tuple(forcing_keys)
        self.tower = neural_net
        self.filter_fn = filter_fn
        self.compute_dtype = compute_dtype
        osc = torch.as_tensor(output_scale, dtype=torch.float32).reshape(-1)
        if osc.numel() == 1:
            osc = osc.expand(self.n_outputs).clone()
        self.register_buffer("output_scale", osc.reshape(-1, 1, 1))
        isc = torch.ones(self.n_inputs) if input_scale is None else torch.as_tensor(input_scale, dtype=torch.float32)
        self.register_buffer("input_scale", isc.reshape(-1, 1, 1))

    @property
    def n_inputs(self) -> int:
        return self.n_levels * (3 + len(self.tracer_keys)) + 1 + len(self.forcing_keys)

    @property
    def n_outputs(self) -> int:
        return self.n_levels * (3 + len(self.tracer_keys)) + 1

    def nodal_prognostics(self, state: State) -> torch.Tensor:
        """(…, C, lon, lat) with channels [u, v, T', tracers…, ln ps] (u, v physical)."""
        g = self.grid
        uc, vc = spherical_harmonic.get_cos_lat_vector(state.vorticity, state.divergence, g, clip=False)
        tr = [state.tracers[k] if k in state.tracers else torch.zeros_like(state.temperature_variation)
              for k in self.tracer_keys]
        nodal = g.to_nodal(torch.cat([uc, vc, state.temperature_variation] + tr + [state.log_surface_pressure],
                                     dim=-3))
        n = self.n_levels
        sec = 1.0 / g.const("cos_lat", nodal.device, nodal.dtype)
        u = nodal[..., :n, :, :] * sec
        v = nodal[..., n:2 * n, :, :] * sec
        return torch.cat([u, v, nodal[..., 2 * n:, :, :]], dim=-3)

    def forward(self, state: State, forcings=None, memory=None) -> State:
        x = self.nodal_prognostics(state)
        lead = tuple(x.shape[:-3])
        extra = _forcing_channels(forcings, x, lead, self.forcing_keys)
        if extra:
            x = torch.cat([x] + extra, dim=-3)
        elif self.forcing_keys:
            x = torch.cat([x, x.new_zeros(*lead, len(self.forcing_keys), *x.shape[-2:])], dim=-3)
        y = self.tower((x * self.input_scale).to(self.compute_dtype)).to(state.vorticity.dtype) * self.output_scale
        return self.nodal_tendency_to_modal(y, state)

    # ── packed path (lat-major nodal, table-driven spectral operators) ──────
    def _packed_recipes(self, state_keys: tuple):
        cache = self.__dict__.setdefault("_recipes", {})
        r = cache.get(state_keys)
        if r is None:
            from tornado_gcm_b200.ops import spectral

            r = (spectral.param_pre_recipe(self.grid, self.n_levels, state_keys, self.tracer_keys),
                 spectral.param_post_recipe(self.grid, self.n_levels, state_keys, self.tracer_keys))
            cache[state_keys] = r
        return r

    def _lat_factors(self, device, dtype):
        """Per-channel × per-latitude input and output factors, (C, J, 1) each."""
        n = self.n_levels
        sec = (1.0 / self.grid.const("cos_lat", device, dtype)).reshape(-1, 1)  # (J, 1)
        cin = self.n_outputs
        fin = self.input_scale[:cin].to(device, dtype).expand(cin, sec.shape[0], 1).clone()
        fin[: 2 * n] = fin[: 2 * n] * sec
        fout = self.output_scale.to(device, dtype).expand(cin, sec.shape[0], 1).clone()
        fout[: 2 * n] = fout[: 2 * n] * sec
        return fin, fout

    def _token_path_ok(self, nod: torch.Tensor) -> bool:
        """The column tower can run on BF16 token rows (ops/tokens.py) instead of a permuted copy."""
        from tornado_gcm_b200.neural.standard_layers import Mlp
        from tornado_gcm_b200.neural.towers import ForwardTower
        from tornado_gcm_b200.ops import linear as linear_ops

        t = self.tower
        if not (nod.is_cuda and isinstance(t, ForwardTower) and isinstance(t.neural_net, Mlp)
                and t.final_activation is None and t.feature_axis % 4 == 1 and self.compute_dtype == torch.bfloat16):
            return False
        return None not in t.neural_net.layer_activations() and linear_ops.supports(nod, t.neural_net.layers)

    def _lat_factors_2d(self, device):
        """(C, J) fp32 input and output factors (cached per device)."""
        cache = self.__dict__.setdefault("_latf2d", {})
        key = (str(device), self.input_scale._version, self.output_scale._version)
        ent = cache.get(key)
        if ent is None:
            fin, fout = self._lat_factors(device, torch.float32)
            ent = (fin[..., 0].contiguous(), fout[..., 0].contiguous())
            cache.clear()
            cache[key] = ent
        return ent

    def _tower_tokens(self, nod, forcings, B: int, C: int, J: int, I: int) -> torch.Tensor:
        """Column tower on BF16 token rows: scale + forcing columns + layout change in one kernel each way."""
        from tornado_gcm_b200.ops import linear as linear_ops, tokens as tok_ops

        net = self.tower.neural_net
        nf = len(self.forcing_keys)
        ld = (C + nf + 7) // 8 * 8
        ex = None
        if nf:
            like = nod.new_empty((1, 1, I, J))
            extra = _forcing_channels(forcings, like, (B,), self.forcing_keys)
            if extra:  # (B, nf, I, J) → (B·J·I, nf) rows, input-scaled, BF16
                f = torch.cat(extra, dim=-3) * self.input_scale[C:].to(nod.dtype)
                ex = f.permute(0, 3, 2, 1).reshape(B * J * I, nf).to(torch.bfloat16).contiguous()
        fin, fout = self._lat_factors_2d(nod.device)
        tok = tok_ops.nodal_to_tokens(nod, fin, ex, ld)
        fsdp = self.__dict__.get("_fsdp_layers")
        if fsdp is not None and not torch.is_grad_enabled():
            from tornado_gcm_b200.parallel.fsdp_gather import gathered_mlp_forward

            hid = gathered_mlp_forward(fsdp, tok)[:, : self.n_outputs]
        else:
            hid = linear_ops.mlp_forward(tok, net.layers, net.layer_activations(), last_bf16=True)
        return tok_ops.tokens_to_nodal(hid, fout, B, J, I, ld_grad=(C + 7) // 8 * 8)

    def shard_tower_weights(self, group=None) -> None:
        """FSDP-style inference: every rank keeps 1/W of each tower layer's BF16 weight rows in
        symmetric memory and the GEMMs read the other rows from the peers as they run (the
        all-gather fused into the consuming GEMM, ``parallel/fsdp_gather.py``).  Used when no
        gradient is being recorded; training keeps the replicated weights."""
        from tornado_gcm_b200.parallel.fsdp_gather import shard_mlp

        self.__dict__["_fsdp_layers"] = shard_mlp(self.tower.neural_net, group=group)

    def forward_packed(self, y: torch.Tensor, state_keys, forcings=None) -> torch.Tensor:
        """Packed state ``(B, C, 2M-1, L)`` → packed tendency of the same layout.

        Same mathematics as :meth:`forward` with the spectral pre/post work in
        two table-driven kernels and the nodal fields kept latitude-major
        ``(B, C, J, I)`` between the transforms (the column network is
        pointwise, so its layout does not matter).
        """
        from tornado_gcm_b200.ops import dycore as dyops, spectral

        state_keys = tuple(state_keys)
        g = self.grid
        M2, L = g.modal_shape
        I, J = g.nodal_shape
        B = y.shape[0]
        pre, post = self._packed_recipes(state_keys)
        lp = (L + 3) // 4 * 4 if y.is_cuda else L
        xm = spectral.spectral_linear(y, pre, out_lpad=lp, grad_lpad=L)
        C = self.n_outputs
        nod = dyops._synth_lat(xm.reshape(B * C, M2, L), g).reshape(B, C, J, I)
        if self._token_path_ok(nod):
            out = self._tower_tokens(nod, forcings, B, C, J, I)
            modal = dyops._anal_lat(out.reshape(B * C, J, I), g).reshape(B, C, M2, L)
            res = spectral.spectral_linear(modal, post, out_lpad=L, grad_lpad=lp)
            return self.filter_fn(res) if self.filter_fn is not None else res
        fin, fout = self._lat_factors(y.device, nod.dtype)
        x = nod * fin
        if self.forcing_keys:
            like = y.new_empty((1, 1, I, J))
            extra = _forcing_channels(forcings, like, (B,), self.forcing_keys)
            nf = len(self.forcing_keys)
            if extra:
                f = torch.cat(extra, dim=-3).transpose(-1, -2)
                x = torch.cat([x, f * self.input_scale[C:].to(f.dtype)], dim=-3)
            else:
                x = torch.cat([x, x.new_zeros(B, nf, J, I)], dim=-3)
        out = self.tower(x.to(self.compute_dtype)).to(nod.dtype) * fout
        modal = dyops._anal_lat(out.reshape(B * C, J, I), g).reshape(B, C, M2, L)
        res = spectral.spectral_linear(modal, post, out_lpad=L, grad_lpad=lp)
        if self.filter_fn is not None:
            res = self.filter_fn(res)
        return res

    def nodal_tendency_to_modal(self, y: torch.Tensor, state: State) -> State:
        g = self.grid
        n = self.n_levels
        cos = g.const("cos_lat", y.device, y.dtype)
        # u, v tendencies → divide by cosθ before the transform (curl/div of v·cosθ / cos²θ)
        uv = y[..., : 2 * n, :, :] / cos
        modal = g.to_modal(torch.cat([uv, y[..., 2 * n:, :, :]], dim=-3))
        um, vm = modal[..., :n, :, :], modal[..., n:2 * n, :, :]
        vort = g.curl_cos_lat((um, vm), clip=True)
        div = g.div_cos_lat((um, vm), clip=True)
        temp = modal[..., 2 * n:3 * n, :, :]
        tr = {}
        off = 3 * n
        for k in self.tracer_keys:
            tr[k] = modal[..., off:off + n, :, :]
            off += n
        lsp = modal[..., off:off + 1, :, :]
        out = State(vort, div, temp, lsp, {k: tr.get(k, torch.zeros_like(v)) for k, v in state.tracers.items()},
                    state.sim_time)
        if self.filter_fn is not None:
            out = out.tree_map(self.filter_fn)
        return out


class JaxAlignedDivCurlParameterization(nn.Module):
    """NeuralGCM's divergence/curl physics parameterization on the full feature set
    — reference ``neural/parameterizations.py:240-504``.

    ``feature_extractor`` (a :class:`~tornado_gcm_b200.neural.features.CombinedFeatures`
    with memory features) → ``feature_transform`` (normalise / level-scale /
    soft-clip) → features packed in sorted-key order → ``neural_net`` →
    output split by ``output_keys``/``output_sizes`` → optional
    ``tendency_transform`` → modal tendencies: nodal (u, v) become (ζ, δ)
    tendencies through ``u·secφ``, ``v·secφ`` and the cos-lat curl /
    divergence, everything in one batched analysis
    (:class:`~tornado_gcm_b200.neural.transforms.ToModalWithDivCurl`).
    Absent cloud tracers enter the features as zeros, so the packed width is
    fixed by the checkpoint, and the memory features fall back to the current
    state when no complete memory is supplied.
    """

    DEFAULT_OUTPUT_KEYS = ["specific_cloud_ice_water_content", "specific_cloud_liquid_water_content",
                           "specific_humidity", "temperature_variation", "u", "v"]
    _EPD_TRACER_KEYS = ("specific_humidity", "specific_cloud_liquid_water_content",
                        "specific_cloud_ice_water_content")

    def __init__(self, grid: Grid, neural_net: nn.Module, feature_extractor: nn.Module, feature_transform: nn.Module,
                 tendency_transform: Optional[nn.Module] = None, n_levels: int = 32,
                 filter_fn: Optional[Callable] = None, output_keys: Optional[list] = None,
                 output_sizes: Optional[list] = None):
        super().__init__()
        from tornado_gcm_b200.neural.transforms import ToModalWithDivCurl

        self.grid = grid
        self.neural_net = neural_net
        self.feature_extractor = feature_extractor
        self.feature_transform = feature_transform
        self.tendency_transform = tendency_transform
        self.n_levels = n_levels
        self.filter_fn = filter_fn
        self.output_keys = list(output_keys or self.DEFAULT_OUTPUT_KEYS)
        self.output_sizes = list(output_sizes or [n_levels] * len(self.output_keys))
        self._to_modal = ToModalWithDivCurl(grid, "u", "v")

    def _state_to_dict(self, state: State) -> dict:
        tracers = dict(state.tracers or {})
        for k in self._EPD_TRACER_KEYS:
            tracers.setdefault(k, torch.zeros_like(state.temperature_variation))
        d = {"vorticity": state.vorticity, "divergence": state.divergence,
             "temperature_variation": state.temperature_variation,
             "log_surface_pressure": state.log_surface_pressure, "tracers": tracers}
        if state.sim_time is not None:
            d["sim_time"] = torch.as_tensor(state.sim_time, dtype=torch.float32,
                                            device=state.vorticity.device).reshape(1)
        return d

    def _memory_to_dict(self, memory) -> Optional[dict]:
        if memory is None or isinstance(memory, dict):
            return memory
        if hasattr(memory, "vorticity") and hasattr(memory, "divergence"):
            return self._state_to_dict(State(memory.vorticity, memory.divergence, memory.temperature_variation,
                                             memory.log_surface_pressure, dict(getattr(memory, "tracers", {}) or {}),
                                             getattr(memory, "sim_time", None)))
        return None

    @staticmethod
    def _memory_dict_matches_inputs(mem: Optional[dict], ref: dict) -> bool:
        if not mem or any(k not in mem for k in ("vorticity", "divergence", "temperature_variation",
                                                  "log_surface_pressure")):
            return False
        rt, mt = ref.get("tracers"), mem.get("tracers")
        return not rt or (isinstance(mt, dict) and set(rt) <= set(mt))

    def _unpack_output(self, y: torch.Tensor) -> dict:
        return dict(zip(self.output_keys, torch.split(y, self.output_sizes, dim=-3)))

    def _nodal_tendencies_to_modal_state(self, tend: dict, state: State) -> State:
        nodal = {k: v for k, v in tend.items() if k in ("u", "v", "temperature_variation") or k in state.tracers}
        if ("u" in nodal) != ("v" in nodal):
            nodal.pop("u", None), nodal.pop("v", None)
        modal = self._to_modal(nodal)
        if self.filter_fn is not None:
            modal = {k: self.filter_fn(v) for k, v in modal.items()}
        z = torch.zeros_like
        return State(modal.get("vorticity", z(state.vorticity)), modal.get("divergence", z(state.divergence)),
                     modal.get("temperature_variation", z(state.temperature_variation)),
                     z(state.log_surface_pressure),
                     {k: modal.get(k, z(v)) for k, v in state.tracers.items()}, state.sim_time)

    def forward(self, state: State, forcings: Optional[dict] = None, memory=None) -> State:
        from tornado_gcm_b200.neural.features import pack_features

        inputs = self._state_to_dict(state)
        mem = self._memory_to_dict(memory)
        if not self._memory_dict_matches_inputs(mem, inputs):
            mem = inputs
        feats = self.feature_transform(self.feature_extractor(inputs, memory=mem, forcing=forcings))
        tend = self._unpack_output(self.neural_net(pack_features(feats)))
        if self.tendency_transform is not None:
            tend = self.tendency_transform(tend)
        return self._nodal_tendencies_to_modal_state(tend, state)
