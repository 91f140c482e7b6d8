"""Trainers — reference ``training/trainer.py:29-816``.

* :class:`MixedPrecisionTrainer` — the reference API (``train_step(batch,
  rollout_steps)`` with a user ``loss_fn``), explicit PZHA zones instead of a
  global autocast, fused AdamW / grad clipping / EMA with no host syncs,
  and one packed metric all-reduce.
* :class:`GCMTrainer` — end-to-end trainer for :class:`HybridGCM`
  (encoder → rollout → decoder → loss) that can capture the whole
  optimizer step (forward, backward-through-rollout, clipping, AdamW, EMA)
  in one CUDA graph and replay it.
* :class:`VariablePrecisionTraining`, :func:`nested_checkpoint_scan`,
  :class:`NaNRecoveryTrainer`, :class:`MultiStageTrainer`,
  :class:`HostOffloadCheckpoint` — same roles as in the reference.
"""

from __future__ import annotations

import dataclasses
import logging
import os
import math
from typing import Any, Callable, Sequence

import torch
import torch.nn as nn
import torch.utils.checkpoint as checkpoint_util

from tornado_gcm_b200.core.primitive_equations import State
from tornado_gcm_b200.precision.policy import PrecisionPolicy

logger = logging.getLogger(__name__)


@dataclasses.dataclass
class TrainingPhaseConfig:
    name: str
    budget_fraction: float
    nn_dtype: torch.dtype
    dycore_tf32: bool
    fixer_dtype: torch.dtype
    rollout_steps: int
    batch_size_multiplier: float


@dataclasses.dataclass
class TrainStage:
    duration: int
    rollout_steps: int = 16
    batch_size: int | None = None
    loss_fn: nn.Module | None = None
    learning_rate: float | None = None
    description: str = ""


@dataclasses.dataclass
class AutoRestartConfig:
    max_nan_restarts: int = 0
    restart_lookback_steps: int = 100
    error_with_nan_loss: bool = True


@dataclasses.dataclass
class AutoRestart:
    iteration: int = 0
    began_at: int | None = None


PHASE_1 = TrainingPhaseConfig("low_precision_pretrain", 0.60, torch.bfloat16, False, torch.float32, 4, 2.0)
PHASE_2 = TrainingPhaseConfig("mixed_precision_train", 0.30, torch.bfloat16, True, torch.float64, 16, 1.0)
PHASE_3 = TrainingPhaseConfig("high_precision_finetune", 0.10, torch.float32, True, torch.float64, 32, 0.5)
DEFAULT_PHASES = [PHASE_1, PHASE_2, PHASE_3]


def _unwrap(model: nn.Module) -> nn.Module:
    raw = model
    while hasattr(raw, "module"):
        raw = raw.module
    return raw


class _Ema:
    """FP32 EMA of parameters, updated with one foreach lerp (no host sync)."""

    def __init__(self, model: nn.Module, num_steps: int):
        self.decay = 1.0 - 2.0 / (num_steps + 1)
        self.names = [n for n, _ in model.named_parameters()]
        self.params = [p for _, p in model.named_parameters()]
        self.shadow = [p.detach().clone().float() for p in self.params]

    @torch.no_grad()
    def update(self):
        src = [p.detach().float() if p.dtype != torch.float32 else p.detach() for p in self.params]
        torch._foreach_lerp_(self.shadow, src, 1.0 - self.decay)

    def state_dict(self) -> dict:
        return dict(zip(self.names, self.shadow))


class MixedPrecisionTrainer:
    """Per-zone precision trainer; BF16 NN without loss scaling."""

    def __init__(self, model: nn.Module, optimizer: torch.optim.Optimizer, loss_fn: nn.Module,
                 policy: PrecisionPolicy | None = None, max_grad_norm: float = 1.0, ema_num_steps: int = 1999):
        self.model = model
        self.optimizer = optimizer
        self.loss_fn = loss_fn
        self.policy = policy or PrecisionPolicy()
        self.max_grad_norm = max_grad_norm
        self.ema_num_steps = ema_num_steps
        self.ema_decay = 1.0 - 2.0 / (ema_num_steps + 1)
        self.step_count = 0
        self._raw_model = _unwrap(model)
        self._ema = _Ema(model, ema_num_steps)

    @property
    def _ema_params(self) -> dict:
        return self._ema.state_dict()

    def _update_ema(self) -> None:
        self._ema.update()

    def get_ema_state_dict(self) -> dict:
        return self._ema.state_dict()

    def _to_device(self, obj, device):
        if isinstance(obj, State):
            return obj.tree_map(lambda t: t.to(device, non_blocking=True))
        if isinstance(obj, torch.Tensor):
            return obj.to(device, non_blocking=True)
        if isinstance(obj, list):
            return [self._to_device(x, device) for x in obj]
        if isinstance(obj, dict):
            return {k: self._to_device(v, device) for k, v in obj.items()}
        return obj

    def _rollout(self, initial_state, steps: int, forcings=None):
        state = initial_state
        traj = []
        for i in range(steps):
            f = forcings[i] if isinstance(forcings, list) else forcings
            state = self._raw_model.step(state, forcings=f)
            traj.append(state)
        return traj, initial_state

    def _rollout_nested(self, initial_state, steps, forcings, frequencies, dt=1, checkpoint_level=-1):
        from tornado_gcm_b200.core.scan_utils import nested_rollout

        _, traj = nested_rollout(step_fn=self._raw_model.step, initial_state=initial_state, forcings=forcings,
                                 frequencies=frequencies, dt=dt, checkpoint_level=checkpoint_level)
        return traj, initial_state

    def compute_loss(self, batch: dict, rollout_steps: int) -> dict:
        device = next(self.model.parameters()).device
        inputs = self._to_device(batch["inputs"], device)
        targets = self._to_device(batch["targets"], device)
        forcings = self._to_device(batch.get("forcings"), device)
        preds, init = self._rollout(inputs, rollout_steps, forcings=forcings)
        diagnostics = {}
        if preds and isinstance(preds[0], State):
            from tornado_gcm_b200.neural.diagnostics import compute_trajectory_diagnostics

            diagnostics = compute_trajectory_diagnostics(preds, init)
        kwargs = dict(predictions=preds, targets=targets)
        extra = dict(energies=diagnostics.get("energies", batch.get("energies")),
                     masses=diagnostics.get("masses", batch.get("masses")),
                     precipitation=diagnostics.get("precipitation", batch.get("precipitation")),
                     evaporation=diagnostics.get("evaporation", batch.get("evaporation")),
                     step=self.step_count)
        try:
            out = self.loss_fn(**kwargs, **extra)
        except TypeError:
            out = self.loss_fn(**kwargs)
        if isinstance(out, torch.Tensor):
            out = {"total": out}
        return out

    def train_step(self, batch: dict[str, Any], rollout_steps: int = 1) -> dict[str, float]:
        from tornado_gcm_b200.ops import linear as linear_ops
        from tornado_gcm_b200.parallel.metrics import all_reduce_metrics

        self.model.train()
        self.optimizer.zero_grad(set_to_none=True)
        self.policy.apply_tf32_setting()
        linear_ops.begin_step()
        loss_dict = self.compute_loss(batch, rollout_steps)
        loss_dict["total"].backward()
        gn = torch.nn.utils.clip_grad_norm_(self.model.parameters(),
                                            self.max_grad_norm if self.max_grad_norm > 0 else float("inf"),
                                            foreach=True)
        loss_dict["pre_clip_grad_norm"] = gn
        self.optimizer.step()
        self._update_ema()
        self.step_count += 1
        return all_reduce_metrics({k: v.detach() if torch.is_tensor(v) else torch.tensor(float(v))
                                   for k, v in loss_dict.items()})

    # CLI-facing helpers (the reference CLI calls these on the trainer)
    def save_checkpoint(self, path, phase: int = 0, best_val_loss: float = float("inf")):
        from tornado_gcm_b200.training.checkpointing import TrainingState, save_checkpoint

        save_checkpoint(path, self.model, self.optimizer, TrainingState(self.step_count, phase, best_val_loss),
                        self.get_ema_state_dict())

    def load_checkpoint(self, path):
        from tornado_gcm_b200.training.checkpointing import load_checkpoint

        ts = load_checkpoint(path, self.model, self.optimizer)
        self.step_count = ts.step
        return ts


class GCMTrainer:
    """Hybrid-GCM training step: encode → K×6 h rollout → decode → MSE → AdamW.

    ``graph=True`` captures one complete optimizer step in a CUDA graph on
    the first call (after warm-up steps on a side stream) and replays it;
    inputs are copied into static device buffers from pinned host memory.
    """

    def __init__(self, gcm: nn.Module, lr: float = 1e-4, weight_decay: float = 0.0, max_grad_norm: float = 1.0,
                 ema_num_steps: int = 1999, graph: bool = False, betas=(0.9, 0.95), eps: float = 1e-6,
                 data_parallel: bool = False, grad_average: bool = True, check_errors_every: int = 0):
        """``data_parallel``: replicated weights, gradients reduced over the ranks after
        backward — averaged (data parallelism: each rank's loss is a full loss of its own
        samples) or summed with ``grad_average=False`` (a model sharded over the ranks:
        each rank's loss is its share of one global loss).  ``data_parallel="sharded"``:
        data parallelism with the averaged gradients and the AdamW state split over the
        ranks (:class:`~tornado_gcm_b200.parallel.sharded_optim.ShardedAdamW`: reduce-scatter,
        clip by the global norm, AdamW on the own chunk, all-gather of the weights).
        ``check_errors_every``: every that many steps, read the device error flag that the
        kernels set when a bounded wait expires or a table index is out of range, and raise
        (one host synchronisation; 0 leaves the check to the caller, see
        :meth:`check_device_errors`)."""
        self.gcm = gcm
        params = [p for p in gcm.parameters() if p.requires_grad]
        self.dp = None
        self.zero_opt = None
        dev = params[0].device
        if data_parallel == "sharded":
            from tornado_gcm_b200.parallel.sharded_optim import ShardedAdamW

            if not grad_average:
                raise ValueError("the sharded optimizer averages gradients (data parallelism)")
            self.zero_opt = ShardedAdamW(params, lr=lr, weight_decay=weight_decay, betas=betas, eps=eps,
                                         max_grad_norm=max_grad_norm, capturable=graph and dev.type == "cuda")
            self.zero_opt.zero_grad()
            self._flat = self.zero_opt.flat_grad
        elif data_parallel:
            from tornado_gcm_b200.parallel.ddp import GradientAllReducer

            self.dp = GradientAllReducer(params, average=grad_average)
            self.dp.broadcast_parameters()
            self.dp.zero()
            self._flat = self.dp.flat
        else:
            # one flat fp32 gradient buffer with each parameter's .grad a view of it:
            # zeroing is one launch, and gradients accumulate in place
            self._flat = torch.zeros(sum(p.numel() for p in params), dtype=torch.float32, device=dev)
        self._grad_views = []
        off = 0
        for p in params:
            self._grad_views.append(self._flat[off:off + p.numel()].view_as(p))
            off += p.numel()
        # the column networks add their weight/bias gradients straight into .grad
        self.fused_grad_accumulation = dev.type == "cuda"
        self.device = dev
        if self.zero_opt is not None:
            self.optimizer = self.zero_opt.optimizer
        else:
            self.optimizer = torch.optim.AdamW(params, lr=lr, weight_decay=weight_decay, betas=betas, eps=eps,
                                               fused=dev.type == "cuda", capturable=graph and dev.type == "cuda")
        self.params = params
        self.max_grad_norm = max_grad_norm
        self.ema = _Ema(gcm, ema_num_steps)
        self.use_graph = graph and dev.type == "cuda"
        self._graph = None
        self._static = None
        self._static_loss = None
        self.step_count = 0
        self.check_errors_every = int(check_errors_every)
        # host-side liveness check and fault injection between steps (see parallel/elastic.py)
        self.heartbeat = None
        self._fault_spec = os.environ.get("TGCM_FAULT_INJECT") or None

    def attach_heartbeat(self, heartbeat) -> None:
        """Beat and check peers before every step; a dead peer raises before any launch."""
        self.heartbeat = heartbeat

    def _pre_step(self) -> None:
        if self._fault_spec is not None:
            from tornado_gcm_b200.parallel.elastic import maybe_inject_fault
            from tornado_gcm_b200.parallel.ddp import get_rank

            maybe_inject_fault(get_rank(), self.step_count, self._fault_spec)
        if self.heartbeat is not None:
            self.heartbeat.beat(self.step_count)
            self.heartbeat.check(self.step_count)

    def _step_body(self, data0, targets, forcings):
        from tornado_gcm_b200.ops import linear as linear_ops

        linear_ops.begin_step()
        self._flat.zero_()
        self._attach()
        loss = self.gcm.loss(data0, targets, forcings)
        prev = linear_ops.fused_grad_accumulation()
        linear_ops.set_fused_grad_accumulation(self.fused_grad_accumulation)
        try:
            loss.backward()
        finally:
            linear_ops.set_fused_grad_accumulation(prev)
        if self.zero_opt is not None:
            self.zero_opt.step()
        else:
            if self.dp is not None:
                self.dp.reduce()
            torch.nn.utils.clip_grad_norm_(self.params, self.max_grad_norm, foreach=True)
            self.optimizer.step()
        self.ema.update()
        return loss.detach()

    def _attach(self):
        for p, v in zip(self.params, self._grad_views):
            if p.grad is None or p.grad.data_ptr() != v.data_ptr():
                p.grad = v

    def _zero(self):
        self._flat.zero_()
        self._attach()
        if self.zero_opt is not None:
            self.zero_opt.attach()

    @property
    def grad_reducer(self) -> str:
        """Which collective reduces the gradients (recorded in benchmark lines)."""
        if self.zero_opt is not None:
            return "sharded optimizer: " + self.zero_opt.backend
        return self.dp.backend if self.dp is not None else "none (one rank)"

    def train_step(self, data0: dict, targets: list, forcings: dict) -> torch.Tensor:
        """One optimizer step; returns the loss as a 0-d device tensor."""
        self.gcm.train()
        self._pre_step()
        if not self.use_graph:
            self._zero()
            loss = self._step_body(data0, targets, forcings)
        else:
            if self._graph is None:
                self._capture(data0, targets, forcings)
            self._copy_in(data0, targets, forcings)
            self._graph.replay()
            loss = self._static_loss
        self.step_count += 1
        if self.check_errors_every > 0 and self.step_count % self.check_errors_every == 0:
            self.check_device_errors()
        return loss

    def check_device_errors(self) -> None:
        """Raise if a kernel of this device recorded an error (expired bounded wait, bad index)."""
        if self.device.type == "cuda":
            from tornado_gcm_b200.ops import _ext

            _ext.check_error_flag(self.device)

    # ── CUDA graph machinery ─────────────────────────────────────────
    def _copy_in(self, data0, targets, forcings):
        sd, st, sf = self._static
        for k, v in data0.items():
            sd[k].copy_(v, non_blocking=True)
        for i, t in enumerate(targets):
            for k, v in t.items():
                st[i][k].copy_(v, non_blocking=True)
        for k, v in forcings.items():
            sf[k].copy_(v, non_blocking=True)

    def _capture(self, data0, targets, forcings, warmup: int = 2):
        dev = self.device
        sd = {k: v.to(dev).clone() for k, v in data0.items()}
        st = [{k: v.to(dev).clone() for k, v in t.items()} for t in targets]
        sf = {k: v.to(dev).clone() for k, v in forcings.items()}
        self._static = (sd, st, sf)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._zero()
                self._step_body(sd, st, sf)
        torch.cuda.current_stream(dev).wait_stream(s)
        self._zero()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._static_loss = self._step_body(sd, st, sf)
        self._graph = g
        self.step_count += warmup

    def release_graph(self):
        self._graph = None
        self._static = None


class VariablePrecisionTraining:
    """Three-phase variable-precision schedule by budget fraction."""

    def __init__(self, trainer: MixedPrecisionTrainer, total_steps: int,
                 phases: list[TrainingPhaseConfig] | None = None, base_batch_size: int = 32):
        self.trainer = trainer
        self.total_steps = total_steps
        self.phases = phases or DEFAULT_PHASES
        self.base_batch_size = base_batch_size
        self._boundaries = []
        acc = 0
        for ph in self.phases:
            acc += int(total_steps * ph.budget_fraction)
            self._boundaries.append(acc)

    def current_phase(self, step: int) -> TrainingPhaseConfig:
        for b, ph in zip(self._boundaries, self.phases):
            if step < b:
                return ph
        return self.phases[-1]

    def current_batch_size(self, step: int) -> int:
        return max(1, int(self.base_batch_size * self.current_phase(step).batch_size_multiplier))

    def configure_for_step(self, step: int) -> TrainingPhaseConfig:
        ph = self.current_phase(step)
        pol = self.trainer.policy
        pol.z3_compute_dtype = ph.nn_dtype
        pol.z1_use_tf32 = ph.dycore_tf32
        pol.z2_compute_dtype = ph.fixer_dtype
        pol.apply_tf32_setting()
        return ph

    def train_step(self, batch: dict, step: int) -> dict:
        ph = self.configure_for_step(step)
        res = self.trainer.train_step(batch, rollout_steps=ph.rollout_steps)
        res["phase"] = self.phases.index(ph)
        return res


def _flatten(s):
    if isinstance(s, torch.Tensor):
        return (s,), None
    if isinstance(s, State):
        keys = sorted(s.tracers)
        return (s.vorticity, s.divergence, s.temperature_variation, s.log_surface_pressure,
                *(s.tracers[k] for k in keys)), {"keys": keys, "sim_time": s.sim_time}
    raise TypeError(f"unsupported state type {type(s)}")


def _unflatten(ts, meta):
    if meta is None:
        return ts[0]
    return State(ts[0], ts[1], ts[2], ts[3], {k: ts[4 + i] for i, k in enumerate(meta["keys"])}, meta["sim_time"])


def nested_checkpoint_scan(step_fn: Callable, initial_state, total_steps: int, segment_length: int = 4,
                           use_reentrant: bool = False):
    """Rollout in checkpointed segments (activations recomputed in backward)."""
    traj: list = []
    flat, meta = _flatten(initial_state)
    holder = {"meta": meta, "traj": []}
    remaining = total_steps
    while remaining > 0:
        n = min(segment_length, remaining)

        def seg(*args, _n=n):
            st = _unflatten(args, holder["meta"])
            out = []
            for _ in range(_n):
                st = step_fn(st)
                out.append(st)
            f, m = _flatten(st)
            holder["meta"] = m
            holder["traj"] = out
            return f

        res = checkpoint_util.checkpoint(seg, *flat, use_reentrant=use_reentrant)
        flat = (res,) if isinstance(res, torch.Tensor) else res
        traj.extend(holder["traj"])
        remaining -= n
    return _unflatten(flat, holder["meta"]), traj


class NaNRecoveryTrainer:
    """Progressive-lookback rollback on NaN loss."""

    def __init__(self, trainer: MixedPrecisionTrainer, config: AutoRestartConfig,
                 checkpoint_fn: Callable[[int], None] | None = None,
                 restore_fn: Callable[[int], tuple[int, Any]] | None = None):
        self.trainer = trainer
        self.config = config
        self.checkpoint_fn = checkpoint_fn or (lambda step: None)
        self.restore_fn = restore_fn or (lambda step: (step, None))
        self._auto_restart = AutoRestart()

    def train_step_with_recovery(self, batch, step: int, rollout_steps: int = 1, prev_loss: float | None = None):
        if prev_loss is not None and math.isnan(prev_loss):
            if self._auto_restart.iteration >= self.config.max_nan_restarts:
                if self.config.error_with_nan_loss:
                    raise RuntimeError(f"NaN loss detected at step {step} after "
                                       f"{self.config.max_nan_restarts} restart attempts")
                logger.warning("NaN loss but max restarts exceeded; continuing")
            else:
                self._auto_restart = AutoRestart(self._auto_restart.iteration + 1,
                                                 self._auto_restart.began_at or step)
                lookback = self._auto_restart.iteration * self.config.restart_lookback_steps
                restored, _ = self.restore_fn(max(0, step - 1 - lookback))
                return {"total": float("nan"), "restored_to": restored}, True
        res = self.trainer.train_step(batch, rollout_steps=rollout_steps)
        if self._auto_restart.iteration > 0:
            max_lb = self.config.max_nan_restarts * self.config.restart_lookback_steps
            if self._auto_restart.began_at is not None and step - max_lb > self._auto_restart.began_at:
                self._auto_restart = AutoRestart()
        return res, False


class MultiStageTrainer:
    def __init__(self, trainer: MixedPrecisionTrainer, stages: Sequence[TrainStage]):
        self.trainer = trainer
        self.stages = list(stages)
        self.current_stage_idx = 0
        self._stage_step = 0

    @property
    def current_stage(self) -> TrainStage:
        return self.stages[self.current_stage_idx]

    @property
    def is_complete(self) -> bool:
        return self.current_stage_idx >= len(self.stages)

    def advance(self):
        self._stage_step = 0
        self.current_stage_idx += 1

    def train_step(self, batch):
        if self.is_complete:
            raise RuntimeError("All training stages complete")
        st = self.current_stage
        orig = None
        if st.loss_fn is not None:
            orig, self.trainer.loss_fn = self.trainer.loss_fn, st.loss_fn
        if st.learning_rate is not None:
            for pg in self.trainer.optimizer.param_groups:
                pg["lr"] = st.learning_rate
        res = self.trainer.train_step(batch, rollout_steps=st.rollout_steps)
        if orig is not None:
            self.trainer.loss_fn = orig
        res["stage"] = self.current_stage_idx
        res["stage_step"] = self._stage_step
        self._stage_step += 1
        if self._stage_step >= st.duration:
            self.advance()
        return res


class _OffloadFn(torch.autograd.Function):
    """Identity whose saved activation lives in pinned host memory."""

    @staticmethod
    def forward(ctx, x):
        return x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        return g


class HostOffloadCheckpoint:
    """Activation offload to pinned host memory via saved-tensor hooks."""

    def __init__(self, max_offloaded: int = 16, pin_memory: bool = True):
        self.max_offloaded = max_offloaded
        self.pin_memory = pin_memory
        self._offloaded: list = []

    def _pack(self, t: torch.Tensor):
        if not t.is_cuda or t.numel() < 1024:
            return t
        host = torch.empty(t.shape, dtype=t.dtype, device="cpu", pin_memory=self.pin_memory)
        host.copy_(t, non_blocking=True)
        self._offloaded.append(host)
        return (t.device, host)

    @staticmethod
    def _unpack(p):
        if isinstance(p, tuple):
            dev, host = p
            return host.to(dev, non_blocking=True)
        return p

    def rollout(self, step_fn: Callable, initial_state, total_steps: int, segment_length: int = 4):
        """``(final state, trajectory)`` of ``total_steps`` calls of ``step_fn``.

        The tensors that autograd saves during the first steps go to pinned host memory
        and come back when backward reaches them; the last ``segment_length`` steps, which
        backward needs first, keep theirs on the device.  At most ``max_offloaded`` steps
        are offloaded (the following ones stay on the device)."""
        self._offloaded.clear()
        n_off = min(max(total_steps - segment_length, 0), self.max_offloaded)
        traj, state = [], initial_state
        for i in range(total_steps):
            if i < n_off:
                with torch.autograd.graph.saved_tensors_hooks(self._pack, self._unpack):
                    state = step_fn(state)
            else:
                state = step_fn(state)
            traj.append(state)
        return state, traj

    def clear(self):
        self._offloaded.clear()
