"""SDA-driven training — reference ``training/sda_trainer.py:27-245``.

:class:`SDATrainer` runs :class:`~tornado_gcm_b200.training.trainer.GCMTrainer`
(whole optimizer step in one CUDA graph on the GPU) on a hybrid model while
the SDA controller's scheduler moves through the precision phases: each
decision can change the rollout length (the graph is re-captured for the new
shape) and the precision policy (transform precision and TF32 switches).
Data come from a batch iterator; by default the synthetic reanalysis
generator of the model's grid.
"""

from __future__ import annotations

import logging
import pathlib
from typing import Callable, Iterator, Optional, Sequence

import torch
import torch.nn as nn

from tornado_gcm_b200.precision.sda import SDAConfig, SDAController
from tornado_gcm_b200.training.trainer import GCMTrainer

logger = logging.getLogger(__name__)


class SDATrainer:
    def __init__(self, model: nn.Module, sda_config: Optional[SDAConfig] = None, total_steps: Optional[int] = None,
                 batch_size: Optional[int] = None, data=None, graph: Optional[bool] = None,
                 data_parallel: bool = False, *, optimizer: Optional[torch.optim.Optimizer] = None,
                 loss_fn: Optional[Callable] = None, max_grad_norm: Optional[float] = None,
                 ema_num_steps: Optional[int] = None):
        """The reference's keywords are accepted: ``optimizer`` supplies the AdamW
        hyperparameters (learning rate, weight decay, betas, eps of its first parameter
        group; the step itself runs on the fused AdamW of the captured training step),
        ``loss_fn(predictions=..., targets=...)`` replaces the per-field MSE of the model,
        ``max_grad_norm`` / ``ema_num_steps`` override the configuration."""
        self.sda_config = sda_config or SDAConfig()
        tr = self.sda_config.training
        if optimizer is not None:
            g = optimizer.param_groups[0]
            tr.learning_rate = float(g.get("lr", tr.learning_rate))
            tr.weight_decay = float(g.get("weight_decay", tr.weight_decay))
            self._betas = tuple(g.get("betas", (0.9, 0.95)))
            self._eps = float(g.get("eps", 1e-6))
        else:
            self._betas, self._eps = (0.9, 0.95), 1e-6
        if max_grad_norm is not None:
            tr.max_grad_norm = float(max_grad_norm)
        if ema_num_steps is not None:
            tr.ema_num_steps = int(ema_num_steps)
        if loss_fn is not None:
            model.loss_fn = loss_fn
        self.total_steps = int(total_steps if total_steps is not None else tr.total_steps)
        self.batch_size = int(batch_size if batch_size is not None else tr.batch_size)
        self.gcm = model
        self.controller = SDAController(self.sda_config)
        self.controller.scheduler.total_steps = self.total_steps
        self.controller.apply()
        dev = next(model.parameters()).device
        self.device = dev
        self._graph = (dev.type == "cuda") if graph is None else graph
        self._data_parallel = data_parallel
        self._trainer = self._make_trainer()
        self._rollout_steps = int(tr.rollout_steps)
        self._data = data
        self.history: list[dict] = []
        self._backward_hooks: list = []

    def _make_trainer(self) -> GCMTrainer:
        tr = self.sda_config.training
        return GCMTrainer(self.gcm, lr=tr.learning_rate, weight_decay=tr.weight_decay, max_grad_norm=tr.max_grad_norm,
                          ema_num_steps=tr.ema_num_steps, graph=self._graph, data_parallel=self._data_parallel,
                          betas=self._betas, eps=self._eps)

    # ── properties of the reference API ──
    @property
    def model(self) -> nn.Module:
        return self.gcm

    @property
    def policy(self):
        return self.controller.policy

    @property
    def step_count(self) -> int:
        return self._trainer.step_count

    @property
    def rollout_steps(self) -> int:
        return self._rollout_steps

    # ── data ──
    def _batches(self) -> Iterator:
        if self._data is not None:
            return iter(self._data)
        return self._synthetic_batches()

    def _synthetic_batches(self) -> Iterator:
        from tornado_gcm_b200.training.synthetic import SyntheticReanalysis

        from tornado_gcm_b200.parallel.ddp import get_rank

        grid = self.gcm.model.config.coords.horizontal
        src = SyntheticReanalysis(grid, seed=get_rank())  # every rank draws its own samples
        enc = self.gcm.encoder
        norm = lambda d: {k: (v.to(self.device) - getattr(enc, f"mean_{k}")) / getattr(enc, f"std_{k}")
                          for k, v in d.items()}
        forc = {k: v.to(self.device) for k, v in src.forcings(self.batch_size).items()}
        step = 0
        while True:
            x0 = norm(src.sample(self.batch_size, step))
            tg = [norm(src.sample(self.batch_size, step + 1 + i)) for i in range(self._rollout_steps)]
            yield x0, tg, forc
            step += 1

    # ── stepping ──
    def _apply_decision(self, decision) -> None:
        if decision is None:
            return
        if getattr(decision, "rollout_changed", False) and decision.new_rollout:
            logger.info("SDA: rollout %d → %d (%s)", self._rollout_steps, decision.new_rollout, decision.reason)
            self._rollout_steps = int(decision.new_rollout)
            self._trainer.release_graph()
        if getattr(decision, "policy_changed", False) and decision.new_policy is not None:
            decision.new_policy.apply_tf32_setting()
            prec = getattr(decision.new_policy, "z1_sht_precision", None)
            if prec and hasattr(self.gcm.model, "set_transform_precision"):
                self.gcm.model.set_transform_precision(prec)
                self._trainer.release_graph()

    def train_step(self, batch=None, rollout_steps: Optional[int] = None) -> dict:
        """One step; ``rollout_steps`` overrides the scheduler's rollout length for this step."""
        if batch is None:
            batch = next(self._it) if hasattr(self, "_it") else next(self._new_iter())
        x0, targets, forcings = batch
        targets = list(targets)[: (self._rollout_steps if rollout_steps is None else int(rollout_steps))]
        loss = self._trainer.train_step(x0, targets, forcings)
        interval = max(int(self.sda_config.scheduler.check_interval), 1)
        if (self.step_count % interval) == 0:  # one host read per scheduler check, not per step
            self.controller.profiler.record_loss(float(loss))
        decision = self.controller.step()
        self._apply_decision(decision)
        return {"loss": loss, "rollout_steps": self._rollout_steps}

    def _new_iter(self):
        self._it = self._batches()
        return self._it

    def fit(self, num_steps: Optional[int] = None, log_every: int = 100,
            callback: Optional[Callable[[int, dict], None]] = None, *, data_iter=None,
            total_steps: Optional[int] = None, callbacks: Optional[Sequence[Callable]] = None,
            log_interval: Optional[int] = None) -> list[dict]:
        """Train ``num_steps`` (the reference: ``total_steps``) steps on the configured data or on
        ``data_iter``; ``callback`` / every entry of ``callbacks`` is called as ``fn(step, out)``."""
        n = self.total_steps if (num_steps is None and total_steps is None) else int(
            num_steps if num_steps is not None else total_steps)
        log_every = log_interval if log_interval is not None else log_every
        fns = ([callback] if callback is not None else []) + list(callbacks or [])
        if data_iter is not None:
            self._it = it = iter(data_iter)
        else:
            it = self._new_iter()
        for i in range(n):
            out = self.train_step(next(it))
            if (i + 1) % max(log_every, 1) == 0 or i == n - 1:
                rec = {"step": self.step_count, "loss": float(out["loss"]), "rollout_steps": out["rollout_steps"]}
                self.history.append(rec)
                logger.info("step %d loss %.5g rollout %d", rec["step"], rec["loss"], rec["rollout_steps"])
            for fn in fns:
                fn(i, out)
        return self.history

    train = fit

    def swap_policy(self, phase) -> None:
        """Adopt a training-phase preset (rollout length, network dtype, TF32)."""
        self._rollout_steps = int(phase.rollout_steps)
        torch.backends.cuda.matmul.allow_tf32 = bool(phase.dycore_tf32)
        self._trainer.release_graph()

    def get_ema_state_dict(self) -> dict:
        return self._trainer.ema.state_dict()

    # ── per-layer backward precision (reference ``training/sda_trainer.py:184-226``) ──
    def configure_backward_precision(self, final_layer_keywords: Sequence[str] = ("output_layer", "head", "final"),
                                     high_precision_dtype: torch.dtype = torch.float32) -> None:
        """Hand the gradients that the final network layers pass back to their inputs over in
        ``high_precision_dtype``: a full backward hook on every module whose name contains one of
        the keywords.  Autograd delivers each gradient in its input's dtype, so the widening
        reaches inputs held in that dtype (fp32 activations or master copies); BF16 inputs keep
        BF16 gradients.  A captured training step picks the hooks up at its next capture."""
        self.remove_backward_hooks()
        words = tuple(k.lower() for k in final_layer_keywords)

        def widen(module, grad_input, grad_output):
            return tuple(g.to(high_precision_dtype) if isinstance(g, torch.Tensor) and g.is_floating_point() else g
                         for g in grad_input)

        for name, module in self.gcm.named_modules():
            if name and any(w in name.lower() for w in words):
                self._backward_hooks.append(module.register_full_backward_hook(widen))
        if self._backward_hooks:
            self._trainer.release_graph()

    def remove_backward_hooks(self) -> None:
        """Remove the hooks of :meth:`configure_backward_precision`."""
        for h in self._backward_hooks:
            h.remove()
        if self._backward_hooks:
            self._trainer.release_graph()
        self._backward_hooks.clear()

    # ── checkpoints ──
    def save_checkpoint(self, path) -> None:
        """One checkpoint file (written by rank 0).  With the sharded optimizer the moments are
        gathered into the replicated AdamW layout first, a collective every rank takes part in."""
        from tornado_gcm_b200.parallel.ddp import get_rank
        from tornado_gcm_b200.training.checkpointing import _atomic_save

        zo = self._trainer.zero_opt
        opt_sd = zo.full_state_dict() if zo is not None else self._trainer.optimizer.state_dict()
        if get_rank() != 0:
            return
        _atomic_save({"model_state_dict": self.gcm.state_dict(), "optimizer_state_dict": opt_sd,
                      "ema": self.get_ema_state_dict(), "step": self.step_count,
                      "rollout_steps": self._rollout_steps}, pathlib.Path(path))

    def load_checkpoint(self, path) -> None:
        ck = torch.load(path, map_location=self.device, weights_only=False)
        self.gcm.load_state_dict(ck["model_state_dict"])
        self._trainer.release_graph()
        if self._trainer.zero_opt is not None:
            self._trainer.zero_opt.load_full_state_dict(ck["optimizer_state_dict"])
        else:
            self._trainer.optimizer.load_state_dict(ck["optimizer_state_dict"])
        for name, shadow in zip(self._trainer.ema.names, self._trainer.ema.shadow):
            if name in ck.get("ema", {}):
                shadow.copy_(ck["ema"][name])
        self._trainer.step_count = int(ck.get("step", 0))
        self._rollout_steps = int(ck.get("rollout_steps", self._rollout_steps))
