"""Forecast evaluation — reference ``training/evaluation.py:68-1012``.

* Forecast start sampling: :func:`get_forecast_starts_equispaced` (00z/12z
  alternation) and :func:`get_forecast_starts_balanced` (even spread over
  the hours of day).
* Metrics per variable and lead time: RMSE, anomaly correlation, bias.
  They are computed on the device for all variables and lead times of a
  forecast and copied to the host ONCE per forecast (the reference performs a
  blocking ``.item()`` per variable per lead time).  An optional per-latitude
  area weight (``cos φ`` on a nodal grid) gives the WeatherBench convention.
* :class:`EvaluationRunner`: in-training evaluation on equispaced samples
  at a cadence, optionally with EMA weights swapped in (and restored).
* :class:`WeatherBenchmarkRunner`: day-3 / day-5 / day-10 headline metrics.

States may be :class:`~tornado_gcm_b200.core.primitive_equations.State`
objects or dicts of tensors; ``step_fn(model, state, forcing)`` defaults to
``model.step(state, forcings=forcing)``.
"""

from __future__ import annotations

import dataclasses
import logging
import time
from typing import Any, Callable, Optional, Sequence

import numpy as np
import torch
import torch.nn as nn

logger = logging.getLogger(__name__)

LEAD_HOURS_DAY3 = 72
LEAD_HOURS_DAY5 = 120
LEAD_HOURS_DAY10 = 240
WB2_HEADLINE_VARS = ["geopotential_500", "temperature_850", "temperature_500", "specific_humidity_700"]
ACC_USEFUL_THRESHOLD = 0.6
ACC_MARGINAL_THRESHOLD = 0.5


# ───────────────────────── start times ─────────────────────────


def get_forecast_starts_equispaced(sample_count: int, first_start, last_start,
                                   alternate_0z_12z: bool = True) -> np.ndarray:
    """``sample_count`` starts spread evenly over ``[first_start, last_start + 1 day)``,
    rounded down to midnight, odd-numbered starts moved to 12z."""
    if sample_count <= 0:
        return np.array([], dtype="datetime64[ns]")
    start = np.datetime64(first_start, "ns")
    stop = np.datetime64(np.datetime64(last_start, "D") + np.timedelta64(1, "D"), "ns")
    span = (stop - start).astype(np.int64)
    offs = np.linspace(0, span, sample_count + 1)[:-1].astype(np.int64).astype("timedelta64[ns]")
    t = (start + offs).astype("datetime64[D]").astype("datetime64[ns]")
    if alternate_0z_12z:
        t = t + (np.arange(sample_count) % 2) * np.timedelta64(12, "h").astype("timedelta64[ns]")
    return t


def get_forecast_starts_balanced(sample_count: int, candidates: np.ndarray,
                                 balance_diurnal_cycle: bool = True) -> np.ndarray:
    """Pick ``sample_count`` of ``candidates``, equally many per time of day, evenly within each."""
    if sample_count <= 0:
        return np.array([], dtype="datetime64[ns]")
    c = np.asarray(candidates).astype("datetime64[ns]")
    if not balance_diurnal_cycle:
        return c[np.linspace(0, len(c) - 1, sample_count).astype(int)]
    tod = c - c.astype("datetime64[D]").astype("datetime64[ns]")
    groups = np.unique(tod)
    if len(groups) == 0:
        raise ValueError("No candidates available.")
    out = []
    for i, g in enumerate(groups):
        n = sample_count // len(groups) + (1 if i < sample_count % len(groups) else 0)
        if n == 0:
            continue
        members = c[tod == g]
        if n > len(members):
            raise ValueError(f"time of day {g} has {len(members)} candidates, {n} needed")
        out.append(members[np.clip(np.round(np.arange(n) * len(members) / n).astype(int), 0, len(members) - 1)])
    return np.sort(np.concatenate(out))


# ───────────────────────── metrics ─────────────────────────


def _state_to_tensor_dict(state) -> dict:
    from tornado_gcm_b200.core.primitive_equations import State

    if isinstance(state, State):
        d = {"vorticity": state.vorticity, "divergence": state.divergence,
             "temperature_variation": state.temperature_variation,
             "log_surface_pressure": state.log_surface_pressure}
        d.update({f"tracer_{k}": v for k, v in state.tracers.items()})
        return d
    if isinstance(state, dict):
        return {k: v for k, v in state.items() if torch.is_tensor(v)}
    if torch.is_tensor(state):
        return {"field": state}
    raise TypeError(f"Unsupported state type: {type(state)}")


def _weights(t: torch.Tensor, lat_weights: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    if lat_weights is None or t.shape[-1] != lat_weights.shape[-1]:
        return None
    w = lat_weights.to(t.device, torch.float64)
    return w / w.mean()


def _mean(x: torch.Tensor, w: Optional[torch.Tensor]) -> torch.Tensor:
    return x.mean() if w is None else (x * w).mean() / 1.0


def _metric_table(predictions: list, targets: list, kind: str, variable_names=None, climatology=None,
                  lat_weights=None) -> dict:
    K = min(len(predictions), len(targets))
    names, vals = [], []
    for k in range(K):
        p_d, t_d = _state_to_tensor_dict(predictions[k]), _state_to_tensor_dict(targets[k])
        for name, p in p_d.items():
            if (variable_names and name not in variable_names) or name not in t_d:
                continue
            t = t_d[name]
            if torch.is_complex(p):
                if kind == "acc":
                    continue
                d = p - t
                v = (d * d.conj()).real.double().mean().sqrt() if kind == "rmse" else d.abs().double().mean()
            else:
                p64, t64 = p.detach().double(), t.detach().double()
                w = _weights(p64, lat_weights)
                if kind == "rmse":
                    v = _mean((p64 - t64) ** 2, w).clamp_min(0).sqrt()
                elif kind == "bias":
                    v = _mean(p64 - t64, w)
                else:
                    clim = climatology[name].to(p64) if climatology and name in climatology else t64.mean()
                    pa, ta = p64 - clim, t64 - clim
                    ww = torch.ones_like(pa) if w is None else w.expand_as(pa)
                    den = torch.sqrt((ww * pa * pa).sum() * (ww * ta * ta).sum())
                    v = torch.where(den > 0, (ww * pa * ta).sum() / den.clamp_min(1e-300), torch.zeros_like(den))
                    v = v.clamp(-1.0, 1.0)
            names.append(name)
            vals.append(v.reshape(()))
    out: dict = {}
    if vals:
        host = torch.stack([v.to(vals[0].device) for v in vals]).cpu().tolist()  # one copy for the table
        for n, v in zip(names, host):
            out.setdefault(n, []).append(float(v))
    return out


@torch.no_grad()
def compute_rmse(predictions: list, targets: list, variable_names: Optional[Sequence[str]] = None,
                 lat_weights: Optional[torch.Tensor] = None) -> dict:
    return _metric_table(predictions, targets, "rmse", variable_names, lat_weights=lat_weights)


@torch.no_grad()
def compute_anomaly_correlation(predictions: list, targets: list, climatology: Optional[dict] = None,
                                variable_names: Optional[Sequence[str]] = None,
                                lat_weights: Optional[torch.Tensor] = None) -> dict:
    """ACC of anomalies from ``climatology`` (the target mean when absent)."""
    return _metric_table(predictions, targets, "acc", variable_names, climatology, lat_weights)


@torch.no_grad()
def compute_bias(predictions: list, targets: list, variable_names: Optional[Sequence[str]] = None,
                 lat_weights: Optional[torch.Tensor] = None) -> dict:
    return _metric_table(predictions, targets, "bias", variable_names, lat_weights=lat_weights)


@dataclasses.dataclass
class EvalResult:
    rmse: dict = dataclasses.field(default_factory=dict)
    acc: dict = dataclasses.field(default_factory=dict)
    bias: dict = dataclasses.field(default_factory=dict)
    eval_loss: float = 0.0
    n_samples: int = 0
    elapsed_seconds: float = 0.0

    def summary(self, variables: Optional[Sequence[str]] = None) -> dict:
        out = {}
        if self.eval_loss > 0:
            out["eval_loss"] = self.eval_loss
        for metric, table in (("rmse", self.rmse), ("acc", self.acc), ("bias", self.bias)):
            for var, values in table.items():
                if variables and var not in variables:
                    continue
                for t, v in enumerate(values):
                    out[f"{metric}/{var}/t+{t + 1}"] = v
                if values:
                    out[f"{metric}/{var}/mean"] = sum(values) / len(values)
        out["n_samples"] = float(self.n_samples)
        out["eval_seconds"] = self.elapsed_seconds
        return out

    def log_summary(self, step: int, prefix: str = "eval", variables: Optional[Sequence[str]] = None,
                    max_lead_times: int = 4) -> None:
        parts = [f"step={step}"] + ([f"loss={self.eval_loss:.6f}"] if self.eval_loss > 0 else [])
        for metric, table in (("rmse", self.rmse), ("acc", self.acc)):
            for var, values in table.items():
                if not variables or var in variables:
                    parts.append(f"{metric}/{var}=[{', '.join(f'{v:.4f}' for v in values[:max_lead_times])}]")
        logger.info("[%s] %s", prefix, " | ".join(parts))


@dataclasses.dataclass
class EvalConfig:
    eval_cadence: int = 1000
    n_eval_samples: int = 20
    rollout_steps: Optional[int] = None
    compute_acc: bool = True
    variable_names: Optional[Sequence[str]] = None


def _to(obj, device):
    if torch.is_tensor(obj):
        return obj.to(device, non_blocking=True)
    if isinstance(obj, dict):
        return {k: _to(v, device) for k, v in obj.items()}
    if hasattr(obj, "tree_map"):
        return obj.tree_map(lambda t: t.to(device, non_blocking=True))
    return obj


def _model_device(model: nn.Module) -> torch.device:
    for p in model.parameters():
        return p.device
    for b in model.buffers():
        return b.device
    return torch.device("cpu")


class EvaluationRunner:
    """Periodic autoregressive evaluation (reference ``training/evaluation.py:451-800``)."""

    def __init__(self, model: nn.Module, config: Optional[EvalConfig] = None, loss_fn: Optional[Callable] = None,
                 ema_params: Optional[dict] = None, climatology: Optional[dict] = None,
                 step_fn: Optional[Callable] = None, lat_weights: Optional[torch.Tensor] = None):
        self.model = model
        self.config = config or EvalConfig()
        self.loss_fn = loss_fn
        self.ema_params = ema_params
        self.climatology = climatology
        self.step_fn = step_fn or (lambda m, s, f: m.step(s, forcings=f))
        self.lat_weights = lat_weights
        self._eval_samples: list = []

    def set_eval_data(self, states: list, forcings=None, rollout_steps: Optional[int] = None) -> None:
        """``n_eval_samples`` equispaced ``(initial, targets, forcings)`` windows of a state sequence;
        ``forcings`` is a per-step list or ``{name: array (time, …)}``."""
        K = rollout_steps or self.config.rollout_steps or 16
        total = len(states) - K
        if total <= 0:
            logger.warning("need at least %d states for K=%d, got %d", K + 1, K, len(states))
            self._eval_samples = []
            return
        dev = _model_device(self.model)
        idx = list(range(total)) if self.config.n_eval_samples >= total else \
            np.linspace(0, total - 1, self.config.n_eval_samples).astype(int).tolist()
        table = forcings is not None and isinstance(forcings, dict)
        self._eval_samples = []
        for i in idx:
            frc = None
            if forcings is not None:
                if table:
                    frc = [{k: torch.as_tensor(np.asarray(a)[min(t, len(a) - 1)], dtype=torch.float32, device=dev)
                            for k, a in forcings.items()} for t in range(i + 1, i + 1 + K)]
                else:
                    frc = [_to(f, dev) for f in forcings[i + 1:i + 1 + K]]
            self._eval_samples.append((_to(states[i], dev), [_to(s, dev) for s in states[i + 1:i + 1 + K]], frc))

    def set_eval_data_from_dataloader(self, dataloader, n_samples: Optional[int] = None,
                                      rollout_steps: Optional[int] = None, device=None) -> None:
        """Batches of ``{name: (batch, time, …)}``; keys ``forcing_<name>`` are forcings."""
        n = n_samples or self.config.n_eval_samples
        K = rollout_steps or self.config.rollout_steps or 16
        dev = device or _model_device(self.model)
        self._eval_samples = []
        for i, batch in enumerate(dataloader):
            if i >= n:
                break
            fields = {k: v[0] for k, v in batch.items() if torch.is_tensor(v) and v.dim() >= 2
                      and not k.startswith("forcing_") and k != "weight"}
            forc = {k[len("forcing_"):]: v[0] for k, v in batch.items() if k.startswith("forcing_")}
            T = min(v.shape[0] for v in fields.values())
            k_eff = min(K, T - 1)
            init = {k: v[0].to(dev) for k, v in fields.items()}
            targets = [{k: v[t].to(dev) for k, v in fields.items()} for t in range(1, 1 + k_eff)]
            frc = [{k: v[t].to(dev) for k, v in forc.items()} for t in range(1, 1 + k_eff)] if forc else None
            self._eval_samples.append((init, targets, frc))

    def should_evaluate(self, step: int) -> bool:
        return bool(self._eval_samples) and (step + 1) % self.config.eval_cadence == 0

    def maybe_evaluate(self, step: int, rollout_steps: Optional[int] = None, use_ema: bool = False):
        return self.evaluate(rollout_steps, use_ema) if self.should_evaluate(step) else None

    @torch.no_grad()
    def evaluate(self, rollout_steps: Optional[int] = None, use_ema: bool = False) -> EvalResult:
        t0 = time.time()
        was_training = self.model.training
        self.model.eval()
        saved = None
        if use_ema and self.ema_params:
            saved = {}
            for n, p in self.model.named_parameters():
                if n in self.ema_params:
                    saved[n] = p.data.clone()
                    p.data.copy_(self.ema_params[n])
        tables = {"rmse": {}, "acc": {}, "bias": {}}
        loss_sum, n_loss = 0.0, 0
        try:
            for init, targets, forc in self._eval_samples:
                K = min(rollout_steps or len(targets), len(targets))
                preds, s = [], init
                for i in range(K):
                    s = self.step_fn(self.model, s, forc[i] if forc is not None and i < len(forc) else None)
                    preds.append(s)
                kinds = ("rmse", "acc", "bias") if self.config.compute_acc else ("rmse", "bias")
                for kind in kinds:
                    t = _metric_table(preds, targets[:K], kind, self.config.variable_names, self.climatology,
                                      self.lat_weights)
                    for var, vals in t.items():
                        tables[kind].setdefault(var, []).append(vals)
                if self.loss_fn is not None:
                    out = self.loss_fn(predictions=preds, targets=targets[:K], step=0)
                    loss_sum += float(out["total"] if isinstance(out, dict) else out)
                    n_loss += 1
        finally:
            if saved is not None:
                for n, p in self.model.named_parameters():
                    if n in saved:
                        p.data.copy_(saved[n])
            self.model.train(was_training)

        def agg(tab):
            res = {}
            for var, runs in tab.items():
                L = max(len(r) for r in runs)
                res[var] = [float(np.mean([r[t] for r in runs if t < len(r)])) for t in range(L)]
            return res

        return EvalResult(agg(tables["rmse"]), agg(tables["acc"]), agg(tables["bias"]), loss_sum / max(n_loss, 1),
                          len(self._eval_samples), time.time() - t0)

    def update_ema_params(self, ema_params: dict) -> None:
        self.ema_params = ema_params


# ───────────────────────── headline benchmark ─────────────────────────


@dataclasses.dataclass
class WeatherBenchmarkResult:
    day3_rmse: dict = dataclasses.field(default_factory=dict)
    day5_rmse: dict = dataclasses.field(default_factory=dict)
    day10_rmse: dict = dataclasses.field(default_factory=dict)
    day3_acc: dict = dataclasses.field(default_factory=dict)
    day5_acc: dict = dataclasses.field(default_factory=dict)
    rmse_by_lead: dict = dataclasses.field(default_factory=dict)
    acc_by_lead: dict = dataclasses.field(default_factory=dict)
    n_samples: int = 0
    dt_hours: float = 6.0

    def headline_summary(self) -> dict:
        out = {}
        for prefix, table in (("day3_rmse", self.day3_rmse), ("day5_rmse", self.day5_rmse),
                              ("day3_acc", self.day3_acc), ("day5_acc", self.day5_acc)):
            out.update({f"{prefix}/{k}": v for k, v in table.items()})
        out["n_samples"] = float(self.n_samples)
        return out

    def log_headline(self, step: int, prefix: str = "benchmark") -> None:
        parts = [f"step={step}"]
        parts += [f"{v}: Day3={self.day3_rmse.get(v, float('nan')):.2f} Day5={self.day5_rmse.get(v, float('nan')):.2f}"
                  for v in sorted(self.day3_rmse)]
        parts += [f"ACC/{v}: Day3={self.day3_acc.get(v, float('nan')):.4f} "
                  f"Day5={self.day5_acc.get(v, float('nan')):.4f}" for v in sorted(self.day3_acc)]
        logger.info("[%s] %s", prefix, " | ".join(parts))


def _lead_time_index(target_hours: float, dt_hours: float) -> Optional[int]:
    i = round(target_hours / dt_hours) - 1
    return i if i >= 0 else None


def extract_day_metrics(eval_result: EvalResult, dt_hours: float = 6.0) -> WeatherBenchmarkResult:
    res = WeatherBenchmarkResult(rmse_by_lead=dict(eval_result.rmse), acc_by_lead=dict(eval_result.acc),
                                 n_samples=eval_result.n_samples, dt_hours=dt_hours)
    slots = ((LEAD_HOURS_DAY3, res.day3_rmse, res.day3_acc), (LEAD_HOURS_DAY5, res.day5_rmse, res.day5_acc),
             (LEAD_HOURS_DAY10, res.day10_rmse, None))
    for hours, rmse_out, acc_out in slots:
        i = _lead_time_index(hours, dt_hours)
        if i is None:
            continue
        rmse_out.update({v: vals[i] for v, vals in eval_result.rmse.items() if i < len(vals)})
        if acc_out is not None:
            acc_out.update({v: vals[i] for v, vals in eval_result.acc.items() if i < len(vals)})
    return res


@dataclasses.dataclass
class WeatherBenchmarkConfig:
    eval_cadence: int = 5000
    n_eval_samples: int = 50
    forecast_hours: float = 360.0
    dt_hours: float = 6.0
    compute_acc: bool = True
    headline_vars: Optional[Sequence[str]] = None


class WeatherBenchmarkRunner:
    def __init__(self, model: nn.Module, config: Optional[WeatherBenchmarkConfig] = None, loss_fn=None,
                 ema_params: Optional[dict] = None, climatology: Optional[dict] = None, step_fn=None,
                 lat_weights: Optional[torch.Tensor] = None):
        self.config = config or WeatherBenchmarkConfig()
        self._eval_runner = EvaluationRunner(
            model, EvalConfig(self.config.eval_cadence, self.config.n_eval_samples,
                              int(self.config.forecast_hours / self.config.dt_hours), self.config.compute_acc,
                              self.config.headline_vars), loss_fn, ema_params, climatology, step_fn, lat_weights)

    def set_eval_data(self, states: list, forcings=None) -> None:
        self._eval_runner.set_eval_data(states, forcings)

    def set_eval_data_from_dataloader(self, dataloader, n_samples: Optional[int] = None, device=None) -> None:
        self._eval_runner.set_eval_data_from_dataloader(dataloader, n_samples=n_samples, device=device)

    def should_evaluate(self, step: int) -> bool:
        return self._eval_runner.should_evaluate(step)

    def maybe_evaluate(self, step: int, use_ema: bool = True):
        return self.evaluate(use_ema) if self.should_evaluate(step) else None

    def evaluate(self, use_ema: bool = True) -> WeatherBenchmarkResult:
        return extract_day_metrics(self._eval_runner.evaluate(use_ema=use_ema), self.config.dt_hours)

    def update_ema_params(self, ema_params: dict) -> None:
        self._eval_runner.update_ema_params(ema_params)
