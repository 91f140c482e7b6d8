"""Training objectives — reference ``training/losses.py:24-741``.

Same classes and formulas (trajectory MSE/MAE, CRPS with cyclic-shift
spread, aggregation state, batched per-variable loss, conservation and
hydrological constraints, spectral MSE with lead-time wavenumber masking,
transformed L2 with legacy time rescaling, spectral-norm matching, batch
mean bias, the combined NeuralGCM loss).  Accumulators start on the
predictions' device so no term forces a host synchronisation.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from tornado_gcm_b200.core.primitive_equations import State
from tornado_gcm_b200.precision.zone_cast import f64_math


def _zero_like(x) -> torch.Tensor:
    if isinstance(x, State):
        x = x.vorticity
    if isinstance(x, dict):
        x = next(iter(x.values()))
    return torch.zeros((), dtype=torch.float32, device=x.device)


def _state_fields(state) -> dict:
    if isinstance(state, State):
        d = {"vorticity": state.vorticity, "divergence": state.divergence,
             "temperature_variation": state.temperature_variation,
             "log_surface_pressure": state.log_surface_pressure}
        for k, v in state.tracers.items():
            d[f"tracer_{k}"] = v
        return d
    if isinstance(state, dict):
        return state
    raise TypeError(f"Cannot extract modal fields from {type(state)}")


_state_to_modal_dict = _state_fields


def _safe_sqrt(x: torch.Tensor) -> torch.Tensor:
    return torch.sqrt(torch.clamp(x, min=1e-30))


def _spectral_norm(x: torch.Tensor) -> torch.Tensor:
    """sqrt(Σ_m |x_{m,l}|²), shape (..., 1, L)."""
    return _safe_sqrt((x * x).sum(dim=-2, keepdim=True))


class TrajectoryMSE(nn.Module):
    def _state_mse(self, p: State, t: State) -> torch.Tensor:
        return (((p.vorticity - t.vorticity) ** 2).mean() + ((p.divergence - t.divergence) ** 2).mean()
                + ((p.temperature_variation - t.temperature_variation) ** 2).mean()
                + ((p.log_surface_pressure - t.log_surface_pressure) ** 2).mean())

    def forward(self, predictions: list, targets: list, **_) -> torch.Tensor:
        total = _zero_like(predictions[0])
        for p, t in zip(predictions, targets):
            if isinstance(p, State):
                total = total + self._state_mse(p, t)
            elif isinstance(p, dict):
                total = total + sum(((p[k] - t[k]) ** 2).mean() for k in p if k in t)
            else:
                total = total + ((p - t) ** 2).mean()
        return total / len(predictions)


class TrajectoryMAE(nn.Module):
    def forward(self, predictions: list, targets: list, **_) -> torch.Tensor:
        total = _zero_like(predictions[0])
        for p, t in zip(predictions, targets):
            if isinstance(p, State):
                total = total + sum((a - b).abs().mean() for a, b in
                                    zip(p.tensors()[:4], t.tensors()[:4]))
            elif isinstance(p, dict):
                total = total + sum((p[k] - t[k]).abs().mean() for k in p if k in t)
            else:
                total = total + (p - t).abs().mean()
        return total / len(predictions)


class CRPSLoss(nn.Module):
    """Ensemble CRPS: E|X−Y| − w·E|X−X'| (X' = cyclic shift of the ensemble axis 0)."""

    def __init__(self, spread_term_weight: float = 0.5, variable_weights: Optional[dict] = None):
        super().__init__()
        self.spread_term_weight = spread_term_weight
        self.variable_weights = variable_weights or {}

    def _crps_tensor(self, ens: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
        skill = (ens - target.unsqueeze(0)).abs().mean(dim=0)
        spread = (ens - ens.roll(shifts=1, dims=0)).abs().mean(dim=0)
        return (skill - self.spread_term_weight * spread).mean()

    def forward(self, predictions: list, targets: list, **_) -> torch.Tensor:
        total = _zero_like(predictions[0])
        for p, t in zip(predictions, targets):
            if isinstance(p, dict) and isinstance(t, dict):
                for k in p:
                    total = total + self.variable_weights.get(k, 1.0) * self._crps_tensor(p[k], t[k])
            else:
                total = total + self._crps_tensor(p, t)
        return total / max(len(predictions), 1)


class AggregationState:
    """Σ(statistic·weight) and Σ(weight) per key, mergeable across batches."""

    def __init__(self):
        self.sum_weighted: dict = {}
        self.sum_weights: dict = {}

    def update(self, values: dict, weights: Optional[dict] = None) -> None:
        for k, v in values.items():
            w = weights[k] if weights is not None and k in weights else torch.ones_like(v)
            if k in self.sum_weighted:
                self.sum_weighted[k] = self.sum_weighted[k] + v * w
                self.sum_weights[k] = self.sum_weights[k] + w
            else:
                self.sum_weighted[k] = v * w
                self.sum_weights[k] = w.clone()

    def mean(self) -> dict:
        return {k: self.sum_weighted[k] / self.sum_weights[k].clamp(min=1e-12) for k in self.sum_weighted}

    def __add__(self, other: "AggregationState") -> "AggregationState":
        m = AggregationState()
        for k in set(self.sum_weighted) | set(other.sum_weighted):
            if k in self.sum_weighted and k in other.sum_weighted:
                m.sum_weighted[k] = self.sum_weighted[k] + other.sum_weighted[k]
                m.sum_weights[k] = self.sum_weights[k] + other.sum_weights[k]
            else:
                src = self if k in self.sum_weighted else other
                m.sum_weighted[k] = src.sum_weighted[k].clone()
                m.sum_weights[k] = src.sum_weights[k].clone()
        return m


class BatchedParameterLoss(nn.Module):
    def __init__(self, variable_weights: Optional[dict] = None, loss_type: str = "mse"):
        super().__init__()
        self.variable_weights = variable_weights or {}
        self.loss_type = loss_type

    def _compute_one(self, p, t):
        return (p - t).abs().mean() if self.loss_type == "mae" else ((p - t) ** 2).mean()

    def forward(self, predictions: dict, targets: dict, agg_state: Optional[AggregationState] = None):
        agg_state = agg_state or AggregationState()
        values = {}
        total = _zero_like(predictions)
        for k in predictions:
            if k not in targets:
                continue
            v = self._compute_one(predictions[k], targets[k])
            values[k] = v
            total = total + self.variable_weights.get(k, 1.0) * v
        agg_state.update(values)
        return total, agg_state


class SumLoss(nn.Module):
    def __init__(self, terms: dict, term_weights: Optional[dict] = None):
        super().__init__()
        self.terms = nn.ModuleDict(terms)
        self.term_weights = term_weights or {}

    def forward(self, **kwargs) -> dict:
        out = {}
        total = None
        for name, fn in self.terms.items():
            v = fn(**kwargs)
            if isinstance(v, dict):
                v = v.get("total", sum(v.values()))
            out[name] = v
            total = self.term_weights.get(name, 1.0) * v if total is None else total + self.term_weights.get(name, 1.0) * v
        out["total"] = total
        return out


class EnergyConservationLoss(nn.Module):
    @f64_math
    def forward(self, energies: torch.Tensor) -> torch.Tensor:
        e0 = energies[0].abs().clamp(min=1e-12)
        return (((energies[1:] - energies[:-1]).abs() / e0) ** 2).mean()


class MassConservationLoss(nn.Module):
    @f64_math
    def forward(self, masses: torch.Tensor) -> torch.Tensor:
        m0 = masses[0].abs().clamp(min=1e-12)
        return (((masses[1:] - masses[0]).abs() / m0) ** 2).mean()


class HydrologicalClosureLoss(nn.Module):
    def forward(self, precipitation: torch.Tensor, evaporation: torch.Tensor) -> torch.Tensor:
        return (torch.clamp(-precipitation, min=0.0) ** 2 + torch.clamp(evaporation, min=0.0) ** 2).mean()


class PhysicsConstrainedLoss(nn.Module):
    """Prediction loss + λ_E energy + λ_M mass + λ_H hydrology (after warmup)."""

    def __init__(self, prediction_loss: Optional[nn.Module] = None, lambda_e: float = 1e-3, lambda_m: float = 1e-3,
                 lambda_h: float = 1e-3, warmup_steps: int = 1000):
        super().__init__()
        self.prediction_loss = prediction_loss or TrajectoryMSE()
        self.lambda_e, self.lambda_m, self.lambda_h = lambda_e, lambda_m, lambda_h
        self.warmup_steps = warmup_steps
        self.energy_loss = EnergyConservationLoss()
        self.mass_loss = MassConservationLoss()
        self.hydro_loss = HydrologicalClosureLoss()

    def forward(self, predictions: list, targets: list, energies=None, masses=None, precipitation=None,
                evaporation=None, step: int = 0) -> dict:
        pred = self.prediction_loss(predictions, targets)
        zero = torch.zeros_like(pred)
        on = step >= self.warmup_steps
        le = self.energy_loss(energies).to(pred.dtype) if on and energies is not None else zero
        lm = self.mass_loss(masses).to(pred.dtype) if on and masses is not None else zero
        lh = self.hydro_loss(precipitation, evaporation).to(pred.dtype) \
            if on and precipitation is not None and evaporation is not None else zero
        total = pred + self.lambda_e * le + self.lambda_m * lm + self.lambda_h * lh
        return {"total": total, "prediction": pred, "energy": le, "mass": lm, "hydro": lh}


class SpectralMSELoss(nn.Module):
    """Modal MSE with sigmoid mask w(l, k) = σ((L·max(0, 1−αk) − l)/τ)."""

    def __init__(self, total_wavenumbers: int, alpha: float = 0.05, tau: float = 2.0,
                 variable_weights: Optional[dict] = None):
        super().__init__()
        self.L, self.alpha, self.tau = total_wavenumbers, alpha, tau
        self.variable_weights = variable_weights or {}

    def _wavenumber_mask(self, k: int, device) -> torch.Tensor:
        l = torch.arange(self.L, dtype=torch.float32, device=device)
        return torch.sigmoid((self.L * max(0.0, 1.0 - self.alpha * k) - l) / self.tau).unsqueeze(0)

    def forward(self, predictions: list, targets: list, **_) -> torch.Tensor:
        total = _zero_like(predictions[0])
        for k, (p, t) in enumerate(zip(predictions, targets)):
            pd, td = _state_fields(p), _state_fields(t)
            mask = self._wavenumber_mask(k, total.device)
            for key in pd:
                if key in td:
                    total = total + self.variable_weights.get(key, 1.0) * (((pd[key] - td[key]) ** 2) * mask).mean()
        return total / max(len(predictions), 1)


class TransformedL2Loss(nn.Module):
    """L2 with legacy time rescaling scale² = 1/((n−1)·steps_per_save) for n > 1."""

    def __init__(self, steps_per_save: int = 1, variable_weights: Optional[dict] = None):
        super().__init__()
        self.steps_per_save = steps_per_save
        self.variable_weights = variable_weights or {}

    def forward(self, predictions: list, targets: list, **_) -> torch.Tensor:
        n = len(predictions)
        s2 = 1.0 if n <= 1 else 1.0 / ((n - 1) * self.steps_per_save)
        total = _zero_like(predictions[0])
        for p, t in zip(predictions, targets):
            pd, td = _state_fields(p), _state_fields(t)
            for key in pd:
                if key in td:
                    total = total + s2 * self.variable_weights.get(key, 1.0) * ((pd[key] - td[key]) ** 2).mean()
        return total / max(n, 1)


class SpectralNormMatchingLoss(nn.Module):
    def __init__(self, variable_weights: Optional[dict] = None):
        super().__init__()
        self.variable_weights = variable_weights or {}

    def forward(self, predictions: list, targets: list, **_) -> torch.Tensor:
        total = _zero_like(predictions[0])
        for p, t in zip(predictions, targets):
            pd, td = _state_fields(p), _state_fields(t)
            for key in pd:
                if key in td:
                    total = total + self.variable_weights.get(key, 1.0) * (
                        (_spectral_norm(pd[key]) - _spectral_norm(td[key])) ** 2).mean()
        return total / max(len(predictions), 1)


class BatchMeanBiasLoss(nn.Module):
    def __init__(self, variable_weights: Optional[dict] = None):
        super().__init__()
        self.variable_weights = variable_weights or {}

    def forward(self, predictions: list, targets: list, **_) -> torch.Tensor:
        ps: dict = {}
        ts: dict = {}
        n = len(predictions)
        for p, t in zip(predictions, targets):
            pd, td = _state_fields(p), _state_fields(t)
            for key in pd:
                if key in td:
                    ps[key] = ps.get(key, 0) + pd[key].abs()
                    ts[key] = ts.get(key, 0) + td[key].abs()
        total = _zero_like(predictions[0])
        for key in ps:
            total = total + self.variable_weights.get(key, 1.0) * ((ps[key] / n - ts[key] / n) ** 2).mean()
        return total


class NeuralGCMLoss(nn.Module):
    """λ_l2·TransformedL2 + λ_spec·spectrum + λ_bias·bias + λ_E·E + λ_M·M + λ_H·H."""

    def __init__(self, steps_per_save: int = 1, lambda_l2: float = 1.0, lambda_spec: float = 1.0,
                 lambda_bias: float = 1.0, lambda_e: float = 1e-3, lambda_m: float = 1e-3, lambda_h: float = 1e-3,
                 warmup_steps: int = 1000):
        super().__init__()
        self.lambda_l2, self.lambda_spec, self.lambda_bias = lambda_l2, lambda_spec, lambda_bias
        self.lambda_e, self.lambda_m, self.lambda_h = lambda_e, lambda_m, lambda_h
        self.warmup_steps = warmup_steps
        self.transformed_l2 = TransformedL2Loss(steps_per_save=steps_per_save)
        self.spectrum_match = SpectralNormMatchingLoss()
        self.bias_loss = BatchMeanBiasLoss()
        self.energy_loss = EnergyConservationLoss()
        self.mass_loss = MassConservationLoss()
        self.hydro_loss = HydrologicalClosureLoss()

    def forward(self, predictions: list, targets: list, energies=None, masses=None, precipitation=None,
                evaporation=None, step: int = 0) -> dict:
        l2 = self.transformed_l2(predictions, targets)
        spec = self.spectrum_match(predictions, targets)
        bias = self.bias_loss(predictions, targets)
        zero = torch.zeros_like(l2)
        on = step >= self.warmup_steps
        le = self.energy_loss(energies).to(l2.dtype) if on and energies is not None else zero
        lm = self.mass_loss(masses).to(l2.dtype) if on and masses is not None else zero
        lh = self.hydro_loss(precipitation, evaporation).to(l2.dtype) \
            if on and precipitation is not None and evaporation is not None else zero
        total = (self.lambda_l2 * l2 + self.lambda_spec * spec + self.lambda_bias * bias + self.lambda_e * le
                 + self.lambda_m * lm + self.lambda_h * lh)
        return {"total": total, "transformed_l2": l2, "spectrum_match": spec, "bias": bias, "energy": le,
                "mass": lm, "hydro": lh}
