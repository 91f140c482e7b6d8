"""Automatic precision-zone discovery (HPS level 2) — reference ``precision/zone_discovery.py:45-753``.

Input: a :class:`~tornado_gcm_b200.precision.sensitivity.SensitivityMap`.
Output: a partition of the profiled modules into zones, each with a
recommended dtype from its sensitivity centroid (``> 0.1`` FP64, ``> 1e-3``
FP32, else BF16).

1. Affinity ``A_ij = exp(-(s_i - s_j)² / 2σ²) + α·[i ~ j in the module graph]``
   where ``s = log10(drift)`` (drifts span many decades; a linear distance
   would merge everything below the largest drift — the reference uses the raw
   drift) and ``σ`` is the median pairwise distance unless given.
2. Normalised Laplacian ``I - D^-½ A D^-½``; eigengap heuristic picks
   ``K = argmax_{2≤k≤K_max} (λ_k - λ_{k-1})``.
3. Spectral clustering: k-means (deterministic farthest-point seeding) on
   the row-normalised first ``K`` eigenvectors.
4. Cast cost = number of graph edges that cross zone boundaries.

Also: :func:`compare_with_pzha`, :func:`detect_monotonicity_violations`
(promoting one zone's precision must not raise the drift) and
:func:`lattice_prune` (if a configuration violates the bound, every
configuration below it in every zone does too).
"""

from __future__ import annotations

import dataclasses
import logging
import math
from typing import Optional

import numpy as np
import torch

from tornado_gcm_b200.precision.policy import PrecisionPolicy
from tornado_gcm_b200.precision.sensitivity import SensitivityMap

logger = logging.getLogger(__name__)

_PRECISIONS = ((0.1, torch.float64, "FP64"), (1e-3, torch.float32, "FP32"), (-math.inf, torch.bfloat16, "BF16"))
PRECISION_ORDER = ["torch.bfloat16", "torch.float32", "torch.float64"]


def _recommend_precision(centroid: float) -> tuple:
    for thr, dt, name in _PRECISIONS:
        if not math.isfinite(centroid) or centroid > thr:
            return dt, name
    return torch.bfloat16, "BF16"


@dataclasses.dataclass
class ModuleGraph:
    """Data-flow graph over profiled module names."""

    nodes: list
    edges: list

    @classmethod
    def from_execution_order(cls, module_names: list) -> "ModuleGraph":
        names = list(module_names)
        return cls(names, list(zip(names[:-1], names[1:])))

    @classmethod
    def for_neuralgcm(cls) -> "ModuleGraph":
        """One physics step: parameterization (Z3) → dycore (Z1) → filters (Z0) → fixer (Z2),
        and the fixer also reads the pre-dycore state."""
        nodes = ["parameterization", "dycore", "filters", "conservation_fixer"]
        edges = [("parameterization", "dycore"), ("dycore", "filters"), ("filters", "conservation_fixer"),
                 ("dycore", "conservation_fixer")]
        return cls(nodes, edges)


@dataclasses.dataclass
class ZoneAssignment:
    zone_id: int
    members: list
    sensitivity_centroid: float
    recommended_precision: str
    recommended_dtype: torch.dtype = torch.float32


@dataclasses.dataclass
class DiscoveryResult:
    zones: list
    k: int = 0
    eigengaps: list = dataclasses.field(default_factory=list)
    module_zone_map: dict = dataclasses.field(default_factory=dict)
    estimated_cast_cost: float = 0.0

    def to_policy(self, base_policy: Optional[PrecisionPolicy] = None) -> PrecisionPolicy:
        """Map zones back onto Z1 / Z2 / Z3 compute dtypes by member name."""
        base = base_policy or PrecisionPolicy()
        dt = {m: z.recommended_dtype for z in self.zones for m in z.members}

        def pick(names, default):
            for n in names:
                if n in dt:
                    return dt[n]
            return default

        return dataclasses.replace(
            base, z0_dtype=torch.float64,
            z1_compute_dtype=pick(("dycore", "_dycore_equation", "zone:Z1_dynamics"), base.z1_compute_dtype),
            z2_compute_dtype=pick(("conservation_fixer", "zone:Z2_fixer"), base.z2_compute_dtype),
            z3_compute_dtype=pick(("parameterization", "zone:Z3_neural"), base.z3_compute_dtype))

    def summary_str(self) -> str:
        lines = [f"DiscoveryResult: K={self.k} zones", f"Eigengaps: {[f'{g:.4f}' for g in self.eigengaps[:8]]}", ""]
        for z in sorted(self.zones, key=lambda z: z.sensitivity_centroid, reverse=True):
            lines.append(f"  Zone {z.zone_id}: {z.recommended_precision} (centroid={z.sensitivity_centroid:.6e})"
                         f"  members=[{', '.join(z.members)}]")
        return "\n".join(lines)


def _kmeans(V: np.ndarray, k: int, iters: int = 50) -> np.ndarray:
    n = V.shape[0]
    centers = [V[int(np.argmax(np.linalg.norm(V - V.mean(0), axis=1)))]]
    while len(centers) < k:  # farthest-point seeding: deterministic
        d = np.min(np.stack([np.linalg.norm(V - c, axis=1) for c in centers]), axis=0)
        centers.append(V[int(np.argmax(d))])
    C = np.stack(centers)
    labels = np.zeros(n, dtype=np.int64)
    for _ in range(iters):
        new = np.argmin(np.linalg.norm(V[:, None, :] - C[None], axis=2), axis=1)
        if np.array_equal(new, labels) and _ > 0:
            break
        labels = new
        for c in range(k):
            if np.any(labels == c):
                C[c] = V[labels == c].mean(0)
    return labels


class ZoneDiscovery:
    def __init__(self, sensitivity_map: SensitivityMap, module_graph: Optional[ModuleGraph] = None,
                 alpha: float = 0.3, sigma: Optional[float] = None, log_scale: bool = True):
        self.smap = sensitivity_map
        self.graph = module_graph
        self.alpha = alpha
        self.sigma = sigma
        self.log_scale = log_scale
        self._names, self._sensitivities = [], []
        for name, ms in sensitivity_map.modules.items():
            if ms.n_children_profiled > 0:  # refined parents are represented by their children
                continue
            self._names.append(name)
            self._sensitivities.append(float(ms.drift))

    @property
    def n_modules(self) -> int:
        return len(self._names)

    def _coords(self) -> np.ndarray:
        s = np.asarray(self._sensitivities, dtype=np.float64)
        s = np.where(np.isfinite(s), s, np.nanmax(np.where(np.isfinite(s), s, np.nan)) * 10 if np.any(
            np.isfinite(s)) else 1.0)
        return np.log10(np.maximum(s, 1e-30)) if self.log_scale else s

    def _build_affinity_matrix(self) -> np.ndarray:
        s = self._coords()
        d2 = (s[:, None] - s[None, :]) ** 2
        sigma = self.sigma
        if sigma is None:
            iu = np.triu_indices(len(s), 1)
            sigma = max(float(np.sqrt(np.median(d2[iu]) + 1e-30)), 1e-10) if len(iu[0]) else 1.0
        A = np.exp(-d2 / (2 * sigma ** 2))
        if self.graph is not None:
            idx = {n: i for i, n in enumerate(self._names)}
            for a, b in self.graph.edges:
                if a in idx and b in idx:
                    A[idx[a], idx[b]] += self.alpha
                    A[idx[b], idx[a]] += self.alpha
        np.fill_diagonal(A, 0.0)
        return A

    @staticmethod
    def _normalized_laplacian(A: np.ndarray) -> np.ndarray:
        d = A.sum(1)
        inv = 1.0 / np.sqrt(d + 1e-30)
        return np.eye(len(A)) - inv[:, None] * A * inv[None, :]

    def _compute_eigengaps(self, A: np.ndarray) -> tuple:
        ev = np.sort(np.linalg.eigvalsh(self._normalized_laplacian(A)))
        return ev, np.diff(ev)

    def _select_k(self, gaps: np.ndarray, max_zones: int) -> int:
        upper = min(max_zones, self.n_modules, len(gaps))
        if upper < 2:
            return max(1, min(2, self.n_modules))
        return int(np.argmax(gaps[1:upper])) + 2

    def _spectral_cluster(self, A: np.ndarray, k: int) -> np.ndarray:
        n = A.shape[0]
        if k >= n:
            return np.arange(n)
        _, vecs = np.linalg.eigh(self._normalized_laplacian(A))
        V = vecs[:, :k]
        V = V / (np.linalg.norm(V, axis=1, keepdims=True) + 1e-30)
        return _kmeans(V, k)

    def _estimate_cast_cost(self, labels: np.ndarray, A: Optional[np.ndarray] = None) -> float:
        if self.graph is None:
            return 0.0
        idx = {n: i for i, n in enumerate(self._names)}
        return float(sum(1 for a, b in self.graph.edges if a in idx and b in idx and labels[idx[a]] != labels[idx[b]]))

    def discover(self, max_zones: int = 8, force_k: Optional[int] = None) -> DiscoveryResult:
        n = self.n_modules
        if n == 0:
            return DiscoveryResult([], 0)
        if n <= 2:
            return self._trivial_assignment()
        A = self._build_affinity_matrix()
        _, gaps = self._compute_eigengaps(A)
        k = min(force_k, n) if force_k is not None else self._select_k(gaps, max_zones)
        labels = self._spectral_cluster(A, k)
        zones, zmap = [], {}
        for z in range(int(labels.max()) + 1):
            idx = [i for i in range(n) if labels[i] == z]
            if not idx:
                continue
            vals = [self._sensitivities[i] for i in idx]
            fin = [v for v in vals if math.isfinite(v)]
            centroid = float(np.mean(fin)) if len(fin) == len(vals) else float("inf")
            dt, name = _recommend_precision(centroid)
            zones.append(ZoneAssignment(len(zones), [self._names[i] for i in idx], centroid, name, dt))
            for i in idx:
                zmap[self._names[i]] = zones[-1].zone_id
        relabeled = np.array([zmap[nm] for nm in self._names])
        return DiscoveryResult(zones, len(zones), gaps.tolist(), zmap, self._estimate_cast_cost(relabeled, A))

    def _trivial_assignment(self) -> DiscoveryResult:
        zones, zmap = [], {}
        for i, (nm, s) in enumerate(zip(self._names, self._sensitivities)):
            dt, name = _recommend_precision(s)
            zones.append(ZoneAssignment(i, [nm], s, name, dt))
            zmap[nm] = i
        return DiscoveryResult(zones, len(zones), module_zone_map=zmap)


_PZHA = {"parameterization": ("Z3 (Neural)", "BF16"), "dycore": ("Z1 (Dynamics)", "FP32"),
         "_dycore_equation": ("Z1 (Dynamics)", "FP32"), "filters": ("Z0 (Basis)", "FP64"),
         "exp_filter": ("Z0 (Basis)", "FP64"), "conservation_fixer": ("Z2 (Fixer)", "FP64"),
         "zone:Z1_dynamics": ("Z1 (Dynamics)", "FP32"), "zone:Z2_fixer": ("Z2 (Fixer)", "FP64"),
         "zone:Z3_neural": ("Z3 (Neural)", "BF16")}


def compare_with_pzha(result: DiscoveryResult, sensitivity_map: SensitivityMap) -> str:
    """Table of discovered zones against the hand-designed PZHA zones, with the agreement rate."""
    lines = ["Comparison: HPS Auto-Discovery vs Manual PZHA", "=" * 50]
    by_id = {z.zone_id: z for z in result.zones}
    agree = total = 0
    for name in sorted(result.module_zone_map):
        z = by_id[result.module_zone_map[name]]
        pz, expected = _PZHA.get(name, ("N/A", None))
        ms = sensitivity_map.modules.get(name)
        lines.append(f"  {name:30s}  PZHA={pz:15s}  HPS=Zone{z.zone_id}({z.recommended_precision:4s})  "
                     f"drift={ms.drift:.6e}" if ms else f"  {name:30s}  PZHA={pz:15s}  HPS=Zone{z.zone_id}")
        if expected is not None:
            total += 1
            agree += int(z.recommended_precision == expected)
    if total:
        lines.append(f"\nAgreement with PZHA: {agree}/{total} ({100 * agree / total:.0f}%)")
    return "\n".join(lines)


def detect_monotonicity_violations(pareto_results: list, precision_order: Optional[list] = None,
                                   tolerance: float = 1.05) -> list:
    """Pairs that differ by promoting ONE zone yet whose drift grew by more than ``tolerance``×."""
    rank = {p: i for i, p in enumerate(precision_order or PRECISION_ORDER)}
    out = []
    for i, lo in enumerate(pareto_results):
        for hi in pareto_results[i + 1:]:
            a, b = lo["zone_dtypes"], hi["zone_dtypes"]
            if len(a) != len(b):
                continue
            ups = [z for z in range(len(a)) if rank.get(b[z], -1) > rank.get(a[z], -1)]
            downs = [z for z in range(len(a)) if rank.get(b[z], -1) < rank.get(a[z], -1)]
            if len(ups) == 1 and not downs and hi["drift"] > lo["drift"] * tolerance:
                out.append({"config_low": lo.get("config_id", i), "config_high": hi.get("config_id"),
                            "drift_low": lo["drift"], "drift_high": hi["drift"], "zone_changed": ups[0],
                            "ratio": hi["drift"] / max(lo["drift"], 1e-30)})
    if out:
        logger.warning("%d monotonicity violations (higher precision → higher drift)", len(out))
    return out


def lattice_prune(configs: list, drift_cache: dict, threshold: float, precision_order: Optional[list] = None) -> list:
    """Drop configurations dominated (≤ in every zone) by a measured infeasible one."""
    rank = {p: i for i, p in enumerate(precision_order or PRECISION_ORDER)}

    def dominates(a, b):
        return all(rank.get(x, 0) >= rank.get(y, 0) for x, y in zip(a, b))

    bad = [c for c, d in drift_cache.items() if d > threshold]
    kept = []
    for cfg in configs:
        if cfg in drift_cache:
            if drift_cache[cfg] <= threshold:
                kept.append(cfg)
        elif not any(dominates(b, cfg) for b in bad):
            kept.append(cfg)
    return kept
