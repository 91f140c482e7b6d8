"""SDA-controlled inference — reference ``inference/sda_runner.py:26-256``.

:class:`SDAInference` extends :class:`MPInference` with the SDA control
plane: BF16 parameter storage for inference, a profiler that audits the
spectral energy tail, adaptive precision escalation (``run_adaptive``: the
transforms switch from the TF32 kernels to FP64 contractions once the tail
energy ratio exceeds a threshold) and split-precision sparse state storage
between outer steps (``run_sparse``).
"""

from __future__ import annotations

import logging
from typing import Any, Optional

import torch

from tornado_gcm_b200.inference.runner import MPInference
from tornado_gcm_b200.precision.policy import PrecisionPolicy
from tornado_gcm_b200.precision.sda import SDAConfig, SDAController

logger = logging.getLogger(__name__)

_HIGH_PRECISION_POLICY = PrecisionPolicy(z1_compute_dtype=torch.float32, z1_use_tf32=False,
                                         z2_compute_dtype=torch.float64, z3_compute_dtype=torch.bfloat16)


class SDAInference(MPInference):
    def __init__(self, model: Any, sda_config: Optional[SDAConfig] = None, use_graph: bool = True):
        self.sda_config = sda_config or SDAConfig()
        base = self.sda_config.policy
        infer_policy = PrecisionPolicy(
            z0_dtype=base.z0_dtype, z1_compute_dtype=base.z1_compute_dtype, z1_use_tf32=base.z1_use_tf32,
            z1_storage_dtype=base.z1_storage_dtype, z2_compute_dtype=base.z2_compute_dtype,
            z2_storage_dtype=base.z2_storage_dtype, z3_compute_dtype=torch.bfloat16,
            z3_param_dtype=torch.bfloat16, z3_master_dtype=torch.bfloat16, data_load_dtype=torch.bfloat16,
            sht_adaptive_threshold=base.sht_adaptive_threshold, enable_precision_audit=base.enable_precision_audit)
        self.controller = SDAController(SDAConfig(policy=infer_policy, profiler=self.sda_config.profiler,
                                                  scheduler=self.sda_config.scheduler))
        super().__init__(model, infer_policy, monitor=self.controller.profiler, use_graph=use_graph)
        self.controller.apply()
        self.escalated = False

    @classmethod
    def from_state_dict(cls, state_dict: dict, sda_config: Optional[SDAConfig] = None,
                        device: str | torch.device = "cuda", resolution: Optional[str] = None, **kwargs):
        from tornado_gcm_b200.models.builders import build_hybrid_gcm

        cfg = sda_config or SDAConfig()
        meta = state_dict.get("meta", {}) if isinstance(state_dict, dict) else {}
        weights = state_dict.get("model", state_dict.get("model_state_dict", state_dict))
        res = resolution or meta.get("resolution") or getattr(getattr(cfg, "model", None), "resolution", None) \
            or "2.8deg"
        gcm, _ = build_hybrid_gcm(res, device)
        gcm.load_state_dict(weights, strict=False)
        return cls(gcm, cfg, **kwargs)

    @torch.no_grad()
    def run(self, initial_state: Any, outer_steps: int, inner_steps: Optional[int] = None, post_process_fn=None,
            forcings: Optional[dict] = None) -> list:
        traj = super().run(initial_state, outer_steps, inner_steps, post_process_fn=post_process_fn,
                           forcings=forcings)
        self.controller.step()
        return traj

    def escalate(self, reason: str = "") -> None:
        """Switch the dycore transforms to FP64 contractions (no CUDA-graph replay)."""
        if self.escalated:
            return
        self.model.set_transform_precision("highest")
        self.controller.hot_swap(_HIGH_PRECISION_POLICY, reason=reason)
        self.policy = self.controller.policy
        self._kernel = None
        self.use_graph = False
        self.escalated = True
        logger.warning("SDAInference: escalated transform precision (%s)", reason)

    @torch.no_grad()
    def run_adaptive(self, initial_state: Any, outer_steps: int, inner_steps: int = 1,
                     quality_threshold: float = 1e-4, forcings: Optional[dict] = None) -> list:
        traj, state = [], initial_state
        for step in range(outer_steps):
            state, out = self._unroll(state, 1, inner_steps, forcings)
            state = out[-1]
            if self.sda_config.profiler.spectral_audit and hasattr(state, "vorticity"):
                self.controller.profiler.audit_spectral_energy(state.vorticity)
                tail = float(self.controller.profiler._spectral_tail)
                if tail > quality_threshold and not self.escalated:
                    self.escalate(f"spectral_tail={tail:.4g} > {quality_threshold} at step {step}")
            traj.append(state)
        return traj

    def report(self) -> dict:
        r = self.controller.report()
        return {"total_steps": r.total_steps, "phase_transitions": r.phase_transitions,
                "profiler_summary": r.profiler_summary, "warnings": r.warnings, "escalated": self.escalated}

    @torch.no_grad()
    def run_sparse(self, initial_state: Any, outer_steps: int, inner_steps: int = 1, sparse_config=None,
                   forcings: Optional[dict] = None) -> tuple[list, dict]:
        from tornado_gcm_b200.core.primitive_equations import State
        from tornado_gcm_b200.precision.sparse import SparseConfig, SpectralSparseState

        cfg = sparse_config or SparseConfig(enabled=True, mode="mixed")
        traj, state, dense_b, sparse_b = [], initial_state, 0, 0
        for _ in range(outer_steps):
            state, out = self._unroll(state, 1, inner_steps, forcings)
            state = out[-1]
            if cfg.enabled and hasattr(state, "vorticity"):
                fields = {"vorticity": state.vorticity, "divergence": state.divergence,
                          "temperature_variation": state.temperature_variation,
                          "log_surface_pressure": state.log_surface_pressure}
                fields.update({"tracer:" + k: v for k, v in state.tracers.items()})
                sp = SpectralSparseState.from_state_dict(fields, cfg)
                dense_b += sp.dense_memory_bytes
                sparse_b += sp.memory_bytes
                d = sp.to_dense_dict()
                state = State(d["vorticity"], d["divergence"], d["temperature_variation"],
                              d["log_surface_pressure"],
                              {k[len("tracer:"):]: v for k, v in d.items() if k.startswith("tracer:")},
                              state.sim_time)
            traj.append(state)
        stats = {"sparse_mode": cfg.mode, "total_dense_bytes": dense_b, "total_sparse_bytes": sparse_b,
                 "memory_savings": 1.0 - sparse_b / dense_b if dense_b else 0.0, "outer_steps": outer_steps}
        return traj, stats
