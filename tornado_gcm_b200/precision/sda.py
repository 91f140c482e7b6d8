"""SDA precision control plane: configs, SDAConfig (YAML), controller
(reference ``precision/sda.py:35-497``).

Differences by design: the YAML ``model`` / ``training`` / ``data`` /
``fixer`` sections are parsed into :class:`ModelSection` etc. (the
reference reads only policy/profiler/scheduler/accelerator/storage/sparse);
the accelerator section selects between this framework's sm_100a kernels
(``backend='sm100'``, default) and plain torch (``'eager'``).
"""

from __future__ import annotations

import dataclasses
import logging
import time
from dataclasses import field
from typing import Any, Optional

import torch

from tornado_gcm_b200.precision.policy import PrecisionPolicy, PrecisionZone

logger = logging.getLogger(__name__)

_DTYPES = {"float16": torch.float16, "float32": torch.float32, "float64": torch.float64,
           "bfloat16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32, "fp64": torch.float64,
           "bf16": torch.bfloat16}
_DTYPE_NAMES = {torch.float16: "float16", torch.float32: "float32", torch.float64: "float64",
                torch.bfloat16: "bfloat16"}


def _filter_fields(cls, d: dict) -> dict:
    names = {f.name for f in dataclasses.fields(cls)}
    unknown = set(d) - names
    if unknown:
        logger.warning("%s: ignoring unknown keys %s", cls.__name__, sorted(unknown))
    return {k: (_DTYPES.get(v, v) if isinstance(v, str) else v) for k, v in d.items() if k in names}


@dataclasses.dataclass
class ProfilerConfig:
    enabled: bool = True
    granularity: str = "zone"
    sample_rate: int = 10
    performance_counters: bool = False
    numerical_audit: bool = True
    gradient_audit: bool = True
    spectral_audit: bool = False
    export_format: str = "tensorboard"


@dataclasses.dataclass
class SchedulerConfig:
    mode: str = "milestone"
    check_interval: int = 100
    loss_plateau_threshold: float = 0.01
    loss_plateau_patience: int = 3
    nan_trigger_count: int = 2
    grad_var_threshold: float = 100.0
    spectral_tail_threshold: float = 0.1
    warmup_steps_after_switch: int = 5
    rollout_ramp_steps: int = 0
    total_steps: int = 100_000


@dataclasses.dataclass
class AcceleratorConfig:
    backend: str = "sm100"
    enable_fused_zone_cast: bool = False
    enable_triton_sht: bool = False
    enable_triton_fixers: bool = False
    compile_mode: str = "reduce-overhead"
    compile_dynamic: bool = False
    cuda_graphs: bool = True


@dataclasses.dataclass
class StorageConfig:
    mode: str = "mixed"
    exact_dtype: torch.dtype = torch.float32
    lossy_dtype: torch.dtype = torch.bfloat16
    critical_variables: list = field(default_factory=lambda: ["vorticity", "divergence", "log_surface_pressure"])
    non_critical_variables: list = field(default_factory=lambda: ["tracers"])
    compressor: str = "zstd"
    compression_level: int = 3


@dataclasses.dataclass
class SparseConfig:
    enabled: bool = False
    mode: str = "structural"
    adaptive_threshold: float = 1e-6
    high_order_cutoff: float = 0.5
    high_order_dtype: torch.dtype = torch.bfloat16
    low_order_dtype: torch.dtype = torch.float32


@dataclasses.dataclass
class ModelSection:
    resolution: str = "2.8deg"
    grid: Optional[str] = None
    layers: int = 32
    dt_minutes: Optional[float] = None
    tower_width: Optional[int] = None
    checkpoint_path: Optional[str] = None
    extra: dict = field(default_factory=dict)


@dataclasses.dataclass
class TrainingSection:
    total_steps: int = 1000
    batch_size: int = 4
    learning_rate: float = 1e-4
    weight_decay: float = 0.0
    rollout_steps: int = 4
    max_grad_norm: float = 1.0
    ema_num_steps: int = 1999
    checkpoint_dir: str = "checkpoints"
    checkpoint_every: int = 500
    extra: dict = field(default_factory=dict)


@dataclasses.dataclass
class DataSection:
    source: str = "synthetic"
    path: Optional[str] = None
    variables: list = field(default_factory=list)
    extra: dict = field(default_factory=dict)


@dataclasses.dataclass
class FixerSection:
    kind: str = "lite"  # "lite" | "f64" | "none"
    cadence: int = 1
    fix_mass: bool = True
    fix_energy: bool = True
    # "levels": each level's T'(0,0) takes deficit / n (restores the energy proxy exactly);
    # "reference": the whole deficit at every level, as reference neural/fixers.py:171-190
    energy_split: str = "levels"


def _section(cls, d: Optional[dict]):
    d = dict(d or {})
    names = {f.name for f in dataclasses.fields(cls)}
    extra = {k: v for k, v in d.items() if k not in names}
    kw = {k: v for k, v in d.items() if k in names}
    obj = cls(**kw)
    if extra and "extra" in names:
        obj.extra.update(extra)
    return obj


@dataclasses.dataclass
class SDAConfig:
    policy: PrecisionPolicy = field(default_factory=PrecisionPolicy)
    profiler: ProfilerConfig = field(default_factory=ProfilerConfig)
    scheduler: SchedulerConfig = field(default_factory=SchedulerConfig)
    accelerator: AcceleratorConfig = field(default_factory=AcceleratorConfig)
    storage: StorageConfig = field(default_factory=StorageConfig)
    sparse: SparseConfig = field(default_factory=SparseConfig)
    model: ModelSection = field(default_factory=ModelSection)
    training: TrainingSection = field(default_factory=TrainingSection)
    data: DataSection = field(default_factory=DataSection)
    fixer: FixerSection = field(default_factory=FixerSection)

    @classmethod
    def from_dict(cls, d: dict) -> "SDAConfig":
        d = dict(d or {})
        pol = _filter_fields(PrecisionPolicy, dict(d.get("policy") or {}))
        return cls(
            policy=PrecisionPolicy(**pol) if pol else PrecisionPolicy(),
            profiler=ProfilerConfig(**_filter_fields(ProfilerConfig, dict(d.get("profiler") or {}))),
            scheduler=SchedulerConfig(**_filter_fields(SchedulerConfig, dict(d.get("scheduler") or {}))),
            accelerator=AcceleratorConfig(**_filter_fields(AcceleratorConfig, dict(d.get("accelerator") or {}))),
            storage=StorageConfig(**_filter_fields(StorageConfig, dict(d.get("storage") or {}))),
            sparse=SparseConfig(**_filter_fields(SparseConfig, dict(d.get("sparse") or {}))),
            model=_section(ModelSection, d.get("model")),
            training=_section(TrainingSection, d.get("training")),
            data=_section(DataSection, d.get("data")),
            fixer=_section(FixerSection, d.get("fixer")),
        )

    @classmethod
    def from_yaml(cls, path: str) -> "SDAConfig":
        import yaml

        with open(path, "r", encoding="utf-8") as fh:
            return cls.from_dict(yaml.safe_load(fh) or {})

    def to_dict(self) -> dict:
        def conv(obj):
            if dataclasses.is_dataclass(obj) and not isinstance(obj, type):
                return {f.name: conv(getattr(obj, f.name)) for f in dataclasses.fields(obj)}
            if isinstance(obj, torch.dtype):
                return _DTYPE_NAMES.get(obj, str(obj))
            if isinstance(obj, (list, tuple)):
                return [conv(x) for x in obj]
            if isinstance(obj, dict):
                return {k: conv(v) for k, v in obj.items()}
            return obj
        return conv(self)

    def to_yaml(self, path: str) -> None:
        import yaml

        with open(path, "w", encoding="utf-8") as fh:
            yaml.safe_dump(self.to_dict(), fh, sort_keys=False)


@dataclasses.dataclass(frozen=True)
class CompiledPolicy:
    z0_compute: torch.dtype
    z0_storage: torch.dtype
    z1_compute: torch.dtype
    z1_storage: torch.dtype
    z2_compute: torch.dtype
    z2_storage: torch.dtype
    z3_compute: torch.dtype
    z3_storage: torch.dtype
    tf32_enabled: bool

    def compute_dtype(self, zone: PrecisionZone) -> torch.dtype:
        return {PrecisionZone.Z0_NUMERICAL_FOUNDATION: self.z0_compute, PrecisionZone.Z1_DYNAMICS_CORE: self.z1_compute,
                PrecisionZone.Z2_CONSERVATION_FIXER: self.z2_compute,
                PrecisionZone.Z3_NEURAL_NETWORK: self.z3_compute}[zone]

    def storage_dtype(self, zone: PrecisionZone) -> torch.dtype:
        return {PrecisionZone.Z0_NUMERICAL_FOUNDATION: self.z0_storage, PrecisionZone.Z1_DYNAMICS_CORE: self.z1_storage,
                PrecisionZone.Z2_CONSERVATION_FIXER: self.z2_storage,
                PrecisionZone.Z3_NEURAL_NETWORK: self.z3_storage}[zone]


@dataclasses.dataclass
class SDAReport:
    total_steps: int = 0
    phase_transitions: list = field(default_factory=list)
    final_policy: Optional[PrecisionPolicy] = None
    profiler_summary: dict = field(default_factory=dict)
    scheduler_decisions: int = 0
    warnings: list = field(default_factory=list)
    wall_time_seconds: float = 0.0


class SDAController:
    """Profiler → scheduler → policy hot-swap loop; call ``apply()`` then ``step()``."""

    def __init__(self, config: SDAConfig) -> None:
        from tornado_gcm_b200.precision.profiler import SDAProfiler
        from tornado_gcm_b200.precision.scheduler import PrecisionScheduler

        self.config = config
        self._policy = config.policy
        self._compiled: Optional[CompiledPolicy] = None
        self._step_count = 0
        self._start_time = 0.0
        self._phase_transitions: list = []
        self._decision_count = 0
        self.profiler = SDAProfiler(config.profiler)
        self.scheduler = PrecisionScheduler(config.scheduler, config.policy, config.scheduler.total_steps)
        self._accelerator = None
        self._storage = None
        self._fused_kernel = None
        self._listeners: list = []

    @property
    def policy(self) -> PrecisionPolicy:
        return self._policy

    @property
    def compiled(self) -> CompiledPolicy:
        if self._compiled is None:
            self._compiled = self.compile(self._policy)
        return self._compiled

    @property
    def storage(self):
        return self._storage

    @property
    def accelerator(self):
        return self._accelerator

    def add_listener(self, fn) -> None:
        """Callback ``fn(new_policy)`` invoked after every hot-swap (e.g. model.set_precision_policy)."""
        self._listeners.append(fn)

    def apply(self) -> None:
        self._compiled = self.compile(self._policy)
        self._policy.apply_tf32_setting()
        if self.config.accelerator.backend != "eager":
            from tornado_gcm_b200.precision.accelerator import AcceleratorRegistry

            self._accelerator = AcceleratorRegistry(default_backend=self.config.accelerator.backend)
        from tornado_gcm_b200.precision.storage import SDAStorageManager

        self._storage = SDAStorageManager(self.config.storage)
        self._start_time = time.monotonic()
        logger.info("SDA applied: Z0=%s Z1=%s(tf32=%s) Z2=%s Z3=%s", self._policy.z0_dtype,
                    self._policy.z1_compute_dtype, self._policy.z1_use_tf32, self._policy.z2_compute_dtype,
                    self._policy.z3_compute_dtype)

    def get_fused_kernel(self, model):
        if not self.config.accelerator.enable_fused_zone_cast:
            return None
        if self._fused_kernel is None:
            from tornado_gcm_b200.precision.accelerator import FusedAdvanceKernel

            self._fused_kernel = FusedAdvanceKernel(model, self._policy)
        return self._fused_kernel

    def step(self):
        """Per-step callback; returns the scheduler decision (or None)."""
        self._step_count += 1
        self.profiler.step()
        dec = self.scheduler.tick_warmup()
        if dec.rollout_changed:
            self._decision_count += 1
        if self._step_count % max(self.config.scheduler.check_interval, 1) != 0:
            return dec
        metrics = self.profiler.collect()
        decision = self.scheduler.decide(metrics, self._step_count)
        if decision.policy_changed and decision.new_policy is not None:
            self.hot_swap(decision.new_policy, reason=decision.reason)
            self._decision_count += 1
        if decision.rollout_changed:
            self._decision_count += 1
        return decision

    def hot_swap(self, new_policy: PrecisionPolicy, *, reason: str = "") -> None:
        old = f"Z1={self._policy.z1_compute_dtype}, Z3={self._policy.z3_compute_dtype}"
        self._policy = new_policy
        self._compiled = self.compile(new_policy)
        new_policy.apply_tf32_setting()
        if self._fused_kernel is not None:
            self._fused_kernel.reset()
            self._fused_kernel = None
        new = f"Z1={new_policy.z1_compute_dtype}, Z3={new_policy.z3_compute_dtype}"
        self._phase_transitions.append({"step": self._step_count, "from": old, "to": new, "reason": reason})
        for fn in self._listeners:
            fn(new_policy)
        logger.info("SDA hot-swap at step %d: %s → %s [%s]", self._step_count, old, new, reason)

    def report(self) -> SDAReport:
        el = time.monotonic() - self._start_time if self._start_time else 0.0
        return SDAReport(self._step_count, list(self._phase_transitions), self._policy, self.profiler.summary(),
                         self._decision_count, list(self.profiler.collect().warnings), el)

    @staticmethod
    def compile(policy: PrecisionPolicy) -> CompiledPolicy:
        return CompiledPolicy(policy.z0_dtype, policy.z0_dtype, policy.z1_compute_dtype, policy.z1_storage_dtype,
                              policy.z2_compute_dtype, policy.z2_storage_dtype, policy.z3_compute_dtype,
                              policy.z3_param_dtype, policy.z1_use_tf32)


DEFAULT_SDA_CONFIG = SDAConfig()
