"""PZHA precision zones and policy (reference ``precision/policy.py:24-225``).

Zones: Z0 numerical foundation (FP64 bases/matrices), Z1 dynamics core
(TF32 transforms on tcgen05 by default, FP32 storage), Z2 conservation
fixers (FP64 accumulation), Z3 neural networks (BF16 compute, FP32
master weights).

Unlike the reference, ``z1_sht_precision`` and ``sht_adaptive_threshold``
are honoured by the transforms (``Grid.precision``), and nothing relies on
a global ``torch.autocast``: each zone casts explicitly.
"""

from __future__ import annotations

import dataclasses
import enum
from typing import Optional

import torch


class PrecisionZone(enum.Enum):
    Z0_NUMERICAL_FOUNDATION = "Z0"
    Z1_DYNAMICS_CORE = "Z1"
    Z2_CONSERVATION_FIXER = "Z2"
    Z3_NEURAL_NETWORK = "Z3"


@dataclasses.dataclass
class PrecisionPolicy:
    z0_dtype: torch.dtype = torch.float64
    z1_compute_dtype: torch.dtype = torch.float32
    z1_use_tf32: bool = True
    z1_storage_dtype: torch.dtype = torch.float32
    z2_compute_dtype: torch.dtype = torch.float64
    z2_storage_dtype: torch.dtype = torch.float32
    z3_compute_dtype: torch.dtype = torch.bfloat16
    z3_param_dtype: torch.dtype = torch.bfloat16
    z3_master_dtype: torch.dtype = torch.float32
    data_load_dtype: torch.dtype = torch.float32
    sht_adaptive_threshold: int = 42
    # Transform precision for Z1 above the threshold: "tf32" | "float32" | "highest".
    # None keeps the reference rule (≤ threshold → float32/TF32, above → FP64).
    z1_sht_precision: Optional[str] = None
    enable_precision_audit: bool = True
    audit_every_n_steps: int = 100

    def compute_dtype(self, zone: PrecisionZone) -> torch.dtype:
        return getattr(self, _ZONE_FIELDS[zone][0])

    def storage_dtype(self, zone: PrecisionZone) -> torch.dtype:
        return getattr(self, _ZONE_FIELDS[zone][1])

    def sht_precision(self, total_wavenumbers: int) -> str:
        """Transform precision for a grid with ``total_wavenumbers`` (honours the threshold)."""
        if total_wavenumbers <= self.sht_adaptive_threshold:
            return "tf32" if self.z1_use_tf32 else "float32"
        if self.z1_sht_precision is not None:
            return self.z1_sht_precision
        return "highest"

    def apply_tf32_setting(self) -> None:
        torch.backends.cuda.matmul.allow_tf32 = self.z1_use_tf32
        torch.backends.cudnn.allow_tf32 = self.z1_use_tf32

    @classmethod
    def for_resolution(cls, total_wavenumber: int) -> "PrecisionPolicy":
        if total_wavenumber <= 127:
            return cls(z1_compute_dtype=torch.float32, z1_use_tf32=True)
        return cls(z1_compute_dtype=torch.float32, z1_use_tf32=False)

    @classmethod
    def for_training_phase(cls, phase: int, base: Optional["PrecisionPolicy"] = None) -> "PrecisionPolicy":
        """Phase 1 aggressive (FP32 fixer), 2 standard PZHA, 3 FP32 network fine-tune."""
        if phase not in _PHASE_OVERRIDES:
            raise ValueError(f"Unknown training phase: {phase}")
        return dataclasses.replace(base or cls(), **_PHASE_OVERRIDES[phase])

    @classmethod
    def pzha_b200(cls) -> "PrecisionPolicy":
        """Z1 TF32 transforms on tensor cores at every resolution, Z3 BF16, Z2 FP64."""
        return cls(z1_sht_precision="tf32", sht_adaptive_threshold=0)


class PolicyEngine:
    """Policy holder with hot-swap and a module→zone heuristic."""

    def __init__(self, policy: PrecisionPolicy | None = None):
        self._policy = policy or PrecisionPolicy()

    @property
    def policy(self) -> PrecisionPolicy:
        return self._policy

    def hot_swap(self, new_policy: PrecisionPolicy) -> None:
        self._policy = new_policy
        new_policy.apply_tf32_setting()

    def get_zone_dtype_map(self):
        return {z: (self._policy.compute_dtype(z), self._policy.storage_dtype(z)) for z in PrecisionZone}

    def get_module_zone_map(self, model: torch.nn.Module) -> dict:
        """Zone of every named submodule: the first rule of ``_MODULE_ZONE_RULES`` whose
        keyword occurs in the lower-cased name, else the dynamics core (Z1)."""
        def zone_of(name: str) -> PrecisionZone:
            low = name.lower()
            for zone, words in _MODULE_ZONE_RULES:
                if any(w in low for w in words):
                    return zone
            return PrecisionZone.Z1_DYNAMICS_CORE

        return {name: zone_of(name) for name, _ in model.named_modules()}


# (compute field, storage field) of each zone
_ZONE_FIELDS = {
    PrecisionZone.Z0_NUMERICAL_FOUNDATION: ("z0_dtype", "z0_dtype"),
    PrecisionZone.Z1_DYNAMICS_CORE: ("z1_compute_dtype", "z1_storage_dtype"),
    PrecisionZone.Z2_CONSERVATION_FIXER: ("z2_compute_dtype", "z2_storage_dtype"),
    PrecisionZone.Z3_NEURAL_NETWORK: ("z3_compute_dtype", "z3_param_dtype"),
}

# the documented variable-precision training phases, as overrides of a base policy
_PHASE_OVERRIDES = {
    1: {"z3_compute_dtype": torch.bfloat16, "z1_use_tf32": True, "z2_compute_dtype": torch.float32},
    2: {"z3_compute_dtype": torch.bfloat16, "z1_use_tf32": True, "z2_compute_dtype": torch.float64},
    3: {"z3_compute_dtype": torch.float32, "z3_param_dtype": torch.float32, "z1_use_tf32": True,
        "z2_compute_dtype": torch.float64},
}

# module-name keywords per zone, tried in this order (networks before fixers before bases)
_MODULE_ZONE_RULES = (
    (PrecisionZone.Z3_NEURAL_NETWORK,
     ("nn", "mlp", "transformer", "encoder", "decoder", "learned", "embed", "tower", "parameterization")),
    (PrecisionZone.Z2_CONSERVATION_FIXER, ("fixer", "conservation", "energy", "mass")),
    (PrecisionZone.Z0_NUMERICAL_FOUNDATION, ("sht", "spectral", "legendre", "basis", "fourier", "sigma")),
)


DEFAULT_POLICY = PrecisionPolicy()
