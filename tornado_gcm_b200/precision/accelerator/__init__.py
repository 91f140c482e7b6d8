"""Accelerated operators (sm_100a) — reference ``precision/accelerator/``."""

from tornado_gcm_b200.precision.accelerator.graphed_step import FusedAdvanceKernel
from tornado_gcm_b200.precision.accelerator.reductions import (KahanAccumulator, spectral_norm,
                                                               sphere_integrate)
from tornado_gcm_b200.precision.accelerator.registry import AcceleratorRegistry, get_global_registry
from tornado_gcm_b200.precision.accelerator.sm100_sht import sht_legendre_forward, sht_legendre_inverse

__all__ = ["AcceleratorRegistry", "FusedAdvanceKernel", "KahanAccumulator", "get_global_registry",
           "sht_legendre_forward", "sht_legendre_inverse", "spectral_norm", "sphere_integrate"]
