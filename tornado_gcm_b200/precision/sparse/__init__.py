"""Sparse and split-precision spectral representations — reference ``precision/sparse/``."""

from tornado_gcm_b200.precision.sparse.adaptive_sparse import SparseSpectralTransform
from tornado_gcm_b200.precision.sparse.ops import (adaptive_threshold_mask, count_structural_zeros,
                                                   memory_savings_ratio, triangular_mask)
from tornado_gcm_b200.precision.sparse.spectral_sparse import (MixedPrecisionSparse, PackedTriangle, SparseConfig,
                                                               SpectralSparseState, ThresholdPacked, TriangleLayout)

__all__ = ["MixedPrecisionSparse", "PackedTriangle", "SparseConfig", "ThresholdPacked", "TriangleLayout", "SparseSpectralTransform", "SpectralSparseState",
           "adaptive_threshold_mask", "count_structural_zeros", "memory_savings_ratio", "triangular_mask"]
