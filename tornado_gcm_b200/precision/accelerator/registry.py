"""Operator registry — reference ``precision/accelerator/registry.py:35-269``.

Maps an operator name to implementations ranked by priority, with an
optional backend filter.  Built-in operators (registered by
:func:`get_global_registry`):

=====================  ======================================  ==========
name                   sm100 implementation (priority 100)     torch (10)
=====================  ======================================  ==========
sht_legendre_inverse   tcgen05 TF32 grouped GEMM               FP64 einsum
sht_legendre_forward   tcgen05 TF32 grouped GEMM               FP64 einsum
sphere_integrate       FP64 row-reduction kernel               FP64 einsum
spectral_norm          FP64 row-reduction kernel               FP64 sum
conservation_fix       FP64 fixer kernel pair (with adjoint)   torch ops
=====================  ======================================  ==========

The torch entries are the numerical oracle and the CPU path; the sm100
entries require CUDA tensors.  The model step does not go through the
registry (it calls the kernels directly); the registry serves users who
select implementations by name.
"""

from __future__ import annotations

import dataclasses
import logging
from typing import Any, Callable, Optional

logger = logging.getLogger(__name__)


@dataclasses.dataclass
class _Entry:
    name: str
    impl: Callable
    priority: int
    backend: str
    meta: dict = dataclasses.field(default_factory=dict)


class AcceleratorRegistry:
    """Priority-ranked implementations per operator name."""

    def __init__(self, default_backend: str = "auto") -> None:
        self._entries: dict[str, list[_Entry]] = {}
        self._default_backend = default_backend
        self._cache: dict[str, Callable] = {}

    def register(self, name: str, impl: Callable, priority: int = 0, backend: str = "torch", **meta: Any) -> None:
        lst = self._entries.setdefault(name, [])
        lst.append(_Entry(name, impl, priority, backend, meta))
        lst.sort(key=lambda e: -e.priority)
        for k in [k for k in self._cache if k.split(":", 1)[0] == name]:
            del self._cache[k]

    def get(self, name: str, backend: Optional[str] = None) -> Callable:
        want = backend or self._default_backend
        key = f"{name}:{want}"
        hit = self._cache.get(key)
        if hit is not None:
            return hit
        entries = self._entries.get(name)
        if not entries:
            raise KeyError(f"No implementation registered for operator '{name}'")
        chosen = entries[0]
        if want != "auto":
            match = [e for e in entries if e.backend == want]
            if match:
                chosen = match[0]
            else:
                logger.warning("no '%s' implementation of %s; using %s", want, name, chosen.backend)
        self._cache[key] = chosen.impl
        return chosen.impl

    def available(self, name: str) -> list[str]:
        return [e.backend for e in self._entries.get(name, [])]

    def list_operators(self) -> list[str]:
        return list(self._entries)

    def info(self, name: str) -> list[dict]:
        return [{"backend": e.backend, "priority": e.priority, "meta": dict(e.meta)}
                for e in self._entries.get(name, [])]

    def clear(self) -> None:
        self._entries.clear()
        self._cache.clear()

    def __contains__(self, name: str) -> bool:
        return name in self._entries

    def __len__(self) -> int:
        return len(self._entries)


_GLOBAL: Optional[AcceleratorRegistry] = None


def _register_builtin_operators(reg: AcceleratorRegistry) -> None:
    from tornado_gcm_b200.precision.accelerator import reductions, sm100_sht

    reg.register("sht_legendre_inverse", sm100_sht.sht_legendre_inverse_sm100, 100, "sm100", precision="tf32")
    reg.register("sht_legendre_inverse", sm100_sht.sht_legendre_inverse_torch, 10, "torch", precision="fp64")
    reg.register("sht_legendre_forward", sm100_sht.sht_legendre_forward_sm100, 100, "sm100", precision="tf32")
    reg.register("sht_legendre_forward", sm100_sht.sht_legendre_forward_torch, 10, "torch", precision="fp64")
    reg.register("sphere_integrate", reductions.sphere_integrate_sm100, 100, "sm100", accumulate="fp64")
    reg.register("sphere_integrate", reductions.sphere_integrate_torch, 10, "torch", accumulate="fp64")
    reg.register("spectral_norm", reductions.spectral_norm_sm100, 100, "sm100", accumulate="fp64")
    reg.register("spectral_norm", reductions.spectral_norm_torch, 10, "torch", accumulate="fp64")
    reg.register("conservation_fix", reductions.conservation_fix_sm100, 100, "sm100", accumulate="fp64")
    reg.register("conservation_fix", reductions.conservation_fix_torch, 10, "torch", accumulate="fp64")


def get_global_registry() -> AcceleratorRegistry:
    global _GLOBAL
    if _GLOBAL is None:
        _GLOBAL = AcceleratorRegistry()
        _register_builtin_operators(_GLOBAL)
    return _GLOBAL
