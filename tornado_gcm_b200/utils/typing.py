"""State containers and type aliases (reference ``typing.py:40-178``)."""

from __future__ import annotations

import dataclasses
from typing import Any, Callable, Generic, Mapping, Optional, TypeVar, Union

import numpy as np
import torch

Tensor = torch.Tensor
Array = Union[np.ndarray, torch.Tensor]
Numeric = Union[float, int, torch.Tensor]
PRNGKeyArray = Any
PyTreeState = TypeVar("PyTreeState")
Pytree = Any
PyTreeMemory = Pytree
PyTreeDiagnostics = Pytree
AuxFeatures = dict[str, Any]
DataState = dict[str, Any]
ForcingData = dict[str, Any]
Forcing = Pytree


@dataclasses.dataclass(eq=True, order=True, frozen=True)
class KeyWithCosLatFactor:
    """A field name plus the power of cos(lat) it carries."""

    name: str
    factor_order: int
    filter_strength: float = 0.0


@dataclasses.dataclass
class RandomnessState:
    """Random field on the sphere: internal core plus nodal/modal values."""

    core: Pytree | None = None
    nodal_value: Pytree | None = None
    modal_value: Pytree | None = None
    prng_key: PRNGKeyArray | None = None
    prng_step: int | None = None


@dataclasses.dataclass
class ModelState(Generic[PyTreeState]):
    """Prognostic state plus memory, diagnostics and randomness."""

    state: PyTreeState
    memory: Pytree = None
    diagnostics: Pytree = dataclasses.field(default_factory=dict)
    randomness: RandomnessState = dataclasses.field(default_factory=RandomnessState)


@dataclasses.dataclass
class TrajectoryRepresentations:
    data_nodal_trajectory: Pytree
    data_modal_trajectory: Pytree
    model_nodal_trajectory: Pytree
    model_modal_trajectory: Pytree

    def get_representation(self, *, is_nodal: bool, is_encoded: bool) -> Pytree:
        return {
            (True, True): self.model_nodal_trajectory,
            (True, False): self.data_nodal_trajectory,
            (False, True): self.model_modal_trajectory,
            (False, False): self.data_modal_trajectory,
        }[(is_nodal, is_encoded)]


StateFn = Callable[[Any], Any]
TimeStepFn = Callable[[Any], Any]
PyTreeTermsFn = Callable[[Any], Any]
PyTreeInverseFn = Callable[[Any, Numeric], Any]
PyTreeFilterFn = Callable[[Any], Any]
PyTreeStepFilterFn = Callable[[Any, Any], Any]
ForcingFn = Callable[[ForcingData, float], Forcing]
PostProcessFn = Callable[..., Any]
Params = Optional[Mapping[str, Mapping[str, Array]]]
ParameterizationFn = Callable[..., Any]
TransformFn = Callable[[Pytree], Pytree]
