"""Model package under the reference's import path (``tornado_gcm.model``)."""

from tornado_gcm_b200.model.atmosphere import AtmosphereConfig, AtmosphericModel
from tornado_gcm_b200.model.dynamic_data_forcing import build_dynamic_data_forcing_torch
from tornado_gcm_b200.model.legacy import PressureLevelConfig, PressureLevelModel
from tornado_gcm_b200.models.api import InferenceModel, ModelConfig, NeuralGCMModel, VectorizedModel

__all__ = ["AtmosphereConfig", "AtmosphericModel", "InferenceModel", "ModelConfig", "NeuralGCMModel",
           "PressureLevelConfig", "PressureLevelModel", "VectorizedModel", "build_dynamic_data_forcing_torch"]
