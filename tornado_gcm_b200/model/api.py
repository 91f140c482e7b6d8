"""Reference import path ``model/api.py``: the model API lives in :mod:`tornado_gcm_b200.models.api`."""

from tornado_gcm_b200.models.api import InferenceModel, ModelConfig, NeuralGCMModel, VectorizedModel  # noqa: F401
