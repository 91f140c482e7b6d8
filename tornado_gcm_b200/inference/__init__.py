"""Inference engines — reference ``inference/``."""

from tornado_gcm_b200.inference.production import (AsyncStoreWriter, AsyncZarrWriter, EnsembleRunner,
                                                   InferenceConfig, InferenceRunner, NumpyWriter, StoreWriter,
                                                   ZarrWriter, load_initial_condition, save_forecast)
from tornado_gcm_b200.inference.runner import MPInference, auto_estimate_chunk_size
from tornado_gcm_b200.inference.sda_runner import SDAInference

__all__ = ["AsyncStoreWriter", "AsyncZarrWriter", "EnsembleRunner", "InferenceConfig", "InferenceRunner",
           "MPInference", "NumpyWriter", "SDAInference", "StoreWriter", "ZarrWriter", "auto_estimate_chunk_size",
           "load_initial_condition", "save_forecast"]
