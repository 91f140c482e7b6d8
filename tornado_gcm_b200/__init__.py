"""tornado_gcm_b200: a Blackwell-native hybrid neural/spectral GCM framework.

Public API mirrors TornadoGCM (``tornado_gcm``): ``NeuralGCMModel`` /
``AtmosphericModel``, ``MPInference`` / ``SDAInference``, the trainers, the
PZHA precision zones and the SDA scheduler.  Hot paths run in hand-written
sm_100a CUDA kernels (``tornado_gcm_b200.ops``); the torch code paths are
the CPU implementation and numerical oracle.
"""

__version__ = "0.1.0"
