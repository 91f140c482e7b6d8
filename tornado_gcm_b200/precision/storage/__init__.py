"""Mixed-precision storage — reference ``precision/storage/``."""

from tornado_gcm_b200.precision.storage.codec import ExactCodec, LossyCodec
from tornado_gcm_b200.precision.storage.manager import SDAStorageManager

__all__ = ["ExactCodec", "LossyCodec", "SDAStorageManager"]
