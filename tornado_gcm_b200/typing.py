"""State containers and type aliases — reference ``typing.py:40-178``.

Re-exports :mod:`tornado_gcm_b200.utils.typing` under the reference's import path.
"""

from tornado_gcm_b200.utils.typing import *  # noqa: F401,F403
from tornado_gcm_b200.utils.typing import (  # noqa: F401
    KeyWithCosLatFactor, ModelState, RandomnessState, TrajectoryRepresentations)
