"""Non-dimensional physical units — reference ``units.py:18-144``.

The implementation is :mod:`tornado_gcm_b200.utils.units` (a dimension-vector
quantity type in place of pint); this module keeps the reference's import path.
"""

from tornado_gcm_b200.utils.units import *  # noqa: F401,F403
from tornado_gcm_b200.utils.units import SimUnits, Quantity, Unit  # noqa: F401
