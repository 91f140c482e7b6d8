"""Associated Legendre functions and latitude quadrature — reference ``core/associated_legendre.py:21-113``.

The implementation is :mod:`tornado_gcm_b200.core.legendre` (FP64 three-term
recurrences, Gauss and equiangular nodes); this module keeps the reference's
import path.
"""

from tornado_gcm_b200.core.legendre import *  # noqa: F401,F403
from tornado_gcm_b200.core.legendre import (  # noqa: F401
    LATITUDE_SPACINGS, equiangular_nodes, equiangular_nodes_with_poles, evaluate, gauss_legendre_nodes,
    get_latitude_nodes)
