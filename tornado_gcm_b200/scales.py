"""Physical constants and non-dimensionalisation scales — reference ``scales.py:35-164``.

Re-exports :mod:`tornado_gcm_b200.utils.units` under the reference's import path:
``units`` (the unit registry), the constants (``RADIUS``, ``ANGULAR_VELOCITY``,
``GRAVITY_ACCELERATION``, …), ``Scale``, ``NEURALGCM_V1_SCALE`` (length = Earth
radius, time = 1/(2Ω)), ``ATMOSPHERIC_SCALE``, ``SI_SCALE`` and ``DEFAULT_SCALE``.
"""

from tornado_gcm_b200.utils.units import *  # noqa: F401,F403
from tornado_gcm_b200.utils.units import (  # noqa: F401
    ANGULAR_VELOCITY, ATMOSPHERIC_SCALE, DEFAULT_SCALE, GRAVITY_ACCELERATION, IDEAL_GAS_CONSTANT,
    IDEAL_GAS_CONSTANT_H20, ISOBARIC_HEAT_CAPACITY, KAPPA, LATENT_HEAT_OF_VAPORIZATION, MASS_OF_DRY_ATMOSPHERE,
    NEURALGCM_V1_SCALE, OMEGA, RADIUS, SI_SCALE, WATER_DENSITY, WATER_VAPOR_CP, Scale, parse_units, units)
