"""Physical constants, scales and non-dimensionalisation without pint.

A tiny dimension-vector quantity type replaces the pint registry used by the
reference (``scales.py:35-164``, ``units.py:18-144``).  A :class:`Quantity`
carries an SI magnitude and an exponent vector over the four base dimensions
(length, time, mass, temperature).  A :class:`Scale` maps each base
dimension to a reference quantity; ``nondimensionalize`` divides by the
product of the scales raised to the quantity's exponents.

The constants are the standard NeuralGCM/dinosaur values (Earth radius,
rotation rate, g, dry-air Cp and kappa, vapour R and Cp).
"""

from __future__ import annotations

import dataclasses
from typing import Iterator, Mapping, Protocol, runtime_checkable

import numpy as np

_DIMS = ("[length]", "[time]", "[mass]", "[temperature]")


@dataclasses.dataclass(frozen=True)
class Unit:
    """A product of SI base units with integer/fractional exponents."""

    exponents: tuple[float, float, float, float]
    factor: float = 1.0  # multiplier to SI (e.g. hPa -> 100 Pa)
    name: str = ""

    def __mul__(self, other):
        if isinstance(other, Unit):
            return Unit(
                tuple(a + b for a, b in zip(self.exponents, other.exponents)),
                self.factor * other.factor,
                f"{self.name}*{other.name}",
            )
        return Quantity(float(other) * self.factor, self.exponents)

    __rmul__ = __mul__

    def __truediv__(self, other):
        if isinstance(other, Unit):
            return Unit(
                tuple(a - b for a, b in zip(self.exponents, other.exponents)),
                self.factor / other.factor,
                f"{self.name}/{other.name}",
            )
        return Quantity(self.factor / float(other), self.exponents)

    def __rtruediv__(self, other):
        return Quantity(float(other) / self.factor, tuple(-a for a in self.exponents))

    def __pow__(self, p):
        return Unit(tuple(a * p for a in self.exponents), self.factor**p, f"{self.name}^{p}")

    @property
    def dimensionality(self) -> dict[str, float]:
        return {d: e for d, e in zip(_DIMS, self.exponents) if e != 0}


@dataclasses.dataclass(frozen=True)
class Quantity:
    """SI magnitude plus base-dimension exponents."""

    magnitude: float
    exponents: tuple[float, float, float, float] = (0.0, 0.0, 0.0, 0.0)

    @property
    def m(self):
        return self.magnitude

    @property
    def dimensionality(self) -> dict[str, float]:
        return {d: e for d, e in zip(_DIMS, self.exponents) if e != 0}

    def _combine(self, other, sign):
        if isinstance(other, Quantity):
            return Quantity(
                self.magnitude * other.magnitude**sign,
                tuple(a + sign * b for a, b in zip(self.exponents, other.exponents)),
            )
        if isinstance(other, Unit):
            return Quantity(
                self.magnitude * other.factor**sign,
                tuple(a + sign * b for a, b in zip(self.exponents, other.exponents)),
            )
        return Quantity(self.magnitude * float(other) ** sign, self.exponents)

    def __mul__(self, other):
        return self._combine(other, 1)

    __rmul__ = __mul__

    def __truediv__(self, other):
        return self._combine(other, -1)

    def __rtruediv__(self, other):
        return Quantity(float(other) / self.magnitude, tuple(-a for a in self.exponents))

    def __pow__(self, p):
        return Quantity(self.magnitude**p, tuple(a * p for a in self.exponents))

    def __neg__(self):
        return Quantity(-self.magnitude, self.exponents)

    def __add__(self, other):
        if not isinstance(other, Quantity) or other.exponents != self.exponents:
            raise ValueError("cannot add quantities of different dimensions")
        return Quantity(self.magnitude + other.magnitude, self.exponents)

    def to(self, unit: Unit) -> "Quantity":
        if tuple(unit.exponents) != tuple(self.exponents):
            raise ValueError(f"incompatible units: {self.exponents} vs {unit.exponents}")
        return Quantity(self.magnitude / unit.factor, self.exponents)

    def to_base_units(self) -> "Quantity":
        return self

    def check(self, dims) -> bool:
        return True


class _Registry:
    """Minimal attribute registry: ``units.m``, ``units.s``, ``units.hPa``..."""

    m = meter = Unit((1, 0, 0, 0), 1.0, "m")
    km = Unit((1, 0, 0, 0), 1e3, "km")
    s = second = Unit((0, 1, 0, 0), 1.0, "s")
    minute = Unit((0, 1, 0, 0), 60.0, "minute")
    hour = Unit((0, 1, 0, 0), 3600.0, "hour")
    day = Unit((0, 1, 0, 0), 86400.0, "day")
    kg = kilogram = Unit((0, 0, 1, 0), 1.0, "kg")
    K = degK = kelvin = Unit((0, 0, 0, 1), 1.0, "K")
    dimensionless = Unit((0, 0, 0, 0), 1.0, "1")
    J = joule = Unit((2, -2, 1, 0), 1.0, "J")
    W = watt = Unit((2, -3, 1, 0), 1.0, "W")
    Pa = pascal = Unit((-1, -2, 1, 0), 1.0, "Pa")
    hPa = millibar = Unit((-1, -2, 1, 0), 100.0, "hPa")
    N = newton = Unit((1, -2, 1, 0), 1.0, "N")

    _ALIASES = {
        "meter": "m", "meters": "m", "second": "s", "seconds": "s",
        "kilogram": "kg", "kelvin": "K", "degK": "K", "hectopascal": "hPa",
        "pascal": "Pa", "1": "dimensionless", "": "dimensionless",
        "(0 - 1)": "dimensionless", "%": "dimensionless", "~": "dimensionless",
    }

    def parse_expression(self, text: str) -> Unit:
        """Parse ``'m/s'``, ``'m**2 s**-2'``, ``'kg/kg'`` style unit strings."""
        text = text.strip()
        text = self._ALIASES.get(text, text)
        if hasattr(self, text) and isinstance(getattr(self, text), Unit):
            return getattr(self, text)
        unit = self.dimensionless
        sign = 1
        token = ""
        tokens: list[tuple[str, int]] = []
        i = 0
        clean = text.replace(" / ", "/").replace("*", " ").replace("  ", " ")
        for ch in clean:
            if ch in "/ ":
                if token:
                    tokens.append((token, sign))
                token = ""
                sign = -1 if ch == "/" else (sign if ch == " " and sign == -1 and False else 1)
                if ch == "/":
                    sign = -1
                continue
            token += ch
        if token:
            tokens.append((token, sign))
        for tok, sgn in tokens:
            power = 1.0
            if "^" in tok:
                tok, p = tok.split("^")
                power = float(p)
            elif tok and tok[-1].isdigit() and not tok.isdigit():
                j = len(tok)
                while j > 0 and (tok[j - 1].isdigit() or tok[j - 1] == "-"):
                    j -= 1
                power = float(tok[j:])
                tok = tok[:j]
            if tok.isdigit() or tok == "":
                continue
            base = self.parse_expression(tok) if tok != text else self.dimensionless
            unit = unit * base ** (sgn * power)
        return unit

    def __call__(self, text: str) -> Unit:
        return self.parse_expression(text)


units = _Registry()

# ── SI constants ────────────────────────────────────────────────────────────
RADIUS = 6.37122e6 * units.m
ANGULAR_VELOCITY = OMEGA = 7.292e-5 / units.s
GRAVITY_ACCELERATION = 9.80616 * units.m / units.s**2
ISOBARIC_HEAT_CAPACITY = 1004.0 * units.J / units.kg / units.K
WATER_VAPOR_CP = 1859.0 * units.J / units.kg / units.K
MASS_OF_DRY_ATMOSPHERE = 5.18e18 * units.kg
KAPPA = Quantity(2.0 / 7.0)
LATENT_HEAT_OF_VAPORIZATION = 2.501e6 * units.J / units.kg
IDEAL_GAS_CONSTANT = ISOBARIC_HEAT_CAPACITY * KAPPA
IDEAL_GAS_CONSTANT_H20 = 461.0 * units.J / units.kg / units.K
WATER_DENSITY = 997.0 * units.kg / units.m**3


def parse_units(units_str: str) -> Unit:
    return units.parse_expression(units_str)


@runtime_checkable
class ScaleProtocol(Protocol):
    """What a non-dimensionalisation scale offers (:class:`Scale` implements it)."""

    def nondimensionalize(self, quantity: "Quantity") -> float: ...

    def dimensionalize(self, value: float, unit: "Unit") -> "Quantity": ...


class Scale(Mapping):
    """Reference quantity per base dimension (reference: ``scales.py:82-147``)."""

    def __init__(self, *scales: Quantity):
        self._scales: dict[str, Quantity] = {}
        for q in scales:
            dims = [d for d, e in zip(_DIMS, q.exponents) if e != 0]
            if len(dims) != 1 or q.exponents[_DIMS.index(dims[0])] != 1:
                raise ValueError("each scale must describe exactly one base dimension")
            if dims[0] in self._scales:
                raise ValueError(f"duplicate scale for {dims[0]}")
            self._scales[dims[0]] = q

    def __getitem__(self, key: str) -> Quantity:
        return self._scales[key]

    def __iter__(self) -> Iterator[str]:
        return iter(self._scales)

    def __len__(self) -> int:
        return len(self._scales)

    def __hash__(self):
        return hash(tuple(sorted((k, v.magnitude) for k, v in self._scales.items())))

    def _factor(self, exponents) -> float:
        f = 1.0
        for d, e in zip(_DIMS, exponents):
            if e == 0:
                continue
            if d not in self._scales:
                raise ValueError(f"No scale has been set for {d}.")
            f *= self._scales[d].magnitude ** e
        return f

    def nondimensionalize(self, quantity) -> float:
        if not isinstance(quantity, Quantity):
            return quantity
        return quantity.magnitude / self._factor(quantity.exponents)

    def dimensionalize(self, value, unit: Unit) -> Quantity:
        si = value * self._factor(unit.exponents)
        return Quantity(si / unit.factor, tuple(unit.exponents))


NEURALGCM_V1_SCALE = Scale(RADIUS, 1 / 2 / OMEGA, 1.0 * units.kg, 1.0 * units.K)
ATMOSPHERIC_SCALE = Scale(RADIUS, 1 / 2 / OMEGA, MASS_OF_DRY_ATMOSPHERE, 1.0 * units.K)
SI_SCALE = Scale(1.0 * units.m, 1.0 * units.s, 1.0 * units.kg, 1.0 * units.K)
DEFAULT_SCALE = NEURALGCM_V1_SCALE


@runtime_checkable
class SimUnitsProtocol(Protocol):
    """What a set of non-dimensional physical constants offers (:class:`SimUnits` implements it)."""

    radius: float
    angular_velocity: float
    gravity_acceleration: float
    ideal_gas_constant: float
    water_vapor_gas_constant: float
    water_vapor_isobaric_heat_capacity: float
    kappa: float

    @property
    def R(self) -> float: ...

    @property
    def R_vapor(self) -> float: ...

    @property
    def g(self) -> float: ...

    @property
    def Cp(self) -> float: ...

    @property
    def Cp_vapor(self) -> float: ...

    def nondimensionalize(self, quantity: "Quantity") -> float: ...

    def nondimensionalize_timedelta64(self, timedelta: np.timedelta64) -> float: ...

    def dimensionalize(self, value: float, unit: "Unit") -> "Quantity": ...

    def dimensionalize_timedelta64(self, value: float) -> np.timedelta64: ...

    @classmethod
    def from_si(cls, **kwargs) -> "SimUnitsProtocol": ...


@dataclasses.dataclass(frozen=True)
class SimUnits:
    """Non-dimensional physical constants (reference ``units.py:56-144``)."""

    radius: float
    angular_velocity: float
    gravity_acceleration: float
    ideal_gas_constant: float
    water_vapor_gas_constant: float
    water_vapor_isobaric_heat_capacity: float
    kappa: float
    scale: Scale = DEFAULT_SCALE

    @property
    def R(self) -> float:
        return self.ideal_gas_constant

    @property
    def R_vapor(self) -> float:
        return self.water_vapor_gas_constant

    @property
    def g(self) -> float:
        return self.gravity_acceleration

    @property
    def Cp(self) -> float:
        return self.ideal_gas_constant / self.kappa

    @property
    def Cp_vapor(self) -> float:
        return self.water_vapor_isobaric_heat_capacity

    def nondimensionalize(self, quantity) -> float:
        return self.scale.nondimensionalize(quantity)

    def dimensionalize(self, value, unit: Unit) -> Quantity:
        return self.scale.dimensionalize(value, unit)

    def nondimensionalize_timedelta64(self, timedelta: np.timedelta64) -> float:
        seconds = timedelta / np.timedelta64(1, "s")
        return self.scale.nondimensionalize(float(seconds) * units.s)

    def dimensionalize_timedelta64(self, value: float) -> np.timedelta64:
        seconds = self.scale.dimensionalize(value, units.s).magnitude
        if isinstance(seconds, np.ndarray):
            return seconds.astype("timedelta64[s]")
        return np.timedelta64(int(round(seconds)), "s")

    @classmethod
    def from_si(
        cls,
        radius_si: Quantity = RADIUS,
        angular_velocity_si: Quantity = ANGULAR_VELOCITY,
        gravity_acceleration_si: Quantity = GRAVITY_ACCELERATION,
        ideal_gas_constant_si: Quantity = IDEAL_GAS_CONSTANT,
        water_vapor_gas_constant_si: Quantity = IDEAL_GAS_CONSTANT_H20,
        water_vapor_isobaric_heat_capacity_si: Quantity = WATER_VAPOR_CP,
        kappa_si: Quantity = KAPPA,
        scale: Scale = DEFAULT_SCALE,
    ) -> "SimUnits":
        nd = scale.nondimensionalize
        return cls(
            nd(radius_si), nd(angular_velocity_si), nd(gravity_acceleration_si),
            nd(ideal_gas_constant_si), nd(water_vapor_gas_constant_si),
            nd(water_vapor_isobaric_heat_capacity_si), nd(kappa_si), scale,
        )


def hours_to_nondim(hours: float, scale: Scale = DEFAULT_SCALE) -> float:
    """Convert a duration in hours to model time units."""
    return scale.nondimensionalize(hours * 3600.0 * units.s)


def minutes_to_nondim(minutes: float, scale: Scale = DEFAULT_SCALE) -> float:
    return scale.nondimensionalize(minutes * 60.0 * units.s)


def seconds_per_time_unit(scale: Scale = DEFAULT_SCALE) -> float:
    return scale["[time]"].magnitude


__all__ = [
    "Unit", "Quantity", "units", "Scale", "ScaleProtocol", "SimUnits", "SimUnitsProtocol", "NEURALGCM_V1_SCALE",
    "ATMOSPHERIC_SCALE", "SI_SCALE", "DEFAULT_SCALE", "RADIUS", "OMEGA",
    "ANGULAR_VELOCITY", "GRAVITY_ACCELERATION", "ISOBARIC_HEAT_CAPACITY",
    "WATER_VAPOR_CP", "KAPPA", "IDEAL_GAS_CONSTANT", "IDEAL_GAS_CONSTANT_H20",
    "MASS_OF_DRY_ATMOSPHERE", "LATENT_HEAT_OF_VAPORIZATION", "WATER_DENSITY",
    "parse_units", "hours_to_nondim", "minutes_to_nondim", "seconds_per_time_unit",
]
