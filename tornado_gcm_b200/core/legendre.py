"""Associated Legendre functions and latitude quadratures (FP64, host side).

Behaviour matches reference ``core/associated_legendre.py:21-113``: the
returned array ``p[m, j, l]`` holds the L2([-1, 1])-normalised associated
Legendre function (Condon-Shortley phase included) of degree ``l`` and
order ``m`` at node ``x_j``; entries with ``l < m`` are zero.

Implementation: for each order ``m`` the sectoral value is built from the
closed-form product ``P_m^m ∝ (-1)^m sqrt(prod_{i<=m} (2i+1)/(2i)) (1-x²)^{m/2}``
and the degree is raised with the standard normalised three-term recurrence
``P_{l}^m = a_lm (x P_{l-1}^m - b_lm P_{l-2}^m)``.  The whole column over
``x`` is vectorised in numpy; everything is done in float64 once per grid.
"""

from __future__ import annotations

import functools

import numpy as np


def _sectoral(n_m: int, x: np.ndarray) -> np.ndarray:
    """Normalised P_m^m(x) for m in [0, n_m), shape (n_m, len(x))."""
    sin_theta = np.sqrt(np.clip(1.0 - x * x, 0.0, None))
    out = np.empty((n_m, x.shape[0]), dtype=np.float64)
    out[0] = np.sqrt(0.5)
    for m in range(1, n_m):
        out[m] = -np.sqrt((2.0 * m + 1.0) / (2.0 * m)) * sin_theta * out[m - 1]
    return out


def evaluate(n_m: int, n_l: int, x: np.ndarray) -> np.ndarray:
    """Normalised associated Legendre table ``p[m, j, l]`` (FP64)."""
    if n_m > n_l:
        raise ValueError(f"Expected n_m <= n_l; got n_m = {n_m} and n_l = {n_l}.")
    x = np.asarray(x, dtype=np.float64)
    p = np.zeros((n_m, x.shape[0], n_l), dtype=np.float64)
    sect = _sectoral(n_m, x)
    for m in range(n_m):
        p[m, :, m] = sect[m]
        if m + 1 < n_l:
            # P_{m+1}^m = sqrt(2m+3) x P_m^m
            p[m, :, m + 1] = np.sqrt(2.0 * m + 3.0) * x * sect[m]
        for l in range(m + 2, n_l):
            a = np.sqrt((4.0 * l * l - 1.0) / (l * l - m * m))
            b = np.sqrt(((l - 1.0) ** 2 - m * m) / (4.0 * (l - 1.0) ** 2 - 1.0))
            p[m, :, l] = a * (x * p[m, :, l - 1] - b * p[m, :, l - 2])
    return p


def gauss_legendre_nodes(n: int) -> tuple[np.ndarray, np.ndarray]:
    """Gauss-Legendre nodes (ascending) and weights summing to 2."""
    x, w = np.polynomial.legendre.leggauss(n)
    return x.astype(np.float64), w.astype(np.float64)


def _weights_for_nodes(x: np.ndarray) -> np.ndarray:
    """Quadrature weights exact for Legendre polynomials up to len(x)-1."""
    n = x.shape[0]
    legendre = evaluate(n_m=1, n_l=n, x=x)[0].T  # (l, j)
    rhs = np.zeros(n)
    rhs[0] = 1.0
    w = np.linalg.solve(legendre, rhs)
    return w / w.sum() * 2.0


@functools.lru_cache(maxsize=64)
def equiangular_nodes(n: int) -> tuple[np.ndarray, np.ndarray]:
    """Cell-centred equally spaced latitudes (no poles)."""
    dtheta = np.pi / n
    theta = -np.pi / 2 + dtheta * (np.arange(n) + 0.5)
    x = np.sin(theta)
    return x, _weights_for_nodes(x)


@functools.lru_cache(maxsize=64)
def equiangular_nodes_with_poles(n: int) -> tuple[np.ndarray, np.ndarray]:
    """Equally spaced latitudes including both poles."""
    theta = np.linspace(-np.pi / 2, np.pi / 2, n)
    x = np.sin(theta)
    return x, _weights_for_nodes(x)


LATITUDE_SPACINGS = dict(
    gauss=gauss_legendre_nodes,
    equiangular=equiangular_nodes,
    equiangular_with_poles=equiangular_nodes_with_poles,
)


def get_latitude_nodes(n: int, spacing: str) -> tuple[np.ndarray, np.ndarray]:
    fn = LATITUDE_SPACINGS.get(spacing)
    if fn is None:
        raise ValueError(f"Unknown spacing: {spacing}. Available: {list(LATITUDE_SPACINGS)}")
    return fn(n)
