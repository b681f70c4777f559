"""The device GELU (erf form) takes erf from Abramowitz & Stegun 7.1.26, whose published bound
is an absolute error of at most 1.5e-7 in erf. This checks the formula as the kernels write it
(common.cuh gelu_erf: 1 + erf as 2 - erfc or erfc, by the sign) against the exact GELU."""
from __future__ import annotations

import math

import numpy as np

P, A = 0.3275911, (0.254829592, -0.284496736, 1.421413741, -1.453152027, 1.061405429)


def _gelu_as(x: np.ndarray) -> np.ndarray:
    z = np.abs(x) / math.sqrt(2.0)
    t = 1.0 / (1.0 + P * z)
    poly = A[0] + t * (A[1] + t * (A[2] + t * (A[3] + t * A[4])))
    c = t * poly * np.exp(-z * z)
    return 0.5 * x * np.where(x >= 0, 2.0 - c, c)


def test_gelu_erf_formula_is_within_its_published_bound():
    x = np.concatenate([np.linspace(-12, 12, 200001), np.geomspace(1e-8, 12, 20001),
                        -np.geomspace(1e-8, 12, 20001)])
    exact = np.array([0.5 * v * (1.0 + math.erf(v / math.sqrt(2.0))) for v in x])
    err = np.abs(_gelu_as(x) - exact)
    # |GELU error| = 0.5 |x| |erf error| <= 0.5 |x| 1.5e-7.
    assert np.all(err <= 0.5 * np.abs(x) * 1.5e-7 + 1e-30), float(np.max(err / (0.5 * np.abs(x) + 1e-30)))
