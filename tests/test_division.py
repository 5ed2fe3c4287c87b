"""The kernels divide sqrt(v') by the launch-uniform c = sqrt(1 - beta2^t) with
Markstein's correction and the exactly rounded reciprocal y = RN(1/c), inside
the guard 2^-59 <= s < 2^60 (csrc/srs_kernels.cuh, div_by_uniform).  Checked
here in IEEE arithmetic (the same single-rounding multiply and FMA as the GPU)
against IEEE division, for divisors from many AdamW settings."""

from fractions import Fraction

import numpy as np
import pytest

import oracle

GUARD_LO, GUARD_HI = 0x22000000, 0x5D800000  # 2^-59, 2^60


def exact_reciprocal(c: np.float32) -> np.float32:
    """RN(1/c) by exact rational comparison of the neighbours of the estimate."""
    target = 1 / Fraction(float(c))
    est = np.float32(1.0 / float(c))
    candidates = [np.nextafter(est, np.float32(0)), est, np.nextafter(est, np.float32(np.inf))]
    return min(candidates, key=lambda t: abs(Fraction(float(t)) - target))


def divisors():
    out = []
    for beta2 in (0.999, 0.99, 0.95, 0.9999, 0.5, 0.0, 1 - 2.0**-30):
        for step in (1, 2, 3, 5, 10, 100, 1000, 10_000):
            out.append(np.float32((1.0 - beta2**step) ** 0.5))
    return sorted(set(out))


@pytest.mark.parametrize("c", divisors(), ids=lambda c: f"{float(c):.6g}")
def test_reciprocal_division_is_correctly_rounded_inside_the_guard(c):
    y = exact_reciprocal(c)
    # Strided over the whole guarded range, plus every encoding near its ends.
    bad, checked = oracle.check_uniform_division(c, y, GUARD_LO, GUARD_HI, 4099, GUARD_LO,
                                                 GUARD_HI)
    assert bad == 0 and checked > 200_000
    for edge in (GUARD_LO, GUARD_HI - (1 << 18)):
        bad, checked = oracle.check_uniform_division(c, y, edge, edge + (1 << 18), 1, GUARD_LO,
                                                     GUARD_HI)
        assert bad == 0 and checked == 1 << 18


def test_the_guard_is_needed_below_it():
    """Just above 2^-125 the residual underflows and the correction fails; the
    kernel sends such numerators to the IEEE division."""
    c = np.float32((1 - 0.999**1000) ** 0.5)
    bad, _ = oracle.check_uniform_division(c, exact_reciprocal(c), 0x01000000, 0x01400000, 1,
                                           0, 0xFFFFFFFF)
    assert bad > 0
