"""The row kernels divide by a per-row scalar b through its correctly rounded reciprocal
y = RN(1/b) and two FMA residual corrections (ctorch_b200/csrc/elementwise.cuh, div_by_row):

    q0 = RN(a*y);  q1 = RN(q0 + RN(a - b*q0)*y);  q2 = RN(q1 + RN(a - b*q1)*y)

and claim q2 == RN(a/b), the IEEE quotient of ctorch's division functor
(src/ops/functors.h:64-66). This file checks the claim on the CPU, independently of the
GPU: every step is restated over exact rationals with one round-to-nearest-even per operation
(an FMA rounds once), at float64 and float32 precision, on quotients that land as close to a
rounding midpoint as the format allows, on all-ones and power-of-two significands, and on random
operands. The GPU tests then compare the kernels bit for bit with the oracle's plain division."""
from fractions import Fraction

import numpy as np
import pytest


def _rn(x: Fraction, p: int) -> Fraction:
    """x rounded to nearest-even with a p-bit significand (no exponent limits: every case here is
    far from overflow and underflow, as the kernels' exponent guards require)."""
    if x == 0:
        return Fraction(0)
    s = -1 if x < 0 else 1
    x = abs(x)
    e = x.numerator.bit_length() - x.denominator.bit_length()
    if Fraction(2) ** e > x:
        e -= 1
    scale = Fraction(2) ** (p - 1 - e)  # x * scale in [2^(p-1), 2^p)
    v = x * scale
    n, r = divmod(v.numerator, v.denominator)
    twice = 2 * r
    if twice > v.denominator or (twice == v.denominator and n % 2 == 1):
        n += 1
    return s * Fraction(n) / scale


def _sequence(a: Fraction, b: Fraction, p: int) -> Fraction:
    y = _rn(1 / b, p)
    q0 = _rn(a * y, p)
    r0 = _rn(a - b * q0, p)
    q1 = _rn(q0 + r0 * y, p)
    r1 = _rn(a - b * q1, p)
    return _rn(q1 + r1 * y, p)


def _sig(rng, p):
    return (1 << (p - 1)) | int(rng.integers(0, 1 << (p - 1)))


def _cases(p: int, n: int, seed: int):
    rng = np.random.default_rng(seed)
    out = []
    ones = (1 << p) - 1
    for i in range(n):
        kind = i % 4
        eb = int(rng.integers(-40, 40))
        if kind == 0:  # random operands
            b = Fraction(_sig(rng, p), 1 << (p - 1)) * Fraction(2) ** eb
            a = Fraction(_sig(rng, p), 1 << (p - 1)) * Fraction(2) ** int(rng.integers(-40, 40))
        else:
            if kind == 1:  # divisor with an all-ones significand
                bs = ones
            elif kind == 2:  # divisor a power of two times a random significand near 1 or 2
                bs = (1 << (p - 1)) + int(rng.integers(0, 8)) if rng.random() < 0.5 else ones - int(rng.integers(0, 8))
            else:
                bs = _sig(rng, p)
            b = Fraction(bs, 1 << (p - 1)) * Fraction(2) ** eb
            # a quotient near the midpoint m between q and its successor: a = RN(b*m) +- k ulp
            q = Fraction(_sig(rng, p), 1 << (p - 1)) * Fraction(2) ** int(rng.integers(-20, 20))
            eq = q.numerator.bit_length() - q.denominator.bit_length()
            if Fraction(2) ** eq > q:
                eq -= 1
            m = q + Fraction(2) ** (eq - p)  # half an ulp above q
            a = _rn(b * m, p)
            k = int(rng.integers(-2, 3))
            if k:
                ea = a.numerator.bit_length() - a.denominator.bit_length()
                if Fraction(2) ** ea > a:
                    ea -= 1
                a = a + k * Fraction(2) ** (ea - p + 1)
        if rng.random() < 0.5:
            a = -a
        if rng.random() < 0.25:
            b = -b
        out.append((a, b))
    return out


@pytest.mark.parametrize("p,name", [(53, "float64"), (24, "float32")])
def test_two_corrections_give_the_correctly_rounded_quotient(p, name):
    bad = []
    for a, b in _cases(p, 6000, seed=p):
        got = _sequence(a, b, p)
        want = _rn(a / b, p)
        if got != want:
            bad.append((a, b, got, want))
    assert not bad, f"{name}: {len(bad)} quotients differ, first {bad[0]}"


def test_the_product_with_the_reciprocal_alone_is_not_enough():
    """q0 = RN(a*y) by itself is often one ulp off on these cases, so the cases do reach the
    rounding boundaries the corrections are there for (the test above does not pass vacuously)."""
    p = 24
    off = 0
    for a, b in _cases(p, 2000, seed=7):
        off += _rn(a * _rn(1 / b, p), p) != _rn(a / b, p)
    assert off > 200
