"""The kernels divide by a value reused many times through its reciprocal with one
correction step (Markstein's method): y = RN(1/b), q0 = RN(a*y), r = RN(a - b*q0) by one
FMA, q = RN(q0 + r*y) by one FMA.  This test checks, in exact rational arithmetic, that
q equals the correctly rounded fp32 quotient RN(a/b) over the value ranges the kernels
divide: logits by sqrt(head_dim), pooled probabilities by row sums, chain vectors by
row sums, scores by their maximum, moments by their normaliser.
"""
from fractions import Fraction

import numpy as np
import pytest


def rn32(x: Fraction) -> np.float32:
    """Round an exact rational to the nearest fp32 (ties to even)."""
    if x == 0:
        return np.float32(0.0)
    # float64 is exact enough to bracket; then pick the nearer fp32 neighbour exactly
    f = np.float32(float(x))
    best, berr = f, abs(Fraction(float(f)) - x)
    for cand in (np.nextafter(f, np.float32(np.inf)), np.nextafter(f, np.float32(-np.inf))):
        err = abs(Fraction(float(cand)) - x)
        if err < berr or (err == berr and (int(np.float32(cand).view(np.uint32)) & 1) == 0 and
                          (int(best.view(np.uint32)) & 1) == 1):
            best, berr = cand, err
    return np.float32(best)


def fma32(a, b, c) -> np.float32:
    return rn32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def markstein(a: np.float32, b: np.float32) -> np.float32:
    y = rn32(Fraction(1) / Fraction(float(b)))
    q0 = rn32(Fraction(float(a)) * Fraction(float(y)))
    r = fma32(-q0, b, a)
    return fma32(r, y, q0)


def exact_quotient(a, b) -> np.float32:
    return rn32(Fraction(float(a)) / Fraction(float(b)))


def _samples(rng, n):
    cases = []
    # logits (16-bit rounded accumulators) by fp32(sqrt(128))
    sd = np.float32(np.sqrt(np.float32(128.0)))
    for a in rng.normal(0, 30, n).astype(np.float32):
        cases.append((np.float32(np.float16(a)), sd))
    # probabilities / row sums; chain vectors / row sums; scores / max
    a = np.exp(rng.uniform(np.log(1e-30), 0.0, n)).astype(np.float32)
    b = np.exp(rng.uniform(np.log(1e-8), np.log(64.0), n)).astype(np.float32)
    cases += list(zip(a, b))
    # divisors with all-ones significands and dividends near powers of two
    ones = [np.float32(np.ldexp(np.float32(2.0) - np.float32(2.0 ** -23), e)) for e in range(-20, 8)]
    near = [np.float32(np.ldexp(np.float32(1.0) + k * np.float32(2.0 ** -23), e))
            for e in range(-30, 1) for k in (0, 1, 2, -1)]
    for bb in ones:
        for aa in near[:: 7]:
            cases.append((np.float32(abs(aa)), bb))
    # small integers (head counts, window lengths)
    for d in range(1, 65):
        for aa in rng.uniform(0, 1, 8).astype(np.float32):
            cases.append((aa, np.float32(d)))
    return cases


@pytest.mark.parametrize("seed", [0, 1])
def test_markstein_division_is_correctly_rounded(seed):
    rng = np.random.default_rng(seed)
    bad = []
    for a, b in _samples(rng, 1500):
        q = markstein(np.float32(a), np.float32(b))
        e = exact_quotient(np.float32(a), np.float32(b))
        if q != e:
            bad.append((float(a), float(b), float(q), float(e)))
    assert not bad, bad[:5]


def rn_bits(x: Fraction, bits: int) -> Fraction:
    """Round an exact rational to `bits` significant bits, nearest, ties to even."""
    if x == 0:
        return x
    sgn, x = (1, x) if x > 0 else (-1, -x)
    e = x.numerator.bit_length() - x.denominator.bit_length()
    while Fraction(2) ** e > x:
        e -= 1
    while Fraction(2) ** (e + 1) <= x:
        e += 1
    ulp = Fraction(2) ** (e - bits + 1)
    q = x / ulp
    fl = q.numerator // q.denominator
    rem = q - fl
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and fl % 2 == 1):
        fl += 1
    return sgn * fl * ulp


def test_bf16_logit_scaling_by_split_constant():
    """The tensor-core passes scale a bf16 logit r by rs = RN_f32(1 / sqrt(128)) as
    RN_bf16(r * hi + RN_bf16(r * lo)) (hi = bf16(rs) = 0x3db5, lo = bf16(rs - hi) =
    0x371e, packed bf16 multiply and FMA) instead of RN_bf16(RN_f32(r * rs)); the two
    agree for every bf16 mantissa (the exponent scales every term alike)."""
    sd = np.float32(np.sqrt(np.float32(128.0)))
    rs = np.float32(np.float32(1.0) / sd)
    hi = Fraction(float(np.array([0x3db50000], np.uint32).view(np.float32)[0]))
    lo = Fraction(float(np.array([0x371e0000], np.uint32).view(np.float32)[0]))
    assert hi == rn_bits(Fraction(float(rs)), 8) and lo == rn_bits(Fraction(float(rs)) - hi, 8)
    for e in (-20, 0, 7):
        for f in range(128):
            for sign in (1, -1):
                r = sign * (1 + Fraction(f, 128)) * Fraction(2) ** e
                ref = rn_bits(Fraction(float(rn32(r * Fraction(float(rs))))), 8)
                assert rn_bits(r * hi + rn_bits(r * lo, 8), 8) == ref, (e, f, sign)
