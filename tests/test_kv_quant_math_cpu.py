"""The KV quantiser's divide-free steps (wzy-flash-serve_b200/csrc/kv_append.cu: kv_group_scale,
kv_recip), restated in exact rational arithmetic and checked against the correctly rounded results
they replace: the reference's scale `__float2half_rn(amax / 127.0f)` (src/wzy_qsa_256k.cuh:117-119)
and the reciprocal RN(1/d) that the packed code path needs for Markstein's quotient."""
from fractions import Fraction

import numpy as np


def rn32(x: Fraction) -> Fraction:
    """x rounded to the nearest fp32 (ties to even), subnormals included, for |x| below fp32's largest
    value."""
    if x == 0:
        return Fraction(0)
    sign = -1 if x < 0 else 1
    x = abs(x)
    e = x.numerator.bit_length() - x.denominator.bit_length()
    if Fraction(2) ** e > x:
        e -= 1
    assert e <= 127, x
    e = max(e, -126)  # subnormals: the quantum stays 2^-149
    m = x / Fraction(2) ** (e - 23)  # in [2^23, 2^24) (below 2^23 for subnormals)
    n, rem = divmod(m.numerator, m.denominator)
    twice = 2 * rem
    if twice > m.denominator or (twice == m.denominator and n & 1):
        n += 1
    return sign * Fraction(n) * Fraction(2) ** (e - 23)


def f32(x: float) -> Fraction:
    return Fraction(float(np.float32(x)))


def neighbours(y: Fraction, k: int):
    """y and the k fp32 values on either side of it."""
    out, lo, hi = [y], np.float32(float(y)), np.float32(float(y))
    for _ in range(k):
        lo, hi = np.nextafter(lo, np.float32(0)), np.nextafter(hi, np.float32(np.inf))
        out += [Fraction(float(lo)), Fraction(float(hi))]
    return out


def test_recip_newton_step_is_correctly_rounded_for_every_fp16_scale():
    """kv_recip: from any start y0 within 2 ulps of 1/d (rcp.approx is specified within 1), the residual
    1 - d*y0 is exact in fp32 and RN(y0 + y0*(1 - d*y0)) equals RN(1/d), for all 31,743 positive finite
    fp16 values d."""
    ds = np.arange(1, 0x7C00, dtype=np.uint16).view(np.float16)
    for d16 in ds:
        d = Fraction(float(d16))
        want = rn32(1 / d)
        for y0 in neighbours(want, 2):
            e_exact = 1 - d * y0
            assert rn32(e_exact) == e_exact, (float(d16), float(y0))
            assert rn32(y0 + y0 * e_exact) == want, (float(d16), float(y0))


def test_group_scale_markstein_matches_division_near_fp16_ties():
    """kv_group_scale: q0 = RN(am*r), e = am - q0*127 (exact), RN(q0 + e*r) with r = RN(1/127) is the
    correctly rounded am / 127, and its fp16 rounding equals the reference's, for fp32 group maxima on
    and within 3 ulps of 127 times every tie point between adjacent positive fp16 values (below fp16's
    largest value and at the tie that rounds to infinity), plus a seeded sample over all exponents
    whose quotient is a normal fp32."""
    r = f32(1 / 127)
    assert np.float32(float(r)).view(np.uint32) == 0x3C010204
    assert abs(r - Fraction(1, 127)) <= abs(Fraction(float(np.nextafter(np.float32(r), np.float32(1)))) -
                                            Fraction(1, 127))
    vals = np.arange(0, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float64)
    ties = [(Fraction(vals[i]) + Fraction(vals[i + 1])) / 2 for i in range(len(vals) - 1)]
    ties.append(Fraction(65504) + Fraction(16))  # 65520: rounds to infinity
    ams = []
    for t in ties:
        ams += neighbours(f32(float(127 * t)), 3)
    rng = np.random.default_rng(7)
    bits = rng.integers(0x04000000, 0x7F7FFFFF, 20000, dtype=np.uint32)  # quotients >= 2^-126
    ams += [Fraction(float(b)) for b in bits.view(np.float32)]
    for am in ams:
        q0 = rn32(am * r)
        e = am - q0 * 127
        assert rn32(e) == e, float(am)
        q = rn32(q0 + e * r)
        assert q == rn32(am / 127), float(am)
        with np.errstate(over="ignore"):
            assert np.float16(float(q)).tobytes() == np.float16(np.float32(float(am)) / np.float32(127)).tobytes()


def test_unclamped_codes_stay_within_127():
    """kv_q8_pack<false> drops the clamp: for a normal fp16 scale d = fp16(RN(am / 127)) every |x| <= am
    gives |x / d| < 127.5, so rint(x / d) is already in [-127, 127]. Checked at the worst case
    (x = am) over fp32 maxima near every normal fp16 scale's rounding interval ends."""
    vals = np.arange(0x0400, 0x7C00, dtype=np.uint16).view(np.float16).astype(np.float64)
    worst = 0.0
    for i in range(len(vals) - 1):
        for edge in ((vals[i] + vals[i + 1]) / 2, vals[i]):
            for am in neighbours(f32(127 * edge), 2):
                d = Fraction(float(np.float16(np.float32(float(am)) / np.float32(127))))
                if d < Fraction(1, 2 ** 14) or d > 65504:
                    continue
                worst = max(worst, float(am / d))
    assert worst < 127.07, worst
