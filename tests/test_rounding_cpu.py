"""The branch-free rounding of act_quant's 16-bit path, restated in exact rational arithmetic and
checked against the IEEE quotient on near-tie operands (no GPU). The kernel computes, in fp32 with
round-to-nearest-even, z = RN(1/s), y = RN(x * z), r = RN(x - y * s) (one FMA), q = RN(y + r * z)
(one FMA) and uses rint(q); the claim (Markstein's theorem) is q == RN(x / s), so rint(q) equals the
reference's round(x / s) (reference.py:13-14)."""
import math
import random
from fractions import Fraction as F

import numpy as np


def rn32(v: F) -> F:
    """v rounded to the nearest fp32 value, ties to even (normal range; subnormal quantum below)."""
    if v == 0:
        return F(0)
    sgn = -1 if v < 0 else 1
    a = abs(v)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while a >= F(2) ** (e + 1):
        e += 1
    while a < F(2) ** e:
        e -= 1
    quantum = F(2) ** (max(e, -126) - 23)
    m = a / quantum
    fl = m.numerator // m.denominator
    rem = m - fl
    if rem > F(1, 2) or (rem == F(1, 2) and fl % 2 == 1):
        fl += 1
    return sgn * fl * quantum


def rint_even(v: F) -> int:
    fl = v.numerator // v.denominator
    rem = v - fl
    if rem > F(1, 2) or (rem == F(1, 2) and fl % 2 == 1):
        fl += 1
    return fl


def to_bf16(v: float) -> F:
    b = int(np.float32(v).view(np.uint32))
    b = ((b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000) & 0xFFFFFFFF
    return F(float(np.uint32(b).view(np.float32)))


def to_f16(v: float) -> F:
    return F(float(np.float16(v)))


def quotient_via_reciprocal(x: F, s: F) -> F:
    z = rn32(1 / s)
    y = rn32(x * z)
    r = rn32(x - y * s)
    return rn32(y + r * z)


def test_branch_free_rounding_equals_ieee_quotient_on_near_ties():
    inv127 = rn32(F(1, 127))
    rng = random.Random(7)
    checked = 0
    for trial in range(300):
        rnd = to_bf16 if trial % 2 == 0 else to_f16
        amax = max(rnd(abs(rng.gauss(0, 1)) * 3 * 2.0 ** rng.randint(-6, 6)), rn32(F(1, 10 ** 4)))
        s = rn32(amax * inv127)
        for ue8m0 in (False, True):
            ss = F(2) ** math.ceil(float(np.float32(math.log2(float(s))))) if ue8m0 else s
            cands = [amax, -amax]
            for _ in range(6):
                k = rng.randint(-127, 126)
                x0 = rnd(float((F(k) + F(1, 2)) * ss))
                b = int(np.float32(float(x0)).view(np.uint32))
                cands += [x0] + [F(float(np.uint32(b + d).view(np.float32))) for d in (-1, 1)]
            for j in (2, 254):
                cands.append(rnd(float(amax * 3 / j)))
            for x in cands:
                if abs(x) > amax:
                    continue
                q = quotient_via_reciprocal(x, ss)
                ref = rn32(x / ss)
                assert q == ref, (float(x), float(ss))
                assert rint_even(q) == rint_even(ref)
                checked += 1
    assert checked > 3000
