"""The int8 activation quantization of the W4A8 / W6A8 kernels (quant_i8_n in csrc/common.cuh) in exact rational
arithmetic: q = rint(y') with r = fl(1 / s), y = fl(x r), y' = fl(fl(x - y s) r + y) (two fused multiply-adds, one
rounding each) equals rint(fl(x / s)), the oracle's IEEE-division form (oracle.moe.quantize_rows_int8), on bf16 rows
with half-way quotients among them; rounding fl(x r) alone does not always."""
from fractions import Fraction

import numpy as np

from oracle import moe


def f32(q):
    """q (Fraction, normal float32 range) rounded to the nearest float32, ties to even."""
    if q == 0:
        return Fraction(0)
    sign = -1 if q < 0 else 1
    a = abs(q)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while Fraction(2) ** e > a:
        e -= 1
    while Fraction(2) ** (e + 1) <= a:
        e += 1
    scale = Fraction(2) ** (e - 23)  # a / scale in [2^23, 2^24)
    m = a / scale
    n, rem = divmod(m.numerator, m.denominator)
    frac = Fraction(rem, m.denominator)
    if frac > Fraction(1, 2) or (frac == Fraction(1, 2) and n % 2 == 1):
        n += 1
    return sign * n * scale


def rint(q):
    """Round half to even of a Fraction."""
    n = q.numerator // q.denominator
    frac = q - n
    if frac > Fraction(1, 2) or (frac == Fraction(1, 2) and n % 2 == 1):
        n += 1
    return n


def quant_kernel(x, s):
    r = f32(1 / s)
    y = f32(x * r)
    yq = f32(f32(x - y * s) * r + y)
    return max(-127, min(127, rint(yq))), max(-127, min(127, rint(y)))


def test_reciprocal_and_correction_equal_ieee_division_on_bf16_rows():
    rng = np.random.default_rng(5)
    rows = moe.bf16_round(rng.normal(size=(8, 1024)).astype(np.float32))
    # a row of max 127 * 2^-4 (s exact) holding x = max / 2: x / s = 63.5 exactly, a tie rounded to even
    rows[0, :4] = [127 / 16, 127 / 32, -127 / 32, 1.5 / 16]
    checked = naive_misses = ties = 0
    for row in rows:
        m = Fraction(float(np.abs(row).max()))
        s = f32(m / 127)
        ref_q, _ = moe.quantize_rows_int8(row[None, :])
        for v, want in zip(row, ref_q[0]):
            x = Fraction(float(v))
            got, naive = quant_kernel(x, s)
            exact = f32(x / s)
            assert got == max(-127, min(127, rint(exact))) == int(want)
            ties += exact.denominator == 2
            naive_misses += naive != got
            checked += 1
    assert checked == rows.size and ties > 0
    assert naive_misses < checked // 1000  # the direct form is close, but not equal


def test_tie_at_half_the_maximum():
    """A bf16 row with max 3.515625 holding 1.7578125 (its half): x / s rounds to exactly 63.5, which the oracle rounds
    to 64 (half to even) while fl(x (1 / s)) falls below the tie and rounds to 63; the correction step restores 64."""
    m, x = Fraction(3.515625), Fraction(1.7578125)
    s = f32(m / 127)
    assert f32(x / s) == Fraction(127, 2)
    got, naive = quant_kernel(x, s)
    assert (got, naive) == (64, 63)
    q, _ = moe.quantize_rows_int8(np.array([[3.515625, 1.7578125, -1.7578125]], np.float32))
    assert q[0].tolist() == [127, 64, -64]
