"""The int8 expansion of W4A8 / W6A8 weight codes in the prompt pass's kind::i8 GEMM (csrc/grouped_mma.cuh,
gm_convert_i8), restated with the same 32-bit word operations: every int6 code becomes the int8 byte 4 x code and
every int4 code the byte 16 x code, in column order, so the s32 sums are exact multiples of the codes' sums
(gm_i8_unscale divides by 4 or 16 in the fold). Codes are two's complement: int6 in -32..31 (stored -31..31), int4
in -8..7; W6A8 packs four codes per 24 bits, code i at bit 6 i of a little-endian group; W4A8 packs column 2 i in
the low nibble of byte i and column 2 i + 1 in its high nibble (oracle.moe's packers)."""
import numpy as np

M32 = 0xFFFFFFFF


def funnelshift_r(lo, hi, s):
    """CUDA __funnelshift_r: the low 32 bits of (hi:lo) >> s, s in 0..31."""
    return ((((hi & M32) << 32) | (lo & M32)) >> s) & M32


def byte_perm(x, y, sel):
    """CUDA __byte_perm: byte n of the result is byte (sel >> 4n) & 7 of the 8-byte value (y:x)."""
    b = [(x >> (8 * i)) & 0xFF for i in range(4)] + [(y >> (8 * i)) & 0xFF for i in range(4)]
    return sum(b[(sel >> (4 * n)) & 7] << (8 * n) for n in range(4))


def six_bit_group_to_int8(t):
    """Four 6-bit codes in bits 0..23 of t -> four bytes, each the code times 4 (the kernel's shifts and masks)."""
    return (((t << 2) & 0xFC) | ((t << 4) & 0xFC00) | ((t << 6) & 0xFC0000) | ((t << 8) & 0xFC000000)) & M32


def s8(b):
    return b - 256 if b >= 128 else b


def test_int6_codes_expand_to_four_times_the_code():
    rng = np.random.default_rng(0)
    for _ in range(2000):
        codes = rng.integers(-32, 32, 16)
        bits = sum((int(c) & 63) << (6 * i) for i, c in enumerate(codes))  # 96 bits, code i at bit 6 i
        w0, w1, w2 = bits & M32, (bits >> 32) & M32, (bits >> 64) & M32
        groups = [w0, funnelshift_r(w0, w1, 24), funnelshift_r(w1, w2, 16), w2 >> 8]
        out = []
        for t in groups:
            o = six_bit_group_to_int8(t)
            out += [s8((o >> (8 * i)) & 0xFF) for i in range(4)]
        assert out == [4 * int(c) for c in codes]


def test_int4_codes_expand_to_sixteen_times_the_code_in_column_order():
    rng = np.random.default_rng(1)
    for _ in range(2000):
        codes = rng.integers(-8, 8, 8)  # columns 0..7 of one 32-bit word
        w = sum(((int(codes[2 * i]) & 15) | ((int(codes[2 * i + 1]) & 15) << 4)) << (8 * i) for i in range(4))
        lo, hi = (w << 4) & 0xF0F0F0F0, w & 0xF0F0F0F0
        out = []
        for o in (byte_perm(lo, hi, 0x5140), byte_perm(lo, hi, 0x7362)):
            out += [s8((o >> (8 * i)) & 0xFF) for i in range(4)]
        assert out == [16 * int(c) for c in codes]


def test_group_sums_fit_the_float_mantissa():
    """The largest |s32| partial of a 128-column group, |code| x 4 (or 16) x 127 x 128, is below 2^24: exact as a
    float, so folding the partial with the group scale loses nothing the f16 form kept."""
    assert 32 * 4 * 127 * 128 < 2 ** 24 and 8 * 16 * 127 * 128 < 2 ** 24
