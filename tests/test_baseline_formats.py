"""The BASELINE layouts' packers, quantizers and oracle arithmetic on the CPU (no reference implementation exists
for them: the tests pin the restatement's own invariants)."""
import numpy as np
import pytest

from oracle import moe


@pytest.mark.parametrize("bits", [4, 6])
def test_pack_unpack_roundtrip_bit_exact(bits):
    rng = np.random.default_rng(bits)
    lim = 8 if bits == 4 else 32
    q = rng.integers(-lim, lim, size=(37, 256))
    packed = moe.pack_int4(q) if bits == 4 else moe.pack_int6(q)
    assert packed.shape == (37, 256 * bits // 8) and packed.dtype == np.uint8
    back = moe.unpack_int4(packed, 256) if bits == 4 else moe.unpack_int6(packed, 256)
    np.testing.assert_array_equal(back, q)
    # and bytes -> values -> bytes
    again = moe.pack_int4(back) if bits == 4 else moe.pack_int6(back)
    np.testing.assert_array_equal(again, packed)


def test_pack_layouts_documented():
    """Low nibble = even column; four 6-bit values per three bytes, little endian, two's complement."""
    assert moe.pack_int4(np.array([[1, -2]]))[0, 0] == (1 | (0xE << 4))
    assert list(moe.pack_int6(np.array([[1, -1, 2, -32]]))[0]) == [
        (1 | (63 << 6)) & 0xFF, ((1 | (63 << 6) | (2 << 12)) >> 8) & 0xFF, ((2 << 12 | 32 << 18) >> 16) & 0xFF]


def test_quantize_rows_int8():
    x = np.array([[0.0, 0.0], [1.0, -0.5], [254.0, 1.0]], np.float32)
    q, s = moe.quantize_rows_int8(x)
    np.testing.assert_array_equal(q, [[0, 0], [127, -64], [127, 0]])  # -63.5 rounds half-even to -64
    np.testing.assert_allclose(s, [0.0, 1 / 127, 2.0], rtol=1e-7)


@pytest.mark.parametrize("kind", ["w4a8", "w6a8"])
def test_wa8_quantizer_and_gemm(kind):
    rng = np.random.default_rng(7)
    w = rng.normal(0, 0.02, size=(2, 64, 256)).astype(np.float32)
    bank = moe.make_baseline_bank(kind, w)
    qmax = 7 if kind == "w4a8" else 31
    codes = moe.wa8_codes(kind, bank, 0, 128, 256)
    assert codes.min() >= -qmax and codes.max() <= qmax and np.abs(codes).max() == qmax
    x = rng.normal(size=(3, 256)).astype(np.float32)
    got = moe.gemm_wa8(kind, x, bank, 64, 64)
    # the same integers and scales through float64 matmuls
    q, s = moe.quantize_rows_int8(x)
    gs = moe.bf16_to_f32(bank["scale"][64:128]).astype(np.float64)
    wd = codes[64:].astype(np.float64) * np.repeat(gs, 128, axis=1)
    want = (q.astype(np.float64) * s[:, None]) @ wd.T
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
    # close to the unquantized product (4-bit / 6-bit weights, 8-bit activations)
    exact = x.astype(np.float64) @ w[1].T.astype(np.float64)
    rel = np.linalg.norm(got - exact) / np.linalg.norm(exact)
    assert rel < (0.2 if kind == "w4a8" else 0.05)


def test_fp8_channel_quantizer():
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.02, size=(128, 256)).astype(np.float32)
    q, s = moe.quantize_fp8_channel(w)
    d = moe.dequant_fp8_channel(q, s)
    assert np.abs(moe.e4m3_to_f32(q)).max() <= 448.0
    assert np.linalg.norm(d - w) / np.linalg.norm(w) < 0.05
