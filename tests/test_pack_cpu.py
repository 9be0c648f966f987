"""The native packers (d3_pack_fp8c, d3_pack_wa8 in csrc/pack.cpp, host code) byte for byte against the oracle's
quantizers (oracle.moe.quantize_fp8_channel, quantize_wa8): random experts, all-zero rows and groups, exact ties of
the rounding, saturation, tiny negatives, and several thread splits."""
import numpy as np
import pytest
import torch

from drama3_b200 import _lib, pack
from oracle import moe

E4M3_POS = moe.E4M3[:0x7F]


def rows(shape, seed):
    return np.random.default_rng(seed).normal(scale=0.05, size=shape).astype(np.float32)


@pytest.mark.parametrize("threads", [1, 3, 0])
def test_fp8c_random_experts(threads):
    w = rows((6, 96, 512), 1)
    got = pack.pack_fp8c(torch.from_numpy(w), threads)
    codes, scale = moe.quantize_fp8_channel(w.reshape(-1, 512))
    assert np.array_equal(got["weight"].numpy(), codes)
    assert np.array_equal(got["scale"].numpy().view(np.uint32), scale.view(np.uint32))


def test_fp8c_edge_rows():
    K = 256
    w = np.zeros((6, K), np.float32)  # row 0 all zero: scale 1, codes 0
    # row 1: absmax 448 (scale exactly 1) and every midpoint between neighbouring e4m3 values: ties to the even code
    mids = ((E4M3_POS[:-1].astype(np.float64) + E4M3_POS[1:]) / 2).astype(np.float32)
    w[1, :126] = mids
    w[1, 126:252] = -mids
    w[1, 255] = 448.0
    # row 2: values just off the midpoints, and a negative value far below the smallest e4m3 (-0 -> 0x80)
    w[2, :126] = np.nextafter(mids, np.float32(np.inf))
    w[2, 126:252] = np.nextafter(mids, np.float32(0))
    w[2, 252] = 448.0
    w[2, 253] = -1e-6
    w[2, 254] = -0.0
    # row 3: a row whose absmax / 448 rounds so that max / scale lands above 448 (saturation); rows 4, 5 random
    w[3] = np.linspace(-1.0, 1.0, K, dtype=np.float32) * np.float32(3.3)
    w[4:] = rows((2, K), 2) * np.float32(1e-30)  # scales in the float32 subnormal range
    got = pack.pack_fp8c(torch.from_numpy(w), 2)
    codes, scale = moe.quantize_fp8_channel(w)
    assert np.array_equal(got["weight"].numpy(), codes)
    assert np.array_equal(got["scale"].numpy().view(np.uint32), scale.view(np.uint32))
    assert got["scale"][0] == 1.0 and not got["weight"][0].any()
    assert got["weight"][2, 253] == 0x80 and got["weight"][2, 254] == 0x00


def test_fp8c_float32_sweep():
    """Every 997th float32 bit pattern in [0, 480), both signs, at scale 1 (a 448 leads each row): the bit-arithmetic
    rounding of the packer against the oracle's nearest-table search."""
    a = np.arange(0, 0x43F00000, 997, dtype=np.uint32).view(np.float32)
    a = np.concatenate([a, -a])
    a = a[:a.size // 255 * 255].reshape(-1, 255)
    w = np.empty((a.shape[0], 256), np.float32)
    w[:, 0], w[:, 1:] = 448.0, a
    got = pack.pack_fp8c(torch.from_numpy(w))
    codes, _ = moe.quantize_fp8_channel(w)
    assert np.array_equal(got["weight"].numpy(), codes)


@pytest.mark.parametrize("bits", [4, 6])
@pytest.mark.parametrize("threads", [1, 5, 0])
def test_wa8_random_experts(bits, threads):
    w = rows((4, 80, 768), 3 + bits)
    got = pack.pack_wa8(torch.from_numpy(w), bits, threads)
    packed, s_bits = moe.quantize_wa8(w.reshape(-1, 768), bits)
    assert np.array_equal(got["_qdata"].numpy(), packed)
    assert np.array_equal(got["scale"].view(torch.int16).numpy().view(np.uint16), s_bits)
    assert got["scale"].dtype == torch.bfloat16 and got["_qdata"].shape == (320, 768 * bits // 8)


@pytest.mark.parametrize("bits", [4, 6])
def test_wa8_edge_groups(bits):
    qmax = 7 if bits == 4 else 31
    w = rows((3, 512), 9)
    w[0, 128:256] = 0.0  # an all-zero group: scale 1, codes 0
    # group 2 of row 0: absmax qmax (scale exactly 1) and exact half-way quotients: ties to even
    half = np.arange(-qmax, qmax, dtype=np.float32) + np.float32(0.5)
    w[0, 256:384] = 0.0
    w[0, 256:256 + half.size] = half
    w[0, 383] = qmax
    w[1] = -w[1]  # negative codes in every position of a packed word
    w[2, :128] = np.float32(1e-38)  # a subnormal-range group
    got = pack.pack_wa8(torch.from_numpy(w), bits, 2)
    packed, s_bits = moe.quantize_wa8(w, bits)
    assert np.array_equal(got["_qdata"].numpy(), packed)
    assert np.array_equal(got["scale"].view(torch.int16).numpy().view(np.uint16), s_bits)
    codes = moe.unpack_int4(packed, 512) if bits == 4 else moe.unpack_int6(packed, 512)
    assert not codes[0, 128:256].any()
    want = np.rint(half).astype(int)  # half to even: -6.5 -> -6, 0.5 -> 0, 1.5 -> 2
    assert codes[0, 256:256 + half.size].tolist() == want.tolist()


def test_bad_arguments_raise():
    w = torch.zeros((4, 200))
    with pytest.raises(_lib.D3Error):
        pack.pack_wa8(w, 4)  # K not a multiple of 128
    with pytest.raises(_lib.D3Error):
        pack.pack_wa8(torch.zeros((4, 256)), 5)
    with pytest.raises(ValueError):
        pack.pack_bank("fp8", w)
