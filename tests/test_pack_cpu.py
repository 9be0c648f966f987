"""The native packers (csrc/pack.cpp, host code) byte for byte against the oracle's quantizers: the reference's
layouts (oracle.moe.make_bank: fp8 block scales, int8 ConvRot, w4 / w6 codes) and the BASELINE ones
(quantize_fp8_channel, quantize_wa8), on random experts, all-zero rows, blocks and groups, exact ties of the rounding,
saturation, tiny negatives, and several thread splits; plus the relative error of what they pack, the check the
reference's converter prints (tools/convert.py:102-109); and the converter's on-disk expert layout (state-dict keys,
comfy_quant configs, a safetensors round trip)."""
import json

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
        pack.pack_bank("nf4", w)


def same(got, want):
    got, want = np.asarray(got), np.asarray(want)
    return (got.shape == want.shape and got.dtype == want.dtype
            and np.array_equal(got.view(np.uint8), want.view(np.uint8)))


@pytest.mark.parametrize("kind", ["fp8", "int8", "w4", "w6"])
@pytest.mark.parametrize("threads", [1, 3, 0])
def test_reference_layouts_random_experts(kind, threads):
    w = rows((3, 256, 768), 20)
    got = pack.pack_bank(kind, torch.from_numpy(w), threads)
    want = moe.make_bank(kind, w)
    assert sorted(got) == sorted(want)
    for name in want:
        assert same(got[name].numpy(), want[name]), name


@pytest.mark.parametrize("kind", ["fp8", "int8", "w4", "w6"])
def test_reference_layouts_edge_rows(kind):
    """All-zero rows and blocks (scale 1; fp8 code 0, int8 0, w4 the first code of the all-zero candidates, w6 32),
    large and tiny magnitudes in one row, and sign-flipped copies."""
    w = rows((1, 384, 512), 21)
    w[0, :128, :128] = 0.0  # a zero fp8 block
    w[0, 130] = 0.0  # a zero row
    w[0, 131] *= np.float32(1e4)
    w[0, 132, ::7] *= np.float32(1e-6)
    w[0, 200:300] = -w[0, 100:200]
    got = pack.pack_bank(kind, torch.from_numpy(w), 2)
    want = moe.make_bank(kind, w)
    for name in want:
        assert same(got[name].numpy(), want[name]), name
    if kind in ("int8", "w4"):
        assert got["s_channel" if kind == "w4" else "scale"][130] == 1.0 and not got["_qdata"][130].any()
    if kind == "w6":  # code 32 everywhere: nibble plane 0, 2-bit plane 0b10101010
        assert got["s_channel"][130] == 1.0
        assert not got["_qdata"][130, :256].any() and (got["_qdata"][130, 256:] == 0xAA).all()
        assert not moe.decode_codes(got["_qdata"][130].numpy(), got["scale"][130].numpy(), 512, 6, None).any()


def test_w4_custom_codebook_with_equal_candidates():
    """A codebook with repeated and near values: several codes give the same rounded candidate, and the first of equal
    distances wins, as numpy's argmin picks it."""
    book = np.array([-1.0, -1.0, -0.5, -0.25, -0.25, -0.125, 0.0, 0.0, 0.01, 0.125, 0.25, 0.25, 0.5, 0.75, 1.0, 1.0],
                    np.float32)
    w = rows((2, 128, 512), 22)
    got = pack.pack_codes(torch.from_numpy(w), 4, book)
    q, g, c = moe.quantize_codes(w.reshape(-1, 512), 4, book)
    assert same(got["_qdata"].numpy(), q) and same(got["scale"].numpy(), g) and same(got["s_channel"].numpy(), c)


@pytest.mark.parametrize("kind, bound", [("fp8", 0.035), ("int8", 0.01), ("w4", 0.1), ("w6", 0.03), ("fp8c", 0.035),
                                         ("w4a8", 0.15), ("w6a8", 0.035)])
def test_packed_relative_error(kind, bound):
    """What the packers write, decoded by the oracle, against the float rows (in the ConvRot basis where the layout
    has it): the relative Frobenius error the reference's converter reports per layer."""
    K = 512
    w = rows((2, 256, K), 23)
    flat = w.reshape(-1, K)
    fields = {n: v.view(torch.int16).numpy().view(np.uint16) if v.dtype == torch.bfloat16 else v.numpy()
              for n, v in pack.pack_bank(kind, torch.from_numpy(w)).items()}
    if kind in ("fp8", "int8", "w4", "w6"):
        back = moe.expert_rows(kind, fields, 0, flat.shape[0], K, moe.CODEBOOK4)
        ref = flat.astype(np.float64) if kind == "fp8" else moe.convrot_weight(flat)
    elif kind == "fp8c":
        back, ref = moe.dequant_fp8_channel(fields["weight"], fields["scale"]), flat.astype(np.float64)
    else:
        codes = moe.wa8_codes(kind, fields, 0, flat.shape[0], K).astype(np.float64)
        scale = np.repeat(moe.bf16_to_f32(fields["scale"]).astype(np.float64), 128, axis=1)
        back, ref = codes * scale, flat.astype(np.float64)
    err = np.linalg.norm(back - ref) / np.linalg.norm(ref)
    assert 0 < err < bound


def test_reference_layout_bad_arguments_raise():
    with pytest.raises(_lib.D3Error):
        pack.pack_fp8_blocks(torch.zeros((100, 256)))  # rows not a multiple of 128
    with pytest.raises(_lib.D3Error):
        pack.pack_int8_convrot(torch.zeros((4, 384)))  # K not a multiple of 256
    with pytest.raises(ValueError):
        pack.pack_codes(torch.zeros((4, 256)), 4, codebook=[0.0] * 8)


@pytest.mark.parametrize("kind", ["fp8", "int8", "w4", "w6"])
def test_expert_state_layout_and_round_trip(kind, tmp_path):
    """One layer through the converter's state-dict layout (keys, shapes, dtypes, comfy_quant JSON), a safetensors
    file and back to flat banks equal to pack_bank's."""
    from safetensors.torch import load_file, save_file
    E, H, I = 4, 512, 256
    gu = torch.from_numpy(rows((E, 2 * I, H), 30))
    dn = torch.from_numpy(rows((E, H, I), 31))
    state = pack.expert_state(kind, 7, gu, dn, threads=2)
    if kind == "fp8":
        assert state["model.layers.7.mlp.experts.gate_up_weight"].dtype == torch.float8_e4m3fn
        assert state["model.layers.7.mlp.experts.gate_up_weight"].shape == (E, 2 * I, H)
        assert state["model.layers.7.mlp.experts.down_scale"].shape == (E, H // 128, I // 128)
    else:
        mod = "model.layers.7.mlp.experts.down_proj"
        conf = json.loads(bytes(state[f"{mod}.comfy_quant"].tolist()).decode())
        assert conf["num_experts"] == E and conf["convrot_groupsize"] == 256
        if kind == "int8":
            assert conf["format"] == "int8_tensorwise" and conf["convrot"] is True
            assert state[f"{mod}.weight"].shape == (E, H, I) and state[f"{mod}.weight_scale"].shape == (E, H, 1)
        else:
            bits = int(kind[1])
            assert conf == {"format": "asym_w4a8_int8" if bits == 4 else "w6a8_int8", "group_size": 16,
                            "convrot_groupsize": 256, "num_experts": E}
            assert state[f"{mod}.weight"].shape == (E, H, I * bits // 8)
            assert state[f"{mod}.weight_s_rel"].shape == (E, H, I // 16)
            assert state[f"{mod}.weight_s_channel"].shape == (E, H)
            assert (f"{mod}.weight_codebook" in state) == (bits == 4)
    path = tmp_path / "experts.safetensors"
    save_file(state, str(path), metadata={"drama3_format": pack.DRAMA3_FORMAT[kind]})
    back = load_file(str(path))
    gu_f, dn_f, books = pack.banks_from_state(kind, back, 7)
    for fields, w in ((gu_f, gu), (dn_f, dn)):
        want = pack.pack_bank(kind, w)
        assert sorted(fields) == sorted(want)
        for name in want:
            assert torch.equal(fields[name], want[name]), name
    if kind == "w4":
        assert all(torch.equal(b, torch.tensor(pack.CODEBOOK4)) for b in books)
    else:
        assert books == (None, None)


def test_banks_from_state_rejects_another_layout():
    state = pack.expert_state("w6", 0, torch.zeros((1, 256, 256)), torch.zeros((1, 256, 256)))
    with pytest.raises(ValueError):
        pack.banks_from_state("w4", state, 0)


def _draw_rows(data, rows, K):
    """Rows with a drawn distribution: a scale of 1e-20 .. 1e20, normal / uniform / heavy-tailed values, some rows and
    columns zeroed, and integer-valued entries (which land on rounding ties)."""
    from hypothesis import strategies as st
    seed = data.draw(st.integers(0, 2 ** 32 - 1))
    rng = np.random.default_rng(seed)
    scale = 10.0 ** data.draw(st.integers(-20, 20))
    shape = data.draw(st.sampled_from(["normal", "uniform", "cauchy", "ints"]))
    if shape == "normal":
        w = rng.normal(size=(rows, K))
    elif shape == "uniform":
        w = rng.uniform(-1, 1, size=(rows, K))
    elif shape == "cauchy":
        w = np.clip(rng.standard_cauchy(size=(rows, K)), -1e6, 1e6)
    else:
        w = rng.integers(-64, 65, size=(rows, K)).astype(np.float64) / 2
        scale = 1.0
    w = (w * scale).astype(np.float32)
    w[rng.random(rows) < 0.1] = 0.0
    w[:, rng.random(K) < 0.05] = 0.0
    return w


def test_packers_property_against_oracle():
    """Drawn rows through every packer, byte for byte against the oracle (hypothesis, 40 draws, the same every run)."""
    from hypothesis import HealthCheck, given, settings
    from hypothesis import strategies as st

    @settings(max_examples=40, deadline=None, derandomize=True, suppress_health_check=[HealthCheck.too_slow])
    @given(st.data())
    def check(data):
        kind = data.draw(st.sampled_from(["fp8", "int8", "w4", "w6", "fp8c", "w4a8", "w6a8"]))
        K = data.draw(st.sampled_from([256, 512]))
        rows_ = 128 * data.draw(st.integers(1, 2))
        w = _draw_rows(data, rows_, K)
        got = pack.pack_bank(kind, torch.from_numpy(w), threads=data.draw(st.integers(0, 3)))
        with np.errstate(over="ignore", invalid="ignore"):
            if kind in ("fp8", "int8", "w4", "w6"):
                want = moe.make_bank(kind, w[None])
            elif kind == "fp8c":
                c, s = moe.quantize_fp8_channel(w)
                want = {"weight": c, "scale": s}
            else:
                q, s = moe.quantize_wa8(w, int(kind[1]))
                want = {"_qdata": q, "scale": s}
        for name in want:
            g = got[name]
            g = g.view(torch.int16).numpy().view(np.uint16) if g.dtype == torch.bfloat16 else g.numpy()
            assert same(g, want[name]), (kind, name)

    check()


@pytest.mark.parametrize("kind", ["int8", "w4", "w6"])
def test_packed_weight_is_recognized_as_a_kernel_bank(kind):
    """A packed bank dressed as a quantized tensor is what offload.kernel_bank recognizes, with pack_bank's fields;
    the host bank of the slot cache takes it as well."""
    from drama3_b200 import offload
    w = torch.from_numpy(rows((4, 64, 512), 40))
    weight = pack.packed_weight(kind, w, threads=2)
    found = offload.kernel_bank(weight)
    assert found is not None and found[0] == kind
    want = pack.pack_bank(kind, w)
    assert set(found[1]) == set(want)
    for name in want:
        assert torch.equal(found[1][name].reshape(want[name].shape), want[name]), name
    bank = offload.QuantHostBank(type("M", (), {"weight": weight, "num_experts": 4})(), pin=False)
    assert bank.kernel == kind and bank.rows("_qdata") == 64
    assert weight.to("cpu")._qdata.data_ptr() != 0
    with pytest.raises(ValueError):
        pack.packed_weight("fp8c", w)
