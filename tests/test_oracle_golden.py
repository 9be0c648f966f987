"""The CPU oracle pinned against golden vectors from the reference's own CPU functions (tests/golden/make_golden.py).
CPU only."""
import numpy as np

from oracle import moe


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_hadamard_matches_reference_rotation(golden):
    # the kernels' butterfly (oracle.rotate) against the reference's x @ hadamard(256)
    out = moe.rotate(golden["rot_in"])
    assert rel(out, golden["rot_out"]) < 1e-6
    np.testing.assert_allclose(moe.hadamard(256) @ moe.hadamard(256), np.eye(256), atol=1e-12)


def test_fp8_dequant_bit_exact(golden):
    out = moe.dequant_fp8(golden["dq_w"], golden["dq_s"]).astype(np.float32)
    np.testing.assert_array_equal(out, golden["dq_out"])


def test_e4m3_round_trip():
    vals = moe.E4M3[np.r_[0:0x7F, 0x80:0xFF]]
    codes = moe.f32_to_e4m3(vals)
    np.testing.assert_array_equal(moe.E4M3[codes], vals)


def _fp8_banks(golden):
    gu = {"weight": golden["fp8_gu_w"].reshape(-1, golden["fp8_gu_w"].shape[-1]),
          "scale": golden["fp8_gu_s"].reshape(-1, golden["fp8_gu_s"].shape[-1])}
    dn = {"weight": golden["fp8_dn_w"].reshape(-1, golden["fp8_dn_w"].shape[-1]),
          "scale": golden["fp8_dn_s"].reshape(-1, golden["fp8_dn_s"].shape[-1])}
    return gu, dn


def test_fp8_decode_matches_reference_cpu_path(golden):
    out = moe.moe_decode("fp8", golden["fp8_decode_x"], golden["fp8_decode_ids"], golden["fp8_decode_w"],
                         _fp8_banks(golden))
    # the reference's fp32 CPU path (experts_decode) does not round to bf16 at the end; the kernel path does
    assert rel(out, golden["fp8_decode_out"]) < 4e-3
    assert rel(out, moe.bf16_round(golden["fp8_decode_out"])) < 1e-5


def test_fp8_prefill_matches_reference_cpu_path(golden):
    out = moe.resident_prefill("fp8", golden["fp8_prefill_x"], golden["fp8_prefill_ids"], golden["fp8_prefill_w"],
                               _fp8_banks(golden))
    assert rel(out, golden["fp8_prefill_out"]) < 4e-3


def test_int8_convrot_matches_reference_cpu_experts(golden):
    # experts_on_cpu runs bf16 activations through torch._weight_int8pack_mm; the kernels run fp32 activations:
    # agreement to bf16 precision
    gu = {"_qdata": golden["int8_gu_q"], "scale": golden["int8_gu_s"].reshape(-1)}
    dn = {"_qdata": golden["int8_dn_q"], "scale": golden["int8_dn_s"].reshape(-1)}
    x, ids = golden["int8_cpu_x"], golden["int8_cpu_ids"]
    n1, n2 = gu["_qdata"].shape[0] // 4, dn["_qdata"].shape[0] // 4
    plan = np.stack([ids, np.zeros_like(ids)], axis=-1)
    outs = []
    for t, e in enumerate(ids):
        h = moe.gemv("int8", x[t:t + 1], [e], plan[t:t + 1], gu, gu, n1)
        outs.append(moe.gemv("int8", moe.rotate(h, swiglu=True), [e], plan[t:t + 1], dn, dn, n2)[0])
    assert rel(np.stack(outs), golden["int8_cpu_out"]) < 2e-2


def test_prefill_routing_matches_reference_expression(golden):
    # torch.topk orders equal logits arbitrarily, the reference kernel by index: compare rows whose top 9 logits
    # are distinct (bf16 logits tie often), and the tied rows as sets
    ids, w = moe.route_prefill(golden["route_logits"], 8)
    dids, dw = moe.route(golden["route_logits"], 8)
    v = moe.bf16_to_f32(golden["route_logits"])
    exact = 0
    for r in range(len(ids)):
        top = np.sort(v[r])[::-1][:9]
        if len(set(top.tolist())) == 9:
            exact += 1
            np.testing.assert_array_equal(ids[r], golden["route_ids"][r])
            np.testing.assert_array_equal(dids[r], golden["route_ids"][r])
            np.testing.assert_allclose(w[r], golden["route_w"][r], rtol=0, atol=2 ** -8)
            np.testing.assert_allclose(dw[r], golden["route_w"][r], rtol=0, atol=2 ** -7)
        else:
            assert np.sort(v[r][ids[r]]).tolist() == np.sort(v[r][golden["route_ids"][r]]).tolist()
    assert exact >= len(ids) // 2


def test_codes_pack_decode_round_trip():
    rng = np.random.default_rng(3)
    w = (rng.standard_normal((32, 512)) * 0.02).astype(np.float32)
    for bits in (4, 6):
        q, g, c = moe.quantize_codes(w, bits)
        assert q.shape == (32, 512 * bits // 8) and g.shape == (32, 32)
        dec = moe.decode_codes(q, g, 512, bits, moe.CODEBOOK4)
        back = dec.astype(np.float64) * c[:, None]
        err = rel(back, moe.convrot_weight(w))
        assert err < (0.2 if bits == 4 else 0.05), err


def test_resolve_invariants():
    st = moe.new_state(layers=4, experts=16, count=10)
    rng = np.random.default_rng(5)
    for step in range(40):
        for layer in range(4):
            ids = rng.choice(16, size=4, replace=False)
            plan = moe.resolve(st, ids, layer, 4, 16, 128.0, 0, 6.0)
            for e, (slot, code) in zip(ids, plan):
                key = layer * 16 + e
                assert code in (0, 1)
                if slot >= 0:
                    assert st["owner"][slot] == key and st["table"][key] == slot
    # table and owner agree everywhere
    for slot, key in enumerate(st["owner"]):
        if key >= 0:
            assert st["table"][key] == slot
    assert int(st["reads"].sum()) == 40 * 4 * 4


def test_cpu_baseline_port_equals_reference_cpu_forward(golden):
    """The CPU baseline's torch port (oracle/cpu_port.py) on the golden decode row: bit for bit the reference's own
    FP8Experts CPU forward (drama3/offload.py:771-784) in fp32."""
    import torch
    from oracle import cpu_port
    t = {k: torch.from_numpy(golden[k]) for k in ("fp8_decode_x", "fp8_decode_ids", "fp8_decode_w", "fp8_gu_w",
                                                   "fp8_gu_s", "fp8_dn_w", "fp8_dn_s")}
    out = cpu_port.fp8_decode_lines(t["fp8_decode_x"], t["fp8_decode_ids"], t["fp8_decode_w"], t["fp8_gu_w"],
                                    t["fp8_gu_s"], t["fp8_dn_w"], t["fp8_dn_s"], dtype=torch.float32)
    np.testing.assert_array_equal(out.numpy(), golden["fp8_decode_out"])
