"""The BASELINE configurations' fixtures on the CPU: config 1's seeded draws pack to the bytes the fixture was made
from, its routing and its oracle decode are the fixture's, and the oracle agrees with the reference's own CPU int8
path on it (golden.npz, made from the reference). Config 4's routing is Zipf-skewed as the config asks. The CPU
port bench.py times as config 1's CPU baseline gives the reference's output bit for bit."""
import numpy as np
import pytest
import torch

import config_data as cd
import gpu_data as gd
from conftest import ROOT
from oracle import moe


@pytest.fixture(scope="module")
def fixture():
    return dict(np.load(ROOT / "tests" / "golden" / "configs.npz"))


@pytest.fixture(scope="module")
def config1():
    d = cd.draw(1)
    return d, cd.pack("int8", d)


def test_config1_draws_routing_and_oracle(fixture, golden, config1):
    d, banks = config1
    assert cd.bank_hash(banks) == bytes(fixture["c1_int8_hash"]).hex()
    np.testing.assert_array_equal(cd.logits(d), fixture["c1_logits"])
    ids, w = cd.routing(1, d)
    np.testing.assert_array_equal(ids, fixture["c1_ids"])
    np.testing.assert_array_equal(w, fixture["c1_w"])
    out = moe.moe_decode("int8", d["x"].float().numpy(), ids, w, tuple(gd.to_np_bank(b) for b in banks))
    np.testing.assert_array_equal(out, fixture["c1_int8_M1"])
    # the reference's CPU path keeps the rotated row and the scales in bf16: within that rounding of the oracle
    ref = golden["c1_ref_cpu_out"].astype(np.float64)
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) <= 1e-2


def test_config4_routing_is_zipf_skewed(fixture):
    counts = fixture["c4_counts"]
    assert counts.sum() == 2048 * cd.TOP_K
    assert counts.max() > 1000 and np.median(counts) < 32  # a few experts take most rows
    assert all(len(set(row)) == cd.TOP_K for row in fixture["c4_ids"].tolist())


def test_cpu_int8_port_is_the_reference_cpu_path(golden, config1):
    """oracle/cpu_port.int8_decode_row (bench.py's config-1 CPU baseline) gives the reference's own CPU int8 decode
    of config 1 bit for bit (golden.npz c1_ref_cpu_out, made by the reference's experts_on_cpu)."""
    from oracle import cpu_port
    d, (gu, dn) = config1
    ids, w = cd.routing(1, d)
    E, I, H = cd.E, cd.I, cd.H
    out = cpu_port.int8_decode_row(d["x"], torch.from_numpy(ids[0]), torch.from_numpy(w[0]),
                                   gu["_qdata"].view(E, 2 * I, H), gu["scale"].view(E, 2 * I),
                                   dn["_qdata"].view(E, H, I), dn["scale"].view(E, H), cpu_port.hadamard())
    np.testing.assert_array_equal(out.to(torch.bfloat16).float().numpy(), golden["c1_ref_cpu_out"])
