"""The torch.library custom ops (drama3_b200.ops) on the GPU: each op returns what the kernels function it wraps
returns on the same inputs, bit for bit (the same launch behind both)."""
import pytest
import torch

import gpu_data as gd
from drama3_b200 import kernels, ops  # noqa: F401  (ops registers torch.ops.drama3_b200)

pytestmark = pytest.mark.gpu
H, I, E = 2048, 768, 32


def test_route_and_plan_ops_equal_the_kernels(cuda):
    logits = torch.randn((16, 128), generator=torch.Generator().manual_seed(1)).to(torch.bfloat16).to(cuda)
    ids, w = torch.ops.drama3_b200.route(logits, 8)
    rid, rw = kernels.route(logits, 8)
    assert torch.equal(ids, rid) and torch.equal(w, rw)
    topk = torch.randint(0, 64, (300, 8), generator=torch.Generator().manual_seed(2)).to(cuda)
    for a, b in zip(torch.ops.drama3_b200.prefill_plan(topk, 64), kernels.prefill_plan(topk, 64)):
        assert torch.equal(a, b)


@pytest.mark.parametrize("kind", ["fp8c", "w4a8"])
def test_moe_decode_op_equals_the_kernel(cuda, kind):
    gu, dn = gd.rand_bank(kind, E, 2 * I, H, 300, cuda), gd.rand_bank(kind, E, H, I, 301, cuda)
    x = gd.rand_rows(4, H, 302, cuda)
    ids, w = gd.rand_routing(4, E, 8, 303, cuda)
    key = "weight" if kind == "fp8c" else "_qdata"
    got = torch.ops.drama3_b200.moe_decode(kind, x, ids, w, gu[key], gu["scale"], None, dn[key], dn["scale"], None)
    assert torch.equal(got, kernels.moe_decode(kind, x, ids, w, (gu, dn)))
