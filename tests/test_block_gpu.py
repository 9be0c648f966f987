"""The MoE block's router and shared expert on the GPU (drama3/model.py:40-47,107-123): kernels.router (the gate
linear and the decode routing in one launch) and kernels.shared_expert (the sigmoid-gated shared expert added into
the experts' output in two launches), against a float64 restatement of the reference's bf16 chain (each linear's
output, silu, the product, the sigmoid, the gated product and the add rounded to bf16 where the bf16 modules round),
against torch's own bf16 modules, and the whole block fused against the block on torch's chain."""
import pytest
import torch

import gpu_data as gd
from drama3_b200 import kernels
from drama3_b200.model import SparseMoeBlock, block_config

pytestmark = pytest.mark.gpu
H, E, IS = 2048, 128, 512


def bf(t):
    return t.to(torch.bfloat16).double()


def rand(shape, seed, std=0.02):
    return (torch.randn(shape, generator=torch.Generator().manual_seed(seed)) * std).to(torch.bfloat16)


@pytest.mark.parametrize("M", [1, 4, 16])
def test_router_logits_and_routing(cuda, M):
    """Logits within one bf16 step of bf16(x W^T) computed in float64 (most equal); ids and weights are route()'s on
    the router's own logits, bit for bit, and route()'s on the float64 logits for every row whose logits agree."""
    x = rand((M, H), 500 + M, std=1.0).to(cuda)
    w = rand((E, H), 510 + M).to(cuda)
    ids, wt, lg = kernels.router(x, w, 8, logits=True)
    exact = (x.double() @ w.double().T).to(torch.bfloat16)
    step = (exact.float().abs() * 2.0 ** -7).clamp_min(2.0 ** -133)
    diff = (lg.float() - exact.float()).abs()
    assert bool((diff <= step * 1.0001).all())
    assert float((lg != exact).float().mean()) < 0.02
    rid, rw = kernels.route(lg, 8)
    assert torch.equal(ids, rid) and torch.equal(wt, rw)
    eid, ew = kernels.route(exact, 8)
    same = (lg == exact).all(dim=1)
    assert torch.equal(ids[same], eid[same]) and torch.equal(wt[same], ew[same])


def shared_oracle(x, gu, dn, g, out):
    """The reference's bf16 chain in float64 with its bf16 roundings."""
    h = bf(x.double() @ gu.double().T)
    I = dn.shape[1]
    gate, up = h[:, :I], h[:, I:]
    a = bf(bf(gate / (1 + torch.exp(-gate))) * up)
    d = bf(a @ dn.double().T)
    s = bf(1 / (1 + torch.exp(-bf(x.double() @ g.double().reshape(-1, 1)))))
    return bf(out.double() + bf(s * d))


@pytest.mark.parametrize("M", [1, 4, 16])
def test_shared_expert_against_the_bf16_chain(cuda, M):
    x = rand((M, H), 600 + M, std=1.0).to(cuda)
    gu, dn, g = rand((2 * IS, H), 610).to(cuda), rand((H, IS), 611).to(cuda), rand((1, H), 612).to(cuda)
    moe = rand((M, H), 613 + M, std=0.05).to(cuda)
    want = shared_oracle(x, gu, dn, g, moe)
    got = kernels.shared_expert(x, gu, dn, g, moe.clone())
    assert gd.rel_l2(got.float(), want) <= 1e-3
    # torch's bf16 modules (the eager path of the block)
    eager = moe + torch.sigmoid(x @ g.T) * (torch.nn.functional.silu((x @ gu.T)[:, :IS]) * (x @ gu.T)[:, IS:]) @ dn.T
    assert gd.rel_l2(got.float(), eager.float()) <= 1e-2


def test_block_fused_matches_eager(cuda):
    """16 decode lines through SparseMoeBlock: the router and shared-expert kernels against torch's chain for the
    same block; identical routing on this seed, outputs within bf16 rounding of each other."""
    torch.manual_seed(7)
    block = SparseMoeBlock(block_config(num_experts=E, intermediate=768, shared_intermediate=IS,
                                        per_channel=True), device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        for lin in (block.gate, block.shared_expert.gate_up_proj, block.shared_expert.down_proj,
                    block.shared_expert_gate):
            lin.weight.normal_(0, 0.02)
        for name in ("gate_up", "down"):
            bank = gd.rand_bank("fp8c", E, 2 * 768 if name == "gate_up" else H, H if name == "gate_up" else 768,
                                620 if name == "gate_up" else 621, cuda)
            getattr(block.experts, f"{name}_weight").view(torch.uint8).view(-1, bank["weight"].shape[1]).copy_(
                bank["weight"])
            getattr(block.experts, f"{name}_scale").view(-1).copy_(bank["scale"])
        x = gd.rand_rows(16, H, 622, cuda).view(16, 1, H)
        assert block.fused_router(x.view(16, H)) and block.fused_shared(x.view(16, H))
        fused = block(x)
        ids_fused, _ = kernels.router(x.view(16, H), block.gate.weight, 8)
        block.fused = False
        eager = block(x)
        ids_eager, _ = kernels.route(block.gate(x.view(16, H)), 8)
    assert torch.equal(ids_fused, ids_eager)
    assert gd.rel_l2(fused.float(), eager.float()) <= 1e-2
