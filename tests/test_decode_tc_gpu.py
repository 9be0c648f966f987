"""The tensor-core decodes (1-16 lines) against the oracle and against the mma.sync decode on the same inputs
(D3_DECODE_TC=0 selects it): per-channel e4m3 rows (tcgen05 kind::f8f6f4, the activations as exact e4m3 terms),
int8 ConvRot rows (kind::i8, the activations rotated while staged and written as three int8 terms) and W4A8
(kind::i8 on int8-expanded int4 codes and int8 activations, group scales folded per 128 columns)."""
import numpy as np
import pytest
import torch

import gpu_data as gd
from drama3_b200 import _lib, ep, kernels

pytestmark = pytest.mark.gpu
H = 2048


def both(monkeypatch, kind, x, ids, w, banks, **kw):
    """(tensor-core decode, mma.sync decode) of the same call."""
    monkeypatch.delenv("D3_DECODE_TC", raising=False)
    tc = kernels.moe_decode(kind, x, ids, w, banks, **kw)
    monkeypatch.setenv("D3_DECODE_TC", "0")
    ref = kernels.moe_decode(kind, x, ids, w, banks, **kw)
    monkeypatch.delenv("D3_DECODE_TC")
    return tc, ref


def oracle(kind, x, ids, w, banks):
    if kind == "int8":
        return gd.oracle_decode(kind, x, ids, w, banks, (None, None), H)
    return gd.baseline_oracle_decode(kind, x, ids, w, banks)


@pytest.mark.parametrize("kind", ["fp8c", "w4a8", "int8"])
@pytest.mark.parametrize("I", [768, 512])
@pytest.mark.parametrize("M", [1, 2, 4, 8, 12, 16])
@pytest.mark.parametrize("bf16", [True, False])
def test_tc_decode_matches_oracle(cuda, monkeypatch, kind, I, M, bf16):
    E = 32
    banks = (gd.rand_bank(kind, E, 2 * I, H, 600 + M, cuda), gd.rand_bank(kind, E, H, I, 700 + M, cuda))
    x = gd.rand_rows(M, H, 800 + M, cuda)
    if not bf16:
        x = torch.randn((M, H), generator=torch.Generator().manual_seed(850 + M)).to(cuda)
    ids, w = gd.rand_routing(M, E, 8, 900 + M, cuda)
    _lib.take_fault()
    tc, old = both(monkeypatch, kind, x, ids, w, banks)
    assert _lib.take_fault() == 0
    ref = oracle(kind, x, ids, w, banks)
    assert gd.rel_l2(tc.float(), ref) <= 1e-3
    assert gd.rel_l2(tc.float(), old.float()) <= 1e-3


@pytest.mark.parametrize("kind", ["fp8c", "w4a8", "int8"])
def test_tc_decode_benchmark_shape_and_repeats(cuda, monkeypatch, kind):
    """128 experts, 16 lines (the benchmark's layer): against the mma.sync decode, and bit-identical over repeated
    calls that share one workspace."""
    E, I, M = 128, 768, 16
    banks = (gd.rand_bank(kind, E, 2 * I, H, 11, cuda), gd.rand_bank(kind, E, H, I, 12, cuda))
    x = gd.rand_rows(M, H, 13, cuda)
    ids, w = gd.rand_routing(M, E, 8, 14, cuda)
    tc, old = both(monkeypatch, kind, x, ids, w, banks)
    assert gd.rel_l2(tc.float(), old.float()) <= 1e-3
    ws = kernels.decode_workspace(M, 8, I, cuda)
    first = kernels.moe_decode(kind, x, ids, w, banks, workspace=ws)
    for _ in range(3):
        assert torch.equal(kernels.moe_decode(kind, x, ids, w, banks, workspace=ws), first)
    assert torch.equal(first, tc)


def test_tc_decode_crowded_and_bad_ids(cuda, monkeypatch):
    """Every line routed to the same 8 experts (segments of 16 pairs), and an out-of-range id (skipped, fault bit 2)."""
    E, I, M = 16, 768, 16
    banks = (gd.rand_bank("fp8c", E, 2 * I, H, 21, cuda), gd.rand_bank("fp8c", E, H, I, 22, cuda))
    x = gd.rand_rows(M, H, 23, cuda)
    ids = torch.arange(8, device=cuda).repeat(M, 1)
    w = torch.full((M, 8), 0.125, device=cuda)
    tc, old = both(monkeypatch, "fp8c", x, ids, w, banks)
    assert gd.rel_l2(tc.float(), gd.baseline_oracle_decode("fp8c", x, ids, w, banks)) <= 1e-3
    assert gd.rel_l2(tc.float(), old.float()) <= 1e-3
    bad = ids.clone()
    bad[3, 2] = 40
    _lib.take_fault()
    tc, old = both(monkeypatch, "fp8c", x, bad, w, banks)
    assert _lib.take_fault() == 2
    assert gd.rel_l2(tc.float(), old.float()) <= 1e-3


@pytest.mark.parametrize("kind", ["fp8c", "w4a8", "int8"])
def test_tc_decode_expert_parallel_partials(cuda, monkeypatch, kind):
    """Expert blocks of 3 emulated ranks: each rank's fp32 partial against the mma.sync kernel's, their rank-order sum
    against the whole decode; then the peer exchange of one rank bit for bit against the same partial."""
    E, I, M, world = 32, 768, 16, 3
    full = (gd.rand_bank(kind, E, 2 * I, H, 31, cuda), gd.rand_bank(kind, E, H, I, 32, cuda))
    x = gd.rand_rows(M, H, 33, cuda)
    ids, w = gd.rand_routing(M, E, 8, 34, cuda)
    parts = []
    for r in range(world):
        first = ep.expert_range(E, r, world)[0]
        banks = ep.local_banks(full, E, r, world)
        monkeypatch.delenv("D3_DECODE_TC", raising=False)
        p = kernels.moe_decode_ep(kind, x, ids, w, banks, first, E)
        monkeypatch.setenv("D3_DECODE_TC", "0")
        q = kernels.moe_decode_ep(kind, x, ids, w, banks, first, E)
        monkeypatch.delenv("D3_DECODE_TC")
        assert gd.rel_l2(p, q) <= 1e-3
        parts.append(p)
    total = ep.sum_in_rank_order(torch.stack(parts)).to(torch.bfloat16)
    assert gd.rel_l2(total.float(), kernels.moe_decode(kind, x, ids, w, full).float()) <= 1e-3
    size, flags = ep.exchange_layout(1, M, H)
    area = torch.zeros((size,), dtype=torch.uint8, device=cuda)
    st = torch.frombuffer(bytearray(ep.exchange_struct([area.data_ptr()], flags, 0, M, H)), dtype=torch.uint8).to(cuda)
    kernels.moe_decode_ep(kind, x, ids, w, full, 0, E, exchange=st)
    whole = kernels.moe_decode_ep(kind, x, ids, w, full, 0, E)
    assert torch.equal(kernels.ep_reduce(st, M, H), whole.to(torch.bfloat16))


@pytest.mark.parametrize("kind", ["fp8c", "w4a8", "int8"])
def test_last_arrival_combine_equals_grid_combine(cuda, monkeypatch, kind):
    """With few segments (one or two lines) each 128-row block is combined by the tile that completes it instead of
    after a grid barrier (D3_LASTARRIVE_NSEG: 0 forces the grid barrier). Same arithmetic, so the outputs agree bit
    for bit, over repeated calls (the block and exit counters reset themselves), for the plain decode and for an
    expert-parallel partial."""
    E = 128
    banks = (gd.rand_bank(kind, E, 1536, H, 400, cuda), gd.rand_bank(kind, E, H, 768, 401, cuda))
    _lib.take_fault()
    for call, M in enumerate((1, 2, 1, 1, 2)):
        x = gd.rand_rows(M, H, 410 + call, cuda)
        ids, w = gd.rand_routing(M, E, 8, 420 + call, cuda)
        monkeypatch.setenv("D3_LASTARRIVE_NSEG", "16")
        fast = kernels.moe_decode(kind, x, ids, w, banks)
        part_fast = kernels.moe_decode_ep(kind, x, ids, w, ep.local_banks(banks, E, 0, 2), 0, E)
        monkeypatch.setenv("D3_LASTARRIVE_NSEG", "0")
        slow = kernels.moe_decode(kind, x, ids, w, banks)
        part_slow = kernels.moe_decode_ep(kind, x, ids, w, ep.local_banks(banks, E, 0, 2), 0, E)
        monkeypatch.delenv("D3_LASTARRIVE_NSEG")
        torch.cuda.synchronize()
        assert torch.equal(fast, slow), (kind, call, M)
        assert torch.equal(part_fast, part_slow), (kind, call, M)
    assert _lib.take_fault() == 0
