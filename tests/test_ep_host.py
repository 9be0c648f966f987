"""Expert parallelism on CPU ranks (gloo, world size 2): the expert partition, the bank slicing and the exchange
(all-gather + rank-order sum) of drama3_b200.ep, with the oracle standing in for each rank's GPU kernel."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from drama3_b200 import ep
from oracle import moe

E, H, I, K = 8, 256, 128, 4


def test_expert_range_covers_all_in_order():
    for E_, world in ((128, 8), (128, 3), (7, 4), (16, 16)):
        ranges = [ep.expert_range(E_, r, world) for r in range(world)]
        assert ranges[0][0] == 0 and sum(c for _, c in ranges) == E_
        for (f0, c0), (f1, _) in zip(ranges, ranges[1:]):
            assert f1 == f0 + c0
        assert max(c for _, c in ranges) - min(c for _, c in ranges) <= 1


def test_exchange_struct_layout():
    """The ctypes mirror of the kernels' exchange struct: its offsets, and the area layout (slots, then the flags and
    the call counter at the next 256-byte boundary)."""
    import ctypes
    S = ep.ExchangeStruct
    assert ctypes.sizeof(S) == 152 and S.flags.offset == 64 and S.epoch.offset == 128 and S.world.offset == 136
    assert S.rank.offset == 140 and S.m_max.offset == 144 and S.h.offset == 148
    size, flags = ep.exchange_layout(2, 3, 2048)
    assert flags == 2 * 2 * 3 * 2048 * 4 and size == flags + 256
    raw = ep.exchange_struct([0x1000, 0x200000], flags, 1, 3, 2048)
    st = S.from_buffer_copy(raw)
    assert list(st.slots[:2]) == [0x1000, 0x200000] and list(st.flags[:2]) == [0x1000 + flags, 0x200000 + flags]
    assert st.epoch == 0x200000 + flags + 64 and (st.world, st.rank, st.m_max, st.h) == (2, 1, 3, 2048)
    with pytest.raises(ValueError):
        ep.exchange_layout(9, 1, 2048)


def _banks():
    rng = np.random.default_rng(11)
    w13 = rng.normal(0, 0.02, size=(E, 2 * I, H)).astype(np.float32)
    w2 = rng.normal(0, 0.02, size=(E, H, I)).astype(np.float32)
    return moe.make_baseline_bank("fp8c", w13), moe.make_baseline_bank("fp8c", w2)


def _inputs():
    rng = np.random.default_rng(12)
    x = moe.bf16_round(rng.normal(size=(3, H)).astype(np.float32))
    ids = np.stack([rng.permutation(E)[:K] for _ in range(3)])
    w = moe.bf16_round(rng.dirichlet(np.ones(K), size=3).astype(np.float32))
    return x, ids, w


def _oracle_partial(banks, x, ids, w, first, count):
    """The routing-weighted sum over the pairs of experts [first, first + count), in rank order (fp32)."""
    gate_up, down = banks
    out = np.zeros((x.shape[0], H), np.float32)
    for t in range(x.shape[0]):
        for j, e in enumerate(ids[t]):
            if not first <= e < first + count:
                continue
            h = moe.baseline_rows("fp8c", x[t:t + 1], gate_up, int(e) * 2 * I, 2 * I)
            a = moe._silu_mul(h[:, :I], h[:, I:])
            part = moe.baseline_rows("fp8c", a, down, int(e) * H, H)[0]
            out[t] = moe.fma32(part, np.full(H, w[t, j], np.float32), out[t])
    return out


def _worker(rank, world, port, result):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        banks = _banks()
        x, ids, w = _inputs()
        first, count = ep.expert_range(E, rank, world)
        local = ep.local_banks(tuple({n: torch.from_numpy(v) for n, v in b.items()} for b in banks), E, rank, world)
        assert local[0]["weight"].shape[0] == count * 2 * I and local[1]["scale"].shape[0] == count * H

        def decode_fn(xt, idt, wt):
            return torch.from_numpy(_oracle_partial(banks, xt.numpy(), idt.numpy(), wt.numpy(), first, count))

        layer = ep.ExpertParallelDecode("fp8c", local, E, decode_fn=decode_fn)
        out = layer(torch.from_numpy(x), torch.from_numpy(ids), torch.from_numpy(w))
        full = moe.baseline_decode("fp8c", x, ids, w, banks)
        err = float(np.linalg.norm(out.float().numpy() - full) / np.linalg.norm(full))
        result[rank] = err
    finally:
        dist.destroy_process_group()


def test_expert_parallel_exchange_two_cpu_ranks():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    result = ctx.Manager().dict()
    mp.start_processes(_worker, args=(2, port, result), nprocs=2, join=True, start_method="spawn")
    assert sorted(result.keys()) == [0, 1]
    assert all(err <= 1e-3 for err in result.values()), dict(result)


# ---- the expert-parallel prompt pass: rows split by rank, pairs sent to their experts' ranks and back

PF_T, PF_E, PF_H, PF_K = 50, 10, 64, 4
PF_SHARDS = {2: [(0, 23), (23, 50)], 3: [(0, 20), (20, 20), (20, 50)]}


def _pf_inputs():
    gen = torch.Generator().manual_seed(21)
    x = torch.randn((PF_T, PF_H), generator=gen).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(PF_E, generator=gen)[:PF_K] for _ in range(PF_T)])
    ids[3, 1], ids[7, 0] = PF_E + 2, -1  # out of range: add nothing
    w = torch.softmax(torch.randn((PF_T, PF_K), generator=gen), -1)
    return x, ids, w


def _pf_pair(x, ids):
    """A stand-in for an expert on a row, exact and different per expert: fp32 x (e + 1) + e."""
    e = ids.to(torch.float32).unsqueeze(1)
    return x.float() * (e + 1) + e


def _pf_combine(pair_out, w):
    """Rank-order weighted sum of each row's pairs, fp32."""
    T, k = w.shape
    p = pair_out.view(T, k, pair_out.shape[1])
    out = torch.zeros((T, pair_out.shape[1]))
    for j in range(k):
        out = out + w[:, j:j + 1] * p[:, j]
    return out


def _pf_worker(rank, world, port, result):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        x, ids, w = _pf_inputs()
        lo, hi = PF_SHARDS[world][rank]
        first, count = ep.expert_range(PF_E, rank, world)
        seen = []

        def pairs_fn(xr, gid):
            seen.append(bool(((gid >= first) & (gid < first + count)).all()))
            return _pf_pair(xr, gid)

        layer = ep.ExpertParallelPrefill("fp8c", None, PF_E, (2 * PF_H, PF_H), pairs_fn=pairs_fn,
                                         combine_fn=_pf_combine)
        out = layer(x[lo:hi], ids[lo:hi], w[lo:hi])
        flat = ids[lo:hi].reshape(-1)
        valid = ((flat >= 0) & (flat < PF_E)).unsqueeze(1)
        ref_pairs = torch.where(valid, _pf_pair(x[lo:hi].repeat_interleave(PF_K, 0), flat), torch.zeros(()))
        want = _pf_combine(ref_pairs, w[lo:hi])
        result[rank] = (tuple(out.shape) == (hi - lo, PF_H) and torch.equal(out, want) and all(seen))
    finally:
        dist.destroy_process_group()


def _pf_fixed_worker(rank, world, port, result, capacity):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        x, ids, w = _pf_inputs()
        lo, hi = PF_SHARDS[world][rank]
        layer = ep.ExpertParallelPrefill("fp8c", None, PF_E, (2 * PF_H, PF_H), pairs_fn=_pf_pair,
                                         combine_fn=_pf_combine, capacity=capacity)
        out = layer(x[lo:hi], ids[lo:hi], w[lo:hi])
        flat = ids[lo:hi].reshape(-1)
        owner = ep.expert_owner(flat, PF_E, world)
        # the pairs sent: per destination rank, the first `capacity` in (row, rank) order
        kept = torch.zeros_like(flat, dtype=torch.bool)
        for r in range(world):
            kept[(owner == r).nonzero().squeeze(1)[:capacity]] = True
        ref_pairs = torch.where(kept.unsqueeze(1), _pf_pair(x[lo:hi].repeat_interleave(PF_K, 0), flat),
                                torch.zeros(()))
        want = _pf_combine(ref_pairs, w[lo:hi])
        dropped = int(((owner >= 0) & ~kept).sum())
        result[rank] = (torch.equal(out, want), int(layer.dropped), dropped)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world, capacity", [(2, 27 * PF_K), (3, 30 * PF_K), (2, 3), (3, 5)])
def test_expert_parallel_prefill_fixed_blocks_cpu_ranks(world, capacity):
    """The exchange in fixed blocks (no split sizes read back): with room for every pair it equals the pass over the
    same rows; with less, each destination takes the first `capacity` pairs and the rest add nothing and are
    counted."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    result = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_pf_fixed_worker, args=(world, port, result, capacity), nprocs=world, join=True,
                       start_method="spawn")
    assert sorted(result) == list(range(world))
    for same, counted, expected in result.values():
        assert same and counted == expected
    if capacity >= 27 * PF_K:
        assert all(v[2] == 0 for v in result.values())


@pytest.mark.parametrize("world", [2, 3])
def test_expert_parallel_prefill_exchange_cpu_ranks(world):
    """Each rank's rows come back equal to the one-process pass over the same rows, bit for bit; every rank receives
    only pairs of its own experts; one rank with no rows at all (world 3) still takes part in the exchanges."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    result = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_pf_worker, args=(world, port, result), nprocs=world, join=True, start_method="spawn")
    assert dict(result) == {r: True for r in range(world)}


def test_expert_owner_matches_expert_range():
    for E_, world in ((128, 8), (128, 3), (10, 4), (3, 8)):
        ids = torch.arange(-2, E_ + 3)
        owner = ep.expert_owner(ids, E_, world)
        for i, o in zip(ids.tolist(), owner.tolist()):
            blocks = [r for r in range(world) if 0 <= i - ep.expert_range(E_, r, world)[0] <
                      ep.expert_range(E_, r, world)[1]]
            assert o == (blocks[0] if blocks else -1)
