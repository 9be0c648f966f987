"""The prompt pass's host-side glue on the CPU, with the two GPU kernels it calls (kernels.grouped_mma and
kernels.prefill_combine) replaced by torch stand-ins that follow their contracts (groups of sorted rows, row_index,
SwiGLU staging, the tile count, rows outside every group untouched; the rank-order weighted sum): the device-side
sort (resident_prefill(sync_free=True)) against the host-side one, and the expert-parallel pass's default path
(ep.local_pairs under the all-to-alls) against the one-process pass, on gloo ranks. Shapes, dtypes and index
arithmetic of the glue are what this checks; the kernels' arithmetic is checked on the GPU."""
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from drama3_b200 import ep, kernels, offload

E, H, I, K_TOP = 12, 256, 256, 4


def expert_weights(n, k, seed):
    return torch.randn((E, n, k), generator=torch.Generator().manual_seed(seed)) / k ** 0.5


W13, W2 = expert_weights(2 * I, H, 1), expert_weights(H, I, 2)


def fake_grouped_mma(kind, x, groups, fields, codebook, n, tiles, row_index=None, rotate=False, swiglu=False):
    """kernels.grouped_mma's contract on the CPU: sorted row s = x[row_index[s]] (or x[s]), SwiGLU first when asked,
    through the weights of its group's slot (fields["first"] + slot indexes the stand-in experts); groups past the
    bank are skipped; at most `tiles` tiles of 128 rows run."""
    rows = row_index.shape[0] if row_index is not None else x.shape[0]
    out = torch.full((rows, n), float("nan"))
    weights = W13 if n == 2 * I else W2
    bank_experts, first = fields["count"], fields["first"]
    need = 0
    for e, slot, _, start, count in groups.tolist():
        need += (count + 127) // 128
        if count == 0 or not 0 <= slot < bank_experts:
            continue
        assert need <= tiles
        src = torch.arange(start, start + count)
        v = x[row_index[src]] if row_index is not None else x[src]
        v = v.float()
        if swiglu:
            v = torch.nn.functional.silu(v[:, :v.shape[1] // 2]) * v[:, v.shape[1] // 2:]
        for r in range(count):  # row by row: a row's result must not depend on the rows beside it
            out[start + r] = v[r] @ weights[first + slot].T
    return out


def fake_combine(sorted_out, pos, weights, dtype=torch.bfloat16):
    T, k = pos.shape
    out = torch.zeros((T, sorted_out.shape[1]))
    for j in range(k):
        out = out + weights[:, j:j + 1].float() * sorted_out[pos[:, j]]
    return out.to(dtype)


@pytest.fixture
def fakes(monkeypatch):
    monkeypatch.setattr(kernels, "grouped_mma", fake_grouped_mma)
    monkeypatch.setattr(kernels, "prefill_combine", fake_combine)


def prompt(T, seed):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn((T, H), generator=gen).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=gen)[:K_TOP] for _ in range(T)])
    w = torch.softmax(torch.randn((T, K_TOP), generator=gen), -1).to(torch.bfloat16)
    return x, ids, w


BANKS = ({"count": E, "first": 0}, {"count": E, "first": 0})


def test_sync_free_glue_equals_host_plan(fakes):
    x, ids, w = prompt(300, 3)
    planned = offload.resident_prefill(x, ids, w, BANKS, (2 * I, H), "fp8c", (None, None), E)
    free = offload.resident_prefill(x, ids, w, BANKS, (2 * I, H), "fp8c", (None, None), E, sync_free=True)
    assert planned.dtype == free.dtype == torch.bfloat16 and not planned.isnan().any()
    assert torch.equal(free, planned)


def test_local_pairs_glue_keeps_the_given_order(fakes):
    x, ids, _ = prompt(40, 4)
    first, count = ep.expert_range(E, 1, 3)
    flat = ids.reshape(-1)
    sel = ((flat >= first) & (flat < first + count)).nonzero().squeeze(1)
    got = ep.local_pairs("fp8c", ({"count": count, "first": first},) * 2, count, (2 * I, H), (None, None),
                         x[sel // K_TOP], (flat[sel] - first).to(torch.int32))
    xs = x[sel // K_TOP].float()
    for j in range(sel.numel()):
        e = int(flat[sel[j]])
        h = xs[j] @ W13[e].T
        want = (torch.nn.functional.silu(h[:I]) * h[I:]) @ W2[e].T
        assert torch.allclose(got[j], want, rtol=1e-5, atol=1e-6)


def _worker(rank, world, port, result, capacity=None):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        kernels.grouped_mma, kernels.prefill_combine = fake_grouped_mma, fake_combine
        x, ids, w = prompt(90, 5)
        lo, hi = 90 * rank // world, 90 * (rank + 1) // world
        first, count = ep.expert_range(E, rank, world)
        local = ({"count": count, "first": first},) * 2
        layer = ep.ExpertParallelPrefill("fp8c", local, E, (2 * I, H), capacity=capacity)
        got = layer(x[lo:hi], ids[lo:hi], w[lo:hi])
        want = offload.resident_prefill(x[lo:hi], ids[lo:hi], w[lo:hi], BANKS, (2 * I, H), "fp8c", (None, None), E)
        result[rank] = bool(torch.equal(got, want)) and (capacity is None or int(layer.dropped) == 0)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world, capacity", [(2, None), (3, None), (2, 45 * K_TOP), (3, 30 * K_TOP)])
def test_expert_parallel_prefill_default_path_on_cpu_ranks(world, capacity):
    """Split sizes read back, or fixed blocks of `capacity` rows (padding rows left out of the GEMMs' groups)."""
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    result = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_worker, args=(world, port, result, capacity), nprocs=world, join=True, start_method="spawn")
    assert dict(result) == {r: True for r in range(world)}
