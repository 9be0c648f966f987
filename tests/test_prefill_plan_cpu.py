"""The device-side sort of a prompt's pairs by expert (offload.prefill_plan), run here on CPU tensors: the same torch
ops the GPU runs, checked against the host-side plan of the reference's prompt pass (argsort + bincount,
drama3/offload.py:141-145): a stable order by expert, its inverse, every expert's group with exclusive-sum offsets,
out-of-range ids in one last group, and a tile bound no routing exceeds."""
import numpy as np
import pytest
import torch

from drama3_b200 import kernels, offload


def check_plan(ids, E):
    order, pos, groups, tiles = offload.prefill_plan(ids, E)
    flat = ids.reshape(-1).numpy()
    P = flat.size
    key = np.where((flat >= 0) & (flat < E), flat, E)
    want_order = np.argsort(key, kind="stable")
    assert order.dtype == torch.int64 and pos.dtype == torch.int64 and groups.dtype == torch.int32
    assert np.array_equal(order.numpy(), want_order)
    assert np.array_equal(pos.numpy()[want_order], np.arange(P))
    counts = np.bincount(key, minlength=E + 1)
    first = np.concatenate([[0], np.cumsum(counts)[:-1]])
    g = groups.numpy()
    assert g.shape == (E + 1, 5)
    assert np.array_equal(g[:, 0], np.arange(E + 1)) and np.array_equal(g[:, 1], np.arange(E + 1))
    assert not g[:, 2].any()
    assert np.array_equal(g[:, 3], first) and np.array_equal(g[:, 4], counts)
    assert tiles >= kernels.grouped_tiles(counts)
    # the host-side plan's non-empty groups over the valid ids are the same groups
    valid = flat[(flat >= 0) & (flat < E)]
    host_order, host_counts = offload._sort_by_expert(torch.from_numpy(valid), E)
    assert host_counts == counts[:E].tolist()
    assert sorted(valid[host_order.numpy()].tolist()) == valid[host_order.numpy()].tolist()
    return order, pos, groups, tiles


@pytest.mark.parametrize("T, k, E", [(2048, 8, 128), (37, 8, 16), (1, 8, 128), (300, 2, 4)])
def test_plan_matches_host_sort(T, k, E):
    gen = torch.Generator().manual_seed(T + E)
    skew = -1.1 * torch.log(torch.randperm(E, generator=gen).float() + 1)
    ids = (torch.rand((T, E), generator=gen).log().neg().reciprocal() * skew.exp()).topk(k, dim=-1).indices
    check_plan(ids, E)


def test_plan_all_pairs_on_one_expert_and_empty_experts():
    ids = torch.full((513, 8), 5, dtype=torch.int64)
    _, _, groups, tiles = check_plan(ids, 128)
    assert groups[5, 4] == 513 * 8 and int(groups[:, 4].sum()) == 513 * 8
    assert tiles >= (513 * 8 + 127) // 128


def test_plan_out_of_range_ids_sort_last():
    ids = torch.randint(0, 16, (40, 8), generator=torch.Generator().manual_seed(3))
    ids[3, 2], ids[5, 0], ids[9, 7] = 16, -1, 99
    order, _, groups, _ = check_plan(ids, 16)
    assert groups[16].tolist() == [16, 16, 0, 40 * 8 - 3, 3]
    assert sorted(order[-3:].tolist()) == [3 * 8 + 2, 5 * 8 + 0, 9 * 8 + 7]


def test_plan_of_no_rows():
    order, pos, groups, tiles = offload.prefill_plan(torch.zeros((0, 8), dtype=torch.int64), 128)
    assert order.numel() == 0 and pos.numel() == 0 and not groups[:, 4].any()
    assert tiles >= 0


def test_tile_bound_is_tight_for_the_worst_routing():
    """Every expert holding one row more than a whole number of tiles is the worst case: the bound equals it."""
    E, t = 8, kernels.grouped_tile_rows()
    counts = [t + 1] * E
    ids = torch.repeat_interleave(torch.arange(E), torch.tensor(counts)).view(-1, 1)
    _, _, groups, tiles = offload.prefill_plan(ids, E)
    need = kernels.grouped_tiles(groups[:, 4].tolist())
    assert need == 2 * E and tiles == need


def test_plan_of_int32_ids_equals_int64():
    ids = torch.randint(0, 32, (100, 8), generator=torch.Generator().manual_seed(9))
    a = offload.prefill_plan(ids, 32)
    b = offload.prefill_plan(ids.to(torch.int32), 32)
    assert all(torch.equal(u, v) for u, v in zip(a[:3], b[:3])) and a[3] == b[3]


# ---- the native plan kernel's own scheme (csrc/plan.cuh, prefill_plan_kernel), restated in integers: 32 warps, each
# owning a contiguous segment of S pairs (S = ceil(P / 32) rounded up to 32), counting and then placing its pairs 32
# a round; the rank of a pair among the equal keys of its round is what __match_any_sync gives (its position among
# the lanes holding the same key)

def warp_segment_plan(ids, E):
    P = ids.size
    keys = E + 1
    S = ((P + 31) // 32 + 31) & ~31
    key = np.where((ids >= 0) & (ids < E), ids, E)
    start = np.zeros((32, keys), np.int64)
    for w in range(32):  # pass 1: each warp's own row of counts
        for i in range(w * S, min(P, w * S + S)):
            start[w, key[i]] += 1
    total = start.sum(axis=0)
    start = (np.cumsum(start, axis=0) - start) + (np.cumsum(total) - total)  # per key over warps, then over keys
    order, pos = np.zeros(P, np.int64), np.zeros(P, np.int64)
    for w in range(32):  # pass 2: place, a round at a time
        seg1 = min(P, w * S + S)
        for i0 in range(w * S, seg1, 32):
            lanes = list(range(i0, min(i0 + 32, seg1)))
            for i in lanes:
                before = sum(1 for j in lanes if j < i and key[j] == key[i])
                pos[i] = start[w, key[i]] + before
                order[pos[i]] = i
            for k in set(key[lanes].tolist()):
                start[w, k] += int((key[lanes] == k).sum())
    return order, pos, total


@pytest.mark.parametrize("P, E, seed", [(16384, 128, 0), (1, 4, 1), (33, 3, 2), (1000, 256, 3), (0, 8, 4),
                                         (5000, 1, 5), (1025, 16, 6)])
def test_warp_segment_scheme_is_a_stable_sort(P, E, seed):
    rng = np.random.default_rng(seed)
    ids = rng.integers(-2, E + 2, P)
    if P > 8:
        ids[: P // 2] = rng.zipf(1.5, P // 2) % E  # skew, ties in every round
    order, pos, total = warp_segment_plan(ids, E)
    key = np.where((ids >= 0) & (ids < E), ids, E)
    assert np.array_equal(order, np.argsort(key, kind="stable"))
    assert np.array_equal(pos[order], np.arange(P))
    assert np.array_equal(total, np.bincount(key, minlength=E + 1))
