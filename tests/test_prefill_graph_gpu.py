"""The prompt pass without host syncs (offload.resident_prefill(sync_free=True): the pairs sorted on the device,
grouped GEMMs sized by a tile bound from the shapes): bit for bit the host-planned pass, and captured in a CUDA graph
that replays new routing and rows written into the same input buffers."""
import pytest
import torch

import gpu_data as gd
from drama3_b200 import _lib, offload

pytestmark = pytest.mark.gpu
E, H, I, T = 128, 2048, 768, 2048


def layer(kind, seed, device):
    gu = gd.rand_bank(kind, E, 2 * I, H, seed, device)
    dn = gd.rand_bank(kind, E, H, I, seed + 1, device)
    return (gu, dn), gd.codebooks(kind, device)


def prompt(seed, device):
    skew = -1.1 * torch.log(torch.randperm(E, generator=torch.Generator().manual_seed(seed)).float() + 1)
    x = gd.rand_rows(T, H, seed + 1, device)
    ids, w = gd.rand_routing(T, E, 8, seed + 2, device, skew=skew)
    return x, ids, w.to(torch.bfloat16)


@pytest.mark.parametrize("kind", ["fp8", "int8", "w4", "w6a8"])
def test_sync_free_prefill_matches_host_plan(cuda, kind):
    banks, cbs = layer(kind, 80, cuda)
    x, ids, w = prompt(82, cuda)
    _lib.take_fault()
    planned = offload.resident_prefill(x, ids, w, banks, (2 * I, H), kind, cbs, E)
    free = offload.resident_prefill(x, ids, w, banks, (2 * I, H), kind, cbs, E, sync_free=True)
    torch.cuda.synchronize()
    assert _lib.take_fault() == 0
    assert torch.equal(free, planned)


def test_sync_free_prefill_replays_new_routing_in_a_cuda_graph(cuda):
    kind = "w6a8"
    banks, cbs = layer(kind, 90, cuda)
    x, ids, w = prompt(92, cuda)

    def run():
        return offload.resident_prefill(x, ids, w, banks, (2 * I, H), kind, cbs, E, sync_free=True)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            run()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = run()
    try:
        _lib.take_fault()
        for seed in (92, 95, 98):
            nx, nids, nw = prompt(seed, cuda)
            x.copy_(nx)
            ids.copy_(nids)
            w.copy_(nw)
            graph.replay()
            want = offload.resident_prefill(nx, nids, nw, banks, (2 * I, H), kind, cbs, E)
            torch.cuda.synchronize()
            assert torch.equal(out, want), seed
        assert _lib.take_fault() == 0
    finally:
        del graph


def test_sync_free_needs_the_tensor_core_shapes(cuda):
    banks, cbs = layer("fp8", 100, cuda)
    x, ids, w = prompt(102, cuda)
    with pytest.raises(ValueError):
        offload.resident_prefill(x.to(torch.float16), ids, w, banks, (2 * I, H), "fp8", cbs, E, sync_free=True)


def test_fp8_experts_prompt_pass_captured(cuda):
    """FP8Experts reached inside a CUDA-graph capture takes the device-side sort by itself: the captured prompt pass
    replays to the eager (host-planned) result bit for bit."""
    from test_offload_gpu import fp8_module
    ex, _ = fp8_module(16, H, I, 110, cuda)
    x, ids, w = prompt(112, cuda)
    ids = ids % 16
    eager = ex(x, ids, w)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ex(x, ids, w)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = ex(x, ids, w)
    try:
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    finally:
        del graph


def _ids_cases():
    g = torch.Generator().manual_seed(91)
    yield "zipf", torch.multinomial(torch.arange(1, E + 1).float().pow(-1.1), 16384, True, generator=g).view(-1, 8), E
    yield "ragged", torch.randint(0, E, (333, 7), generator=g), E
    bad = torch.randint(0, E, (1500, 8), generator=g)
    bad[::7, 3] = -1
    bad[::11, 5] = E
    bad[::13, 0] = 10 ** 6
    yield "out_of_range", bad, E
    yield "one_expert", torch.full((2048, 8), 5, dtype=torch.int64), E
    yield "empty", torch.zeros((0, 8), dtype=torch.int64), E
    yield "e256", torch.randint(0, 256, (4096, 8), generator=g), 256
    yield "e1", torch.randint(0, 2, (100, 3), generator=g), 1


@pytest.mark.parametrize("drop_invalid", [False, True])
def test_native_plan_equals_the_torch_counting_sort(cuda, drop_invalid):
    """kernels.prefill_plan (one block, counting sort) against the torch restatement of the same sort run on the CPU:
    order, inverse and groups identical, for skewed, ragged, out-of-range, one-expert, empty and 256-expert
    routings."""
    from drama3_b200 import kernels
    for name, ids, n_exp in _ids_cases():
        order, pos, groups = kernels.prefill_plan(ids.to(cuda), n_exp, drop_invalid)
        want = offload.prefill_plan(ids, n_exp, drop_invalid)
        assert torch.equal(order.cpu(), want[0]), name
        assert torch.equal(pos.cpu(), want[1]), name
        assert torch.equal(groups.cpu(), want[2]), name
