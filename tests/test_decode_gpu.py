"""The fused decode (d3_moe_decode) against the CPU oracle and the reference's own kernels, at the BASELINE layer
shape (hidden 2048, 128 experts, top-8, intermediate 768), M = 1, 4, 16 rows. Tolerance: rel-L2 <= 1e-3 on the
bf16 outputs."""
import pytest
import torch

import gpu_data as gd

pytestmark = pytest.mark.gpu

E, H, I, K = 128, 2048, 768, 8
TOL = 1e-3


@pytest.fixture(scope="module")
def banks_by_kind(cuda):
    out = {}
    for i, kind in enumerate(gd.KINDS):
        out[kind] = (gd.rand_bank(kind, E, 2 * I, H, 10 + i, cuda), gd.rand_bank(kind, E, H, I, 20 + i, cuda))
    return out


@pytest.mark.parametrize("kind", gd.KINDS)
@pytest.mark.parametrize("M", [1, 4, 16])
def test_decode_matches_oracle(cuda, banks_by_kind, kind, M):
    from drama3_b200 import kernels
    from drama3_b200._lib import take_fault
    banks = banks_by_kind[kind]
    cbs = gd.codebooks(kind, cuda)
    x = gd.rand_rows(M, H, 100 + M, cuda)
    ids, w = gd.rand_routing(M, E, K, 200 + M, cuda)
    out = kernels.moe_decode(kind, x, ids, w, banks, cbs)
    torch.cuda.synchronize()
    assert take_fault() == 0
    ref = gd.oracle_decode(kind, x, ids, w, banks, cbs, H)
    err = gd.rel_l2(out.float(), torch.from_numpy(ref))
    assert err <= TOL, (kind, M, err)


@pytest.mark.parametrize("kind", gd.KINDS)
@pytest.mark.parametrize("M", [1, 16])
def test_decode_matches_reference_kernels(cuda, banks_by_kind, kind, M):
    from drama3_b200 import kernels
    from oracle import ref_gpu
    if not ref_gpu.available():
        pytest.skip("reference cubin not built")
    banks = banks_by_kind[kind]
    cbs = gd.codebooks(kind, cuda)
    x = gd.rand_rows(M, H, 300 + M, cuda)
    ids, w = gd.rand_routing(M, E, K, 400 + M, cuda)
    out = kernels.moe_decode(kind, x, ids, w, banks, cbs)
    ref = ref_gpu.lines_decode(x, ids, w, banks, (2 * I, H), kind, cbs)
    err = gd.rel_l2(out.float(), ref.float())
    assert err <= TOL, (kind, M, err)


def test_decode_repeatable_and_graph_capturable(cuda, banks_by_kind):
    from drama3_b200 import kernels
    banks = banks_by_kind["fp8"]
    x = gd.rand_rows(16, H, 7, cuda)
    ids, w = gd.rand_routing(16, E, K, 8, cuda)
    ws = kernels.decode_workspace(16, K, I, cuda)
    out = torch.empty((16, H), dtype=torch.bfloat16, device=cuda)
    kernels.moe_decode("fp8", x, ids, w, banks, workspace=ws, out=out)
    first = out.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        kernels.moe_decode("fp8", x, ids, w, banks, workspace=ws, out=out)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first)  # deterministic: no atomics in the combine


def test_decode_duplicate_and_bad_ids(cuda, banks_by_kind):
    """Ids a top-k never produces: a repeated expert in one row (computed twice, as the reference would) and an
    out-of-range id (skipped, zeros for that term, fault bit 2)."""
    from drama3_b200 import kernels
    from drama3_b200._lib import take_fault
    banks = banks_by_kind["fp8"]
    x = gd.rand_rows(2, H, 9, cuda)
    ids = torch.tensor([[3, 3, 5, 7, 9, 11, 13, 15], [1, 2, 4, 6, 8, 10, 12, 14]], device=cuda)
    w = torch.full((2, K), 0.125, device=cuda)
    out = kernels.moe_decode("fp8", x, ids, w, banks)
    torch.cuda.synchronize()
    assert take_fault() == 0
    ref = gd.oracle_decode("fp8", x, ids, w, banks, (None, None), H)
    assert gd.rel_l2(out.float(), torch.from_numpy(ref)) <= TOL
    bad = ids.clone()
    bad[1, 3] = E + 5
    out_bad = kernels.moe_decode("fp8", x, bad, w, banks)
    torch.cuda.synchronize()
    assert take_fault() == 2
    ok = ids.clone()
    ok[1, 3] = ids[1, 2]
    w_ok = w.clone()
    w_ok[1, 3] = 0.0
    ref2 = gd.oracle_decode("fp8", x, ok, w_ok, banks, (None, None), H)
    assert gd.rel_l2(out_bad.float(), torch.from_numpy(ref2)) <= TOL
