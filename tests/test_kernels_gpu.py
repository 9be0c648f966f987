"""Each reference kernel's replacement against the reference kernel itself (oracle/_ref cubin, bit-exact where the
arithmetic is integer or order-identical) and against the CPU oracle."""
import numpy as np
import pytest
import torch

import gpu_data as gd
from oracle import moe

pytestmark = pytest.mark.gpu


def ref():
    from oracle import ref_gpu
    if not ref_gpu.available():
        pytest.skip("reference cubin not built")
    return ref_gpu


def lib():
    from drama3_b200 import kernels
    return kernels


# ---------------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("n,k", [(128, 8), (256, 8), (1024, 32), (40, 1)])
def test_route_bit_exact(cuda, n, k):
    kernels, r = lib(), ref()
    gen = torch.Generator().manual_seed(n * 7 + k)
    rows = 64
    logits = (torch.randn((rows, n), generator=gen) * 0.9).to(torch.bfloat16)
    logits[0, :] = 0.5  # all tied
    logits[1, 5:9] = logits[1].max()  # ties at the top
    logits = logits.to(cuda)
    ids, w = kernels.route(logits, k)
    for row in range(rows):
        rid, rw = r.route(logits[row:row + 1], k)
        assert torch.equal(ids[row], rid[0]), row
        assert torch.equal(w[row], rw[0]), row
    oid, ow = moe.route(logits.view(torch.int16).cpu().numpy().view(np.uint16), k)
    np.testing.assert_array_equal(ids.cpu().numpy(), oid)
    np.testing.assert_allclose(w.cpu().numpy(), ow, rtol=0, atol=2 ** -8)


@pytest.mark.parametrize("k,H", [(8, 2048), (4, 300)])
def test_weighted_sum_bit_exact(cuda, k, H):
    kernels, r = lib(), ref()
    gen = torch.Generator().manual_seed(k + H)
    parts = torch.randn((3 * k, H), generator=gen).to(cuda)
    weights = torch.rand((3, k), generator=gen).to(cuda)
    out = kernels.weighted_sum(parts, weights)
    for row in range(3):
        expect = r.weighted_sum(parts[row * k:(row + 1) * k].contiguous(), weights[row].contiguous())
        assert torch.equal(out[row], expect[0])
    o = moe.weighted_sum(parts.cpu().numpy(), weights.cpu().numpy())
    np.testing.assert_allclose(out.float().cpu().numpy(), o, rtol=2 ** -7, atol=1e-6)


@pytest.mark.parametrize("mode", ["fp32", "bf16", "swiglu"])
def test_rotate_bit_exact(cuda, mode):
    kernels, r = lib(), ref()
    gen = torch.Generator().manual_seed(11)
    K = 768
    x = torch.randn((5, 2 * K if mode == "swiglu" else K), generator=gen)
    if mode == "bf16":
        x = x.to(torch.bfloat16)
    x = x.to(cuda)
    always = torch.ones((1,), dtype=torch.int32, device=cuda)
    out = kernels.rotate(x, always, swiglu=mode == "swiglu")
    assert torch.equal(out, r.rotate(x, always, swiglu=mode == "swiglu"))
    o = moe.rotate(x.float().cpu().numpy(), swiglu=mode == "swiglu")
    if mode == "swiglu":
        np.testing.assert_allclose(out.cpu().numpy(), o, rtol=1e-5, atol=1e-6)
    else:
        np.testing.assert_array_equal(out.cpu().numpy(), o)
    never = torch.zeros((1,), dtype=torch.int32, device=cuda)
    kernels.rotate(x, never, swiglu=mode == "swiglu")  # skipped: runs, writes nothing


def _state(layers, experts, count, device):
    st = moe.new_state(layers, experts, count)
    return {n: torch.from_numpy(v.copy()).to(device) for n, v in st.items()}, st


@pytest.mark.parametrize("cpu", [0, 1])
def test_resolve_trace_bit_exact(cuda, cpu):
    """1000 resolves (a seeded decode trace) through this kernel, the reference kernel and the oracle: identical
    plans and identical state after every call."""
    kernels, r = lib(), ref()
    layers, experts, count, k = 4, 32, 20, 8
    mine, st = _state(layers, experts, count, cuda)
    theirs, _ = _state(layers, experts, count, cuda)
    for s in (mine, theirs):
        s["share"].fill_(0.4)
        s["budget"].copy_(torch.tensor([6, 2]))
    st["share"][0] = 0.4
    st["budget"][:] = [6, 2]
    rng = np.random.default_rng(17)
    order = ("table", "owner", "score", "at", "pending", "clock", "budget", "reads", "step", "share")
    for call in range(1000):
        layer = call % layers
        ids_np = rng.choice(experts, size=k, replace=False)
        ids = torch.from_numpy(ids_np).to(cuda)
        p1 = kernels.resolve(ids, layer, layers, experts, 128, cpu, 6.0, *(mine[n] for n in order))
        p2 = r.resolve(ids, layer, layers, experts, 128, cpu, 6.0, *(theirs[n] for n in order))
        p3 = moe.resolve(st, ids_np, layer, layers, experts, 128, cpu, 6.0)
        assert torch.equal(p1, p2), call
        np.testing.assert_array_equal(p1.cpu().numpy(), p3, err_msg=f"call {call}")
        if cpu and call % 7 == 6:  # the host copies reserved slots in and refills the budget between steps
            for s in (mine, theirs):
                pend = s["pending"].nonzero().flatten()
                s["pending"][pend] = 0
                s["budget"][0] = 6
            st["pending"][:] = 0
            st["budget"][0] = 6
    for n in order:
        assert torch.equal(mine[n], theirs[n]), n
        if n == "score":  # numpy's exp2 may differ from CUDA's exp2f in the last place
            np.testing.assert_allclose(mine[n].cpu().numpy(), st[n], rtol=2e-5, err_msg=n)
        else:
            np.testing.assert_array_equal(mine[n].cpu().numpy(), st[n], err_msg=n)


# ---------------------------------------------------------------------------------------------------------------
def _plan_case(kind, device, E=16, slots=6, N=512, K=768):
    host = gd.rand_bank(kind, E, N, K, 31, "cpu")
    host = {n: t.pin_memory() for n, t in host.items()}
    slot = {n: torch.zeros((slots * t.shape[0] // E, *t.shape[1:]), dtype=t.dtype, device=device)
            for n, t in host.items()}
    for n, t in slot.items():  # slots 0..2 hold experts 9, 4, 1
        per = t.shape[0] // slots
        for s_, e in enumerate((9, 4, 1)):
            t[s_ * per:(s_ + 1) * per] = host[n][e * per:(e + 1) * per].to(device)
    ids = torch.tensor([4, 9, 12, 1, 7, 15], device=device)
    # codes: 0 = cached in its slot, 1 = from host memory (filling slot 3/4 or no slot)
    plan = torch.tensor([[1, 0], [0, 0], [3, 1], [2, 0], [-1, 1], [4, 1]], dtype=torch.int32, device=device)
    return host, slot, ids, plan, N, K


@pytest.mark.parametrize("kind", gd.KINDS)
@pytest.mark.parametrize("x_rows", ["one", "per_expert"])
def test_gemv_plan_matches_reference(cuda, kind, x_rows):
    kernels, r = lib(), ref()
    host, slot, ids, plan, N, K = _plan_case(kind, cuda)
    k = ids.shape[0]
    gen = torch.Generator().manual_seed(5)
    x = torch.randn((1 if x_rows == "one" else k, K), generator=gen).to(cuda)
    cb = gd.codebooks(kind, cuda)[0]
    slot2 = {n: t.clone() for n, t in slot.items()}
    took_over = torch.zeros((1,), dtype=torch.int32, device=cuda)
    if kind == "fp8":
        out = kernels.gemv_fp8(x, ids, plan, slot, host, N)
        expect = r.gemv_fp8(x, ids, plan, slot2, host, N)
    elif kind == "int8":
        out = kernels.gemv_int8(x, ids, plan, took_over, False, slot, host, N)
        expect = r.gemv_int8(x, ids, plan, took_over, False, slot2, host, N)
    else:
        out = kernels.gemv_codes(x, ids, plan, slot, host, cb, int(kind[1]), N)
        expect = r.gemv_codes(x, ids, plan, slot2, host, cb, int(kind[1]), N)
    torch.cuda.synchronize()
    assert gd.rel_l2(out, expect) < 1e-5
    for n in slot:  # the fills left the same bytes in the slots
        assert torch.equal(slot[n], slot2[n]), n
    o = moe.gemv(kind, x.cpu().numpy(), ids.cpu().numpy(), plan.cpu().numpy(), gd.to_np_bank(slot2),
                 gd.to_np_bank(host), N, None if cb is None else cb.cpu().numpy())
    assert gd.rel_l2(out, torch.from_numpy(o)) < 1e-5


def test_gemv_int8_cpu_codes(cuda):
    """Plan code 2 (an expert left to the CPU) gives zeros; with `late` only those run, and only after a takeover."""
    kernels = lib()
    host, slot, ids, plan, N, K = _plan_case("int8", cuda)
    plan[2, 1] = 2
    x = torch.randn((1, K), device=cuda)
    took = torch.zeros((1,), dtype=torch.int32, device=cuda)
    out = kernels.gemv_int8(x, ids, plan, took, False, slot, host, N)
    assert torch.count_nonzero(out[2]) == 0 and torch.count_nonzero(out[0]) > 0
    late = kernels.gemv_int8(x, ids, plan, took, True, slot, host, N)
    assert torch.count_nonzero(late) == 0
    took.fill_(1)
    late = kernels.gemv_int8(x, ids, plan, took, True, slot, host, N)
    assert torch.count_nonzero(late[2]) > 0 and torch.count_nonzero(late[0]) == 0


@pytest.mark.parametrize("kind", gd.KINDS)
def test_grouped_matches_reference(cuda, kind):
    kernels, r = lib(), ref()
    host, slot, _, _, N, K = _plan_case(kind, cuda)
    gen = torch.Generator().manual_seed(8)
    counts = [37, 0, 5, 64, 1, 130]
    rows = sum(counts)
    x = torch.randn((rows, K), generator=gen).to(cuda)
    first = np.cumsum([0] + counts[:-1])
    # (expert, slot, fill, first, rows): cached, host without slot, host filling slot 4, cached, host filling 5
    spec = [(9, 0, 0), (3, -1, 0), (12, -1, 0), (4, 1, 0), (7, 4, 1), (15, 5, 1)]
    groups = torch.tensor([(e, s_, f, int(first[i]), counts[i]) for i, (e, s_, f) in enumerate(spec) if counts[i]],
                          dtype=torch.int32, device=cuda)
    cb = gd.codebooks(kind, cuda)[0]
    slot2 = {n: t.clone() for n, t in slot.items()}
    if kind == "fp8":
        out = kernels.grouped_fp8(x, groups, slot, host, N)
        expect = r.grouped_fp8(x, groups, slot2, host, N)
    elif kind == "int8":
        out = kernels.grouped_int8(x, groups, slot, host, N)
        expect = r.grouped_int8(x, groups, slot2, host, N)
    else:
        out = kernels.grouped_codes(x, groups, slot, host, cb, int(kind[1]), N)
        expect = r.grouped_codes(x, groups, slot2, host, cb, int(kind[1]), N)
    torch.cuda.synchronize()
    assert gd.rel_l2(out, expect) < 1e-5
    for n in slot:
        assert torch.equal(slot[n], slot2[n]), n
