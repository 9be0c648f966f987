"""Expert parallelism across the GPUs of this node (2 or more): each rank holds a block of the experts, and the
exchanged decode equals the single-GPU decode of the whole banks. Skipped with fewer than 2 GPUs."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def run_workers(script):
    """stdout of `script` run on every GPU of this node under torchrun (skipped with fewer than 2)."""
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs 2 or more GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={min(n, 8)}", "--master-addr", "127.0.0.1", "--master-port", str(port),
           str(ROOT / "tests" / script)]
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=400)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-3000:]
    return proc.stdout


def test_expert_parallel_decode_matches_one_gpu():
    assert "ok=True" in run_workers("ep_worker.py")


def test_expert_parallel_prefill_matches_one_gpu():
    assert "ok=True" in run_workers("ep_prefill_worker.py")


# ---- the peer exchange's kernels on one GPU: ranks emulated by areas in this GPU's memory, their calls issued one
# after another on one stream (no kernel waits on one still running)

import gpu_data as gd  # noqa: E402
from drama3_b200 import _lib, ep, kernels, offload  # noqa: E402

E, H, I = 16, 2048, 768


def local_exchanges(world, m_max, device):
    """world exchange areas in this GPU's memory and each emulated rank's device struct over all of them."""
    size, flags_offset = ep.exchange_layout(world, m_max, H)
    areas = [torch.zeros((size,), dtype=torch.uint8, device=device) for _ in range(world)]
    ptrs = [a.data_ptr() for a in areas]
    structs = [torch.frombuffer(bytearray(ep.exchange_struct(ptrs, flags_offset, r, m_max, H)),
                                dtype=torch.uint8).to(device) for r in range(world)]
    return areas, structs


@pytest.mark.parametrize("kind", ["fp8c", "w4a8"])
def test_exchange_one_rank_equals_moe_decode(cuda, monkeypatch, kind):
    """World 1: the partial pushed into the area and reduced is the tensor-core decode's output bit for bit (the
    exchanged decode runs that kernel at every line count; D3_DECODE_GV=0 makes moe_decode run it at one line too),
    over calls of both parities and fewer lines than the area holds."""
    monkeypatch.setenv("D3_DECODE_GV", "0")
    banks = (gd.rand_bank(kind, E, 2 * I, H, 200, cuda), gd.rand_bank(kind, E, H, I, 201, cuda))
    areas, (st,) = local_exchanges(1, 16, cuda)  # the areas stay referenced while the structs point at them
    _lib.take_fault()
    for call, M in enumerate((16, 1, 5, 16)):
        x = gd.rand_rows(M, H, 210 + call, cuda)
        ids, w = gd.rand_routing(M, E, 8, 220 + call, cuda)
        assert kernels.moe_decode_ep(kind, x, ids, w, banks, 0, E, exchange=st) is None
        got = kernels.ep_reduce(st, M, H)
        assert torch.equal(got, kernels.moe_decode(kind, x, ids, w, banks)), call
    assert _lib.take_fault() == 0


@pytest.mark.parametrize("world", [2, 3])
def test_exchange_ranks_on_one_gpu(cuda, world):
    """world emulated ranks, each with its block of the experts: every rank's reduce returns the rank-order sum of
    the partials (the all-gather exchange's result) bit for bit, and the single-GPU decode within 1e-3."""
    kind = "fp8c"
    full = (gd.rand_bank(kind, E, 2 * I, H, 230, cuda), gd.rand_bank(kind, E, H, I, 231, cuda))
    areas, structs = local_exchanges(world, 16, cuda)  # kept referenced while the structs point at them
    _lib.take_fault()
    for call, M in enumerate((16, 3, 16)):
        x = gd.rand_rows(M, H, 240 + call, cuda)
        ids, w = gd.rand_routing(M, E, 8, 250 + call, cuda)
        partials = []
        for r in range(world):
            first = ep.expert_range(E, r, world)[0]
            banks = ep.local_banks(full, E, r, world)
            partials.append(kernels.moe_decode_ep(kind, x, ids, w, banks, first, E))
            kernels.moe_decode_ep(kind, x, ids, w, banks, first, E, exchange=structs[r])
        want = ep.sum_in_rank_order(torch.stack(partials)).to(torch.bfloat16)
        for r in range(world):
            assert torch.equal(kernels.ep_reduce(structs[r], M, H), want), (call, r)
        assert gd.rel_l2(want.float(), kernels.moe_decode(kind, x, ids, w, full).float()) <= 1e-3
    assert _lib.take_fault() == 0


def test_exchange_reduce_times_out_without_peer(cuda):
    """A reduce whose peer never pushes gives up after its wait limit: fault bit 1, zeros out, the context usable."""
    areas, structs = local_exchanges(2, 1, cuda)
    _lib.take_fault()
    out = kernels.ep_reduce(structs[0], 1, H, out=torch.full((1, H), 7.0, dtype=torch.bfloat16, device=cuda))
    torch.cuda.synchronize()
    assert _lib.take_fault() == 1 and not out.any()
    assert torch.ones(4, device=cuda).sum().item() == 4


def test_exchange_geometry_checked(cuda):
    """More lines than the area holds: nothing is pushed or awaited, fault bit 16, zeros out."""
    kind = "fp8c"
    banks = (gd.rand_bank(kind, E, 2 * I, H, 260, cuda), gd.rand_bank(kind, E, H, I, 261, cuda))
    areas, (st,) = local_exchanges(1, 2, cuda)
    x = gd.rand_rows(4, H, 262, cuda)
    ids, w = gd.rand_routing(4, E, 8, 263, cuda)
    _lib.take_fault()
    kernels.moe_decode_ep(kind, x, ids, w, banks, 0, E, exchange=st)
    out = kernels.ep_reduce(st, 4, H)
    torch.cuda.synchronize()
    assert _lib.take_fault() == 16 and not out.any()
    assert not areas[0][:-256].any()


@pytest.mark.parametrize("kind", ["fp8c", "w6a8", "fp8", "w4"])
def test_prefill_pairs_of_emulated_ranks_equal_one_gpu(cuda, kind):
    """The expert-parallel prompt pass's local step on one GPU: the pairs of each of 3 emulated ranks through that
    rank's block of the experts (ep.local_pairs), put together and combined, equal the one-GPU prompt pass bit for
    bit."""
    T, k, world = 512, 8, 3
    full = (gd.rand_bank(kind, E * 2, 2 * I, H, 130, cuda), gd.rand_bank(kind, E * 2, H, I, 131, cuda))
    cbs = gd.codebooks(kind, cuda)
    x = gd.rand_rows(T, H, 132, cuda)
    ids, w = gd.rand_routing(T, E * 2, k, 133, cuda)
    w = w.to(torch.bfloat16)
    _lib.take_fault()
    want = offload.resident_prefill(x, ids, w, full, (2 * I, H), kind, cbs, E * 2)
    flat = ids.reshape(-1)
    owner = ep.expert_owner(flat, E * 2, world)
    pair_out = torch.zeros((T * k, H), dtype=torch.float32, device=cuda)
    for r in range(world):
        first, count = ep.expert_range(E * 2, r, world)
        sel = (owner == r).nonzero().squeeze(1)
        pair_out[sel] = ep.local_pairs(kind, ep.local_banks(full, E * 2, r, world), count, (2 * I, H), cbs,
                                       x[sel // k], (flat[sel] - first).to(torch.int32))
    got = kernels.prefill_combine(pair_out, torch.arange(T * k, device=cuda).view(T, k), w)
    torch.cuda.synchronize()
    assert _lib.take_fault() == 0
    assert torch.equal(got, want)


def test_local_pairs_leave_padding_rows_out(cuda):
    """Rows marked -1 (the padding of the fixed-block exchange) are left out of the grouped GEMMs without a fault;
    the other rows equal the same call without the padding, bit for bit."""
    kind, R, count = "fp8c", 300, 11
    full = (gd.rand_bank(kind, E * 2, 2 * I, H, 140, cuda), gd.rand_bank(kind, E * 2, H, I, 141, cuda))
    local = ep.local_banks(full, E * 2, 0, 3)
    x = gd.rand_rows(R, H, 142, cuda)
    ids = torch.randint(0, count, (R,), generator=torch.Generator().manual_seed(143)).to(torch.int32).to(cuda)
    pad = torch.zeros(R, dtype=torch.bool)
    pad[::3] = True
    pad = pad.to(cuda)
    _lib.take_fault()
    padded = ep.local_pairs(kind, local, count, (2 * I, H), (None, None), x,
                            torch.where(pad, torch.full_like(ids, -1), ids))
    keep = (~pad).nonzero().squeeze(1)
    plain = ep.local_pairs(kind, local, count, (2 * I, H), (None, None), x[keep], ids[keep])
    torch.cuda.synchronize()
    assert _lib.take_fault() == 0
    assert torch.equal(padded[keep], plain)
