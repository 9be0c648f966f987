"""One rank of the multi-GPU expert-parallel check (run by tests/test_ep_gpu.py under torchrun): each rank holds a
block of the experts; the exchanged result must equal the single-GPU decode of the whole banks."""
import datetime
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "comfyui-drama3_b200"), str(ROOT / "tests")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import gpu_data as gd  # noqa: E402
from drama3_b200 import ep, kernels  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    E, H, I = 16, 2048, 768
    worst, same = 0.0, True
    peer = ep.PeerExchange(16, H, device)
    for kind in ("fp8c", "fp8", "w4a8"):
        full = (gd.rand_bank(kind, E, 2 * I, H, 80, device), gd.rand_bank(kind, E, H, I, 81, device))
        local = ep.local_banks(full, E, rank, world)
        layer = ep.ExpertParallelDecode(kind, local, E)
        fused = ep.ExpertParallelDecode(kind, local, E, peer=peer)
        for M in (1, 16, 7):
            x = gd.rand_rows(M, H, 90 + M, device)
            ids, w = gd.rand_routing(M, E, 8, 95 + M, device)
            got = layer(x, ids, w)
            want = kernels.moe_decode(kind, x, ids, w, full)
            worst = max(worst, gd.rel_l2(got.float(), want.float()))
            # the peer exchange: the same rank-order sum as the all-gather, bit for bit, call after call
            for _ in range(3):
                same = same and torch.equal(fused(x, ids, w), got)
    # graph-captured steps through the peer exchange (the call counter lives on the device)
    kind = "fp8c"
    full = (gd.rand_bank(kind, E, 2 * I, H, 82, device), gd.rand_bank(kind, E, H, I, 83, device))
    fused = ep.ExpertParallelDecode(kind, ep.local_banks(full, E, rank, world), E, peer=peer)
    x = gd.rand_rows(16, H, 99, device)
    ids, w = gd.rand_routing(16, E, 8, 98, device)
    want = kernels.moe_decode(kind, x, ids, w, full)
    fused(x, ids, w)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = fused(x, ids, w)
        out2 = fused(x, ids, w)
    for _ in range(5):
        graph.replay()
    torch.cuda.synchronize()
    worst = max(worst, gd.rel_l2(out.float(), want.float()), gd.rel_l2(out2.float(), want.float()))
    fault = kernels._lib.take_fault()
    del graph
    peer.close()
    ok = torch.tensor([1.0 if worst <= 1e-3 and same and fault == 0 else 0.0], device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(f"EP_RESULT world={world} worst_rel_l2={worst:.3e} peer_same={same} fault={fault} "
              f"ok={bool(ok.item())}", flush=True)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok.item() else 1)


if __name__ == "__main__":
    main()
