"""One rank of the multi-GPU expert-parallel prompt pass check (run by tests/test_ep_gpu.py under torchrun): the
prompt's rows split by rank, each rank holding a block of the experts; every rank's rows must come back equal, bit
for bit, to the one-GPU prompt pass of the same rows over the whole banks."""
import datetime
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "comfyui-drama3_b200"), str(ROOT / "tests")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

import gpu_data as gd  # noqa: E402
from drama3_b200 import ep, kernels, offload  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    E, H, I, T = 32, 2048, 768, 1024
    same = True
    for kind in ("fp8c", "w6a8", "fp8"):
        full = (gd.rand_bank(kind, E, 2 * I, H, 120, device), gd.rand_bank(kind, E, H, I, 121, device))
        layer = ep.ExpertParallelPrefill(kind, ep.local_banks(full, E, rank, world), E, (2 * I, H))
        x = gd.rand_rows(T, H, 122, device)
        ids, w = gd.rand_routing(T, E, 8, 123, device)
        w = w.to(torch.bfloat16)
        lo, hi = T * rank // world, T * (rank + 1) // world
        got = layer(x[lo:hi], ids[lo:hi], w[lo:hi])
        want = offload.resident_prefill(x[lo:hi], ids[lo:hi], w[lo:hi], full, (2 * I, H), kind, (None, None), E)
        same = same and torch.equal(got, want)
        # fixed blocks (no split sizes read back), eagerly and captured in a CUDA graph
        fixed = ep.ExpertParallelPrefill(kind, ep.local_banks(full, E, rank, world), E, (2 * I, H),
                                         capacity=(T // world + 1) * 8)
        same = same and torch.equal(fixed(x[lo:hi], ids[lo:hi], w[lo:hi]), want)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fixed(x[lo:hi], ids[lo:hi], w[lo:hi])
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            captured = fixed(x[lo:hi], ids[lo:hi], w[lo:hi])
        graph.replay()
        torch.cuda.synchronize()
        same = same and torch.equal(captured, want) and int(fixed.dropped) == 0
        del graph
    torch.cuda.synchronize()
    fault = kernels._lib.take_fault()
    ok = torch.tensor([1.0 if same and fault == 0 else 0.0], device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if rank == 0:
        print(f"EP_PREFILL_RESULT world={world} same={same} fault={fault} ok={bool(ok.item())}", flush=True)
    dist.barrier()
    dist.destroy_process_group()
    sys.exit(0 if ok.item() else 1)


if __name__ == "__main__":
    main()
