"""Expert parallelism for the routed-expert decode over the GPUs of one node (one process per GPU,
torch.distributed): rank r holds a contiguous block of the experts, every rank sees all rows (lines are
replicated), runs the fused decode over its own experts only and produces an fp32 partial [M, H]; the partials are
gathered and summed in rank order, then rounded to bf16 once, so every rank ends with the same output.

The reference runs on one GPU; this is the multi-GPU layout of its decode step (experts split, tokens replicated,
partial combines reduced). The exchange is a 128 KB all-gather per layer at 16 lines over NCCL (NVLink).
"""
import torch
import torch.distributed as dist

from . import kernels


def expert_range(num_experts, rank, world):
    """(first, count) of the contiguous block of experts rank `rank` of `world` holds: the blocks differ by at most
    one expert and cover [0, num_experts) in rank order."""
    base, extra = divmod(num_experts, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def local_banks(banks, num_experts, rank, world):
    """This rank's slice of whole banks (gate_up, down) laid out [E * rows, ...]: every per-row field sliced by expert
    (fp8 128 x 128 block scales by blocks of rows)."""
    first, count = expert_range(num_experts, rank, world)
    out = []
    for bank in banks:
        sl = {}
        for name, t in bank.items():
            per = t.shape[0] // num_experts
            sl[name] = t[first * per:(first + count) * per]
        out.append(sl)
    return tuple(out)


def sum_in_rank_order(gathered):
    """gathered [world, M, H] fp32 -> [M, H] fp32: ((p0 + p1) + p2) + ..., the same on every rank."""
    out = gathered[0].clone()
    for r in range(1, gathered.shape[0]):
        out += gathered[r]
    return out


class ExpertParallelDecode:
    """The decode of one MoE layer with this rank's experts. `decode_fn(x, ids, weights) -> fp32 [M, H]` replaces
    the GPU kernel (kernels.moe_decode_ep over `banks`) when given, so the exchange can be exercised on CPU ranks."""

    def __init__(self, kind, banks, num_experts, group=None, codebooks=(None, None), decode_fn=None):
        self.kind, self.banks, self.num_experts, self.group = kind, banks, num_experts, group
        self.codebooks, self.decode_fn = codebooks, decode_fn
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.e_first, self.e_count = expert_range(num_experts, self.rank, self.world)
        self.workspace = {}

    def partial(self, x, ids, weights):
        if self.decode_fn is not None:
            return self.decode_fn(x, ids, weights)
        key = (x.device, x.shape[0], ids.shape[-1])
        if key not in self.workspace:
            wkey = kernels._lib.WEIGHT_KEY[self.kind]
            e_local = self.banks[1][wkey].shape[0] // x.shape[1]
            inter = self.banks[0][wkey].shape[0] // (2 * e_local)
            self.workspace[key] = kernels.decode_workspace(x.shape[0], ids.shape[-1], inter, x.device)
        return kernels.moe_decode_ep(self.kind, x, ids, weights, self.banks, self.e_first, self.num_experts,
                                     self.codebooks, workspace=self.workspace[key])

    def __call__(self, x, ids, weights):
        """[M, H] bfloat16, the same on every rank: the whole layer's decode of rows x [M, H] routed to ids [M, k]."""
        part = self.partial(x, ids, weights).float().contiguous()
        gathered = torch.empty((self.world * part.shape[0], part.shape[1]), dtype=part.dtype, device=part.device)
        dist.all_gather_into_tensor(gathered, part, group=self.group)
        return sum_in_rank_order(gathered.view(self.world, *part.shape)).to(torch.bfloat16)
