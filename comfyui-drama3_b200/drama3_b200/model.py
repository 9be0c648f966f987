"""The MoE block of the reference model (drama3/model.py:40-124) around this library's expert path.

`SparseMoeBlock` keeps the reference's routing and shared expert; its routed experts are `FP8Experts`,
`Experts` (quantized banks the kernels read) or an `OffloadedExperts` stand-in. One change on the hot path: the decode
rows of lines batched together ([B, 1, H]) are routed together by one `kernels.route` launch and run through the
experts as one call (one fused decode kernel for up to 16 rows), where the reference loops the block row by row
(drama3/model.py:111-113). Routing and combine keep the reference's numerics, so each row's result is the one the
per-row loop gives up to the fused kernel's summation order.
"""
from types import SimpleNamespace

import torch
import torch.nn as nn

from . import kernels
from .offload import FP8Experts, MAX_DECODE_ROWS, capturing, kernel_bank, resident_decode_lines, resident_prefill, \
    fused_decode_fits


def swiglu(h):
    """SiLU of the first half times the second half (the gate rows come first in every fused bank)."""
    gate, up = h.chunk(2, dim=-1)
    return nn.functional.silu(gate) * up


class SharedExpert(nn.Module):
    """The dense shared expert: down(SwiGLU(gate_up(x))) (drama3/model.py:40-47)."""

    def __init__(self, hidden, intermediate, device=None, dtype=None):
        super().__init__()
        self.gate_up_proj = nn.Linear(hidden, 2 * intermediate, bias=False, device=device, dtype=dtype)
        self.down_proj = nn.Linear(intermediate, hidden, bias=False, device=device, dtype=dtype)

    def forward(self, x):
        return self.down_proj(swiglu(self.gate_up_proj(x)))


class Experts(nn.Module):
    """Routed experts in quantized banks (drama3/model.py:50-89): `gate_up_proj` and `down_proj` are modules whose
    `.weight` is a flat bank the kernels read (`kernel_bank`: int8 ConvRot, W4A8, W6A8)."""

    def __init__(self, num_experts, gate_up_proj, down_proj):
        super().__init__()
        self.num_experts = num_experts
        self.gate_up_proj = gate_up_proj
        self.down_proj = down_proj
        self._workspace = {}

    def sync_free(self, device):
        return (kernels.available(device) and kernel_bank(self.gate_up_proj.weight) is not None
                and kernel_bank(self.down_proj.weight) is not None)

    def forward(self, x, topk_idx, topk_weight):
        weights = self.gate_up_proj.weight, self.down_proj.weight
        found = [kernel_bank(w) for w in weights]
        if None in found:
            raise ValueError("these experts are not in a layout the kernels read")
        kernels.available(x.device)
        kind, banks = found[0][0], [fields for _, fields in found]
        rows = [bank["_qdata"].shape[0] // self.num_experts for bank in banks]
        codebooks = [w._params.codebook for w in weights] if kind == "w4" else (None, None)
        M, k = topk_idx.shape
        hidden, intermediate = rows[1], rows[0] // 2
        if M == 1 or fused_decode_fits(hidden, intermediate, M, k):
            ws = None
            if fused_decode_fits(hidden, intermediate, M, k):
                key = (x.device, M, k)
                if key not in self._workspace:
                    self._workspace[key] = kernels.decode_workspace(M, k, intermediate, x.device)
                ws = self._workspace[key]
            return resident_decode_lines(x, topk_idx, topk_weight, banks, rows, kind, codebooks, workspace=ws)
        return resident_prefill(x, topk_idx, topk_weight, banks, rows, kind, codebooks, self.num_experts,
                                sync_free=capturing(x))


class SparseMoeBlock(nn.Module):
    """Softmax router over all experts, renormalized top-k, plus a sigmoid-gated shared expert
    (drama3/model.py:92-124). `config` carries text.hidden_size, num_experts, num_experts_per_tok,
    moe_intermediate_size, shared_expert_intermediate_size and fp8_experts; `experts` may be passed in (an
    `Experts` or an `OffloadedExperts`) instead of the FP8Experts the config would make."""

    def __init__(self, config, device=None, dtype=None, experts=None):
        super().__init__()
        hidden = config.text.hidden_size
        self.top_k = config.num_experts_per_tok
        self.gate = nn.Linear(hidden, config.num_experts, bias=False, device=device, dtype=dtype)
        if experts is None:
            if not config.fp8_experts:
                raise ValueError("pass the quantized `experts` module: only FP8 experts are built from the config")
            experts = FP8Experts(config.num_experts, hidden, config.moe_intermediate_size, device=device, dtype=dtype)
        self.experts = experts
        self.shared_expert = SharedExpert(hidden, config.shared_expert_intermediate_size, device=device, dtype=dtype)
        self.shared_expert_gate = nn.Linear(hidden, 1, bias=False, device=device, dtype=dtype)

    def route(self, logits, decode):
        """(ids, weights) of router logits [rows, E]: the route kernel for decode rows (bit-identical to the
        reference's), the reference's softmax / top-k / renormalization expression for a prompt's rows
        (drama3/model.py:115-121)."""
        if decode:
            return kernels.route(logits, self.top_k)
        weights, ids = torch.softmax(logits.float(), dim=-1).topk(self.top_k, dim=-1)
        return ids, (weights / weights.sum(dim=-1, keepdim=True)).to(logits.dtype)

    def forward(self, x, norm=None):
        if norm is not None:
            x = norm(x)
        flat = x.reshape(-1, x.shape[-1])
        logits = self.gate(flat)
        # decode: one row, or the rows of lines decoded together ([B, 1, H]) routed and run at once
        decode = flat.shape[0] == 1 or (x.dim() == 3 and x.shape[1] == 1 and flat.shape[0] <= MAX_DECODE_ROWS)
        topk_idx, topk_weight = self.route(logits, decode)
        if decode and flat.shape[0] > 1 and not isinstance(self.experts, (FP8Experts, Experts)):
            # a slot-cache store decodes one row at a time
            out = torch.cat([self.experts(flat[r:r + 1], topk_idx[r:r + 1], topk_weight[r:r + 1])
                             for r in range(flat.shape[0])])
        else:
            out = self.experts(flat, topk_idx, topk_weight)
        out = out + torch.sigmoid(self.shared_expert_gate(flat)) * self.shared_expert(flat)
        return out.view_as(x)


def block_config(hidden=2048, num_experts=128, top_k=8, intermediate=768, shared_intermediate=512, fp8=True):
    """A config object with the fields SparseMoeBlock reads (defaults: the benchmark's layer shape)."""
    return SimpleNamespace(text=SimpleNamespace(hidden_size=hidden), num_experts=num_experts,
                           num_experts_per_tok=top_k, moe_intermediate_size=intermediate,
                           shared_expert_intermediate_size=shared_intermediate, fp8_experts=fp8)
