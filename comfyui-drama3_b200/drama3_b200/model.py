"""The MoE block of the reference model (drama3/model.py:40-124) around this library's expert path.

Same classes and constructors as the reference: `SharedExpert(hidden, intermediate, device, dtype, ops)`,
`Experts(num_experts, hidden, intermediate, device, dtype, ops)` and `SparseMoeBlock(config, device, dtype, ops)`.
`ops` is the factory namespace the reference takes from ComfyUI (`ops.Linear`, `ops.MoEExperts`); without ComfyUI,
`ops=None` uses `OPS`: torch's Linear and `MoEBank`, a module whose `weight` takes a quantized bank (a converted
checkpoint's QuantizedTensor or `pack.packed_weight`). The routed experts are FP8Experts (config.fp8_experts;
per-channel scales with config.fp8_per_channel), Experts over quantized banks, or any module passed as `experts=`
(an `OffloadedExperts` of a slot-cache store).

Changes on the hot path: the decode rows of lines batched together ([B, 1, H]) are routed together and run through
the experts as one call (one fused decode kernel for up to 16 rows), where the reference loops the block row by row
(drama3/model.py:111-113); and for decode rows the router linear with its routing is one launch (`kernels.router`)
and the sigmoid-gated shared expert two (`kernels.shared_expert`, added into the experts' output), where torch runs
about a dozen. Routing keeps the reference's rule on the router's bf16 logits (whose fp32 sums may differ from
cuBLAS's in the last bf16 place), and each row's result is the one the per-row loop gives up to summation order.
"""
import contextlib
from types import SimpleNamespace

import torch
import torch.nn as nn

from . import kernels
from .offload import (FP8Experts, MAX_DECODE_ROWS, capturing, fused_decode_fits, kernel_bank, resident_decode_lines,
                      resident_prefill, swiglu)


class MoEBank(nn.Module):
    """Stand-in for ComfyUI's `ops.MoEExperts(num_experts, in_features, out_features, bias, device, dtype)`: holds one
    flat expert bank in `weight` ([num_experts * out_features] rows of in_features columns, packed), assigned after
    construction as a converted checkpoint's loader assigns it. No bias (the reference builds none)."""

    def __init__(self, num_experts, in_features, out_features, bias=False, device=None, dtype=None):
        super().__init__()
        if bias:
            raise ValueError("routed expert banks carry no bias")
        self.num_experts, self.in_features, self.out_features = num_experts, in_features, out_features
        self.weight = None


OPS = SimpleNamespace(Linear=nn.Linear, MoEExperts=MoEBank)


def _bank_of(module, x):
    """Context manager giving the module's bank on x's device: ComfyUI's `bank_resident` (its dynamic VRAM loads
    the bank for the call) where the module has it, else the module's `weight` as it is."""
    if hasattr(module, "bank_resident"):
        @contextlib.contextmanager
        def resident():
            with module.bank_resident(x) as loaded:
                yield loaded._resident_bank[0]
        return resident()
    return contextlib.nullcontext(module.weight)


class SharedExpert(nn.Module):
    """The dense shared expert: down(SwiGLU(gate_up(x))) (drama3/model.py:40-47)."""

    def __init__(self, hidden, intermediate, device=None, dtype=None, ops=None):
        super().__init__()
        ops = ops or OPS
        self.gate_up_proj = ops.Linear(hidden, 2 * intermediate, bias=False, device=device, dtype=dtype)
        self.down_proj = ops.Linear(intermediate, hidden, bias=False, device=device, dtype=dtype)

    def forward(self, x):
        return self.down_proj(swiglu(self.gate_up_proj(x)))


class Experts(nn.Module):
    """Routed experts in quantized banks (drama3/model.py:50-89): `gate_up_proj` and `down_proj` are `ops.MoEExperts`
    modules whose weight is a flat bank the kernels read (`kernel_bank`: int8 ConvRot, W4A8, W6A8, and the BASELINE
    int8-activation layouts). Other layouts raise: there is no torch fallback."""

    def __init__(self, num_experts, hidden, intermediate, device=None, dtype=None, ops=None):
        super().__init__()
        ops = ops or OPS
        self.num_experts = num_experts
        self.gate_up_proj = ops.MoEExperts(num_experts, hidden, 2 * intermediate, bias=False, device=device,
                                           dtype=dtype)
        self.down_proj = ops.MoEExperts(num_experts, intermediate, hidden, bias=False, device=device, dtype=dtype)
        self._workspace = {}

    def sync_free(self, device):
        return (kernels.available(device) and kernel_bank(self.gate_up_proj.weight) is not None
                and kernel_bank(self.down_proj.weight) is not None)

    def _workspace_for(self, M, k, intermediate, device):
        key = (torch.device(device), M, k)
        if key not in self._workspace:
            self._workspace[key] = kernels.decode_workspace(M, k, intermediate, device)
        return self._workspace[key]

    def forward(self, x, topk_idx, topk_weight):
        with _bank_of(self.gate_up_proj, x) as w13, _bank_of(self.down_proj, x) as w2:
            found = [kernel_bank(w) for w in (w13, w2)]
            if None in found:
                raise ValueError("these experts are not in a layout the kernels read")
            kernels.available(x.device)
            kind, banks = found[0][0], [fields for _, fields in found]
            rows = [bank["_qdata"].shape[0] // self.num_experts for bank in banks]
            codebooks = [w._params.codebook for w in (w13, w2)] if kind == "w4" else (None, None)
            M, k = topk_idx.shape
            hidden, intermediate = rows[1], rows[0] // 2
            fits = fused_decode_fits(hidden, intermediate, M, k)
            if M == 1 or fits:
                ws = self._workspace_for(M, k, intermediate, x.device) if fits else None
                return resident_decode_lines(x, topk_idx, topk_weight, banks, rows, kind, codebooks, workspace=ws)
            return resident_prefill(x, topk_idx, topk_weight, banks, rows, kind, codebooks, self.num_experts,
                                    sync_free=capturing(x))


class SparseMoeBlock(nn.Module):
    """Softmax router over all experts, renormalized top-k, plus a sigmoid-gated shared expert
    (drama3/model.py:92-124). `config` carries text.hidden_size, num_experts, num_experts_per_tok,
    moe_intermediate_size, shared_expert_intermediate_size and fp8_experts (and, optionally, fp8_per_channel).
    `experts`, when given, replaces the routed experts the config would make (an `OffloadedExperts`, say)."""

    def __init__(self, config, device=None, dtype=None, ops=None, experts=None):
        super().__init__()
        ops = ops or OPS
        hidden = config.text.hidden_size
        self.top_k = config.num_experts_per_tok
        self.gate = ops.Linear(hidden, config.num_experts, bias=False, device=device, dtype=dtype)
        if experts is None:
            if config.fp8_experts:
                experts = FP8Experts(config.num_experts, hidden, config.moe_intermediate_size, device=device,
                                     dtype=dtype, per_channel=getattr(config, "fp8_per_channel", False))
            else:
                experts = Experts(config.num_experts, hidden, config.moe_intermediate_size, device=device,
                                  dtype=dtype, ops=ops)
        self.experts = experts
        self.shared_expert = SharedExpert(hidden, config.shared_expert_intermediate_size, device=device, dtype=dtype,
                                          ops=ops)
        self.shared_expert_gate = ops.Linear(hidden, 1, bias=False, device=device, dtype=dtype)
        # decode rows: the router (linear + routing) in one launch and the gated shared expert in two, where the
        # modules are plain bias-free bf16 linears of shapes the kernels take; False keeps torch's chain
        self.fused = True

    def route(self, logits, decode):
        """(ids, weights) of router logits [rows, E]: the route kernel for decode rows (bit-identical to the
        reference's), the reference's softmax / top-k / renormalization expression for a prompt's rows
        (drama3/model.py:115-121)."""
        if decode:
            return kernels.route(logits, self.top_k)
        weights, ids = torch.softmax(logits.float(), dim=-1).topk(self.top_k, dim=-1)
        return ids, (weights / weights.sum(dim=-1, keepdim=True)).to(logits.dtype)

    def _plain(self, *linears):
        """Whether these modules are bias-free bf16 torch linears on a CUDA device (what the fused kernels read)."""
        return all(type(m) is nn.Linear and m.bias is None and m.weight.dtype == torch.bfloat16 and m.weight.is_cuda
                   for m in linears)

    def fused_router(self, flat):
        return (self.fused and flat.dtype == torch.bfloat16 and self._plain(self.gate)
                and kernels.router_fits(flat.shape[0], flat.shape[1], self.gate.weight.shape[0], self.top_k))

    def fused_shared(self, flat):
        se = self.shared_expert
        return (self.fused and flat.dtype == torch.bfloat16
                and self._plain(se.gate_up_proj, se.down_proj, self.shared_expert_gate)
                and kernels.shared_expert_fits(flat.shape[0], flat.shape[1], se.down_proj.weight.shape[1]))

    def forward(self, x, norm=None):
        if norm is not None:
            x = norm(x)
        flat = x.reshape(-1, x.shape[-1])
        # decode: one row, or the rows of lines decoded together ([B, 1, H]) routed and run at once
        decode = flat.shape[0] == 1 or (x.dim() == 3 and x.shape[1] == 1 and flat.shape[0] <= MAX_DECODE_ROWS)
        if decode and self.fused_router(flat):
            topk_idx, topk_weight = kernels.router(flat, self.gate.weight, self.top_k)
        else:
            topk_idx, topk_weight = self.route(self.gate(flat), decode)
        if decode and flat.shape[0] > 1 and not isinstance(self.experts, (FP8Experts, Experts)):
            # a slot-cache store decodes one row at a time
            out = torch.cat([self.experts(flat[r:r + 1], topk_idx[r:r + 1], topk_weight[r:r + 1])
                             for r in range(flat.shape[0])])
        else:
            out = self.experts(flat, topk_idx, topk_weight)
        if decode and self.fused_shared(flat) and out.dtype == torch.bfloat16 and out.is_contiguous():
            se = self.shared_expert
            out = kernels.shared_expert(flat, se.gate_up_proj.weight, se.down_proj.weight,
                                        self.shared_expert_gate.weight, out)
        else:
            out = out + torch.sigmoid(self.shared_expert_gate(flat)) * self.shared_expert(flat)
        return out.view_as(x)


def block_config(hidden=2048, num_experts=128, top_k=8, intermediate=768, shared_intermediate=512, fp8=True,
                 per_channel=False):
    """A config object with the fields SparseMoeBlock reads (defaults: the benchmark's layer shape)."""
    return SimpleNamespace(text=SimpleNamespace(hidden_size=hidden), num_experts=num_experts,
                           num_experts_per_tok=top_k, moe_intermediate_size=intermediate,
                           shared_expert_intermediate_size=shared_intermediate, fp8_experts=fp8,
                           fp8_per_channel=per_channel)
