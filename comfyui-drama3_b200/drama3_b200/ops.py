"""The library's kernels as torch.library custom ops, torch.ops.drama3_b200.<name>, for callers that build graphs
(torch.compile, CUDA graph capture, exported programs): every op takes and returns plain tensors, ints, bools and
strings, writes fresh outputs (shared_expert updates `out` in place and declares it), and has a fake implementation
that gives the output shapes and dtypes without running anything. Each op calls the matching function of
drama3_b200.kernels; there is no CPU or torch fallback, so a call on tensors that are not on a B200 fails loudly.

Import this module once to register the ops. The expert banks of moe_decode and grouped_mma are passed field by
field: `w` is the bank's weight rows ("weight" for fp8 / fp8c, "_qdata" for the integer layouts), `scale` its scales
and `s_channel` the W4 / W6 per-row factors (None for the other layouts), as drama3/offload.py:72-90 names them."""
from typing import Optional

import torch
from torch import Tensor

from . import _lib, kernels

NAMESPACE = "drama3_b200"
OPS = ("route", "weighted_sum", "rotate", "router", "shared_expert", "moe_decode", "grouped_mma", "prefill_plan",
       "prefill_combine")


def _fields(kind, w, scale, s_channel):
    fields = {_lib.WEIGHT_KEY[kind]: w, "scale": scale}
    if s_channel is not None:
        fields["s_channel"] = s_channel
    return fields


# ---- routing and the per-kernel reference API (drama3/kernels.py:636-661)

@torch.library.custom_op(f"{NAMESPACE}::route", mutates_args=())
def route(logits: Tensor, k: int) -> tuple[Tensor, Tensor]:
    """(ids [rows, k] int64, weights [rows, k] float32) of bfloat16 router logits: kernels.route."""
    return kernels.route(logits, k)


@route.register_fake
def _(logits, k):
    rows = logits.shape[0]
    return logits.new_empty((rows, k), dtype=torch.int64), logits.new_empty((rows, k), dtype=torch.float32)


@torch.library.custom_op(f"{NAMESPACE}::weighted_sum", mutates_args=())
def weighted_sum(parts: Tensor, weights: Tensor) -> Tensor:
    """[rows, H] bfloat16: parts [rows * k, H] float32 summed per row by weights [rows, k], in rank order."""
    return kernels.weighted_sum(parts, weights)


@weighted_sum.register_fake
def _(parts, weights):
    rows = weights.reshape(-1, weights.shape[-1]).shape[0]
    return parts.new_empty((rows, parts.shape[-1]), dtype=torch.bfloat16)


@torch.library.custom_op(f"{NAMESPACE}::rotate", mutates_args=())
def rotate(x: Tensor, only_if: Tensor, swiglu: bool = False) -> Tensor:
    """float32 rows of x in the ConvRot basis (through SiLU(gate) * up first with `swiglu`): kernels.rotate."""
    return kernels.rotate(x, only_if, swiglu)


@rotate.register_fake
def _(x, only_if, swiglu=False):
    rows, width = x.shape
    return x.new_empty((rows, width // 2 if swiglu else width), dtype=torch.float32)


# ---- the fused MoE block pieces (drama3/model.py:40-47,107-123)

@torch.library.custom_op(f"{NAMESPACE}::router", mutates_args=())
def router(x: Tensor, weight: Tensor, k: int) -> tuple[Tensor, Tensor]:
    """(ids, weights) of decode rows through a bf16 router linear and the decode routing: kernels.router."""
    return kernels.router(x, weight, k)


@router.register_fake
def _(x, weight, k):
    rows = x.shape[0]
    return x.new_empty((rows, k), dtype=torch.int64), x.new_empty((rows, k), dtype=torch.float32)


@torch.library.custom_op(f"{NAMESPACE}::shared_expert", mutates_args=("out",))
def shared_expert(x: Tensor, gate_up: Tensor, down: Tensor, gate: Tensor, out: Tensor) -> None:
    """out += the sigmoid-gated shared expert of decode rows x, in place: kernels.shared_expert."""
    kernels.shared_expert(x, gate_up, down, gate, out)


@shared_expert.register_fake
def _(x, gate_up, down, gate, out):
    return None


@torch.library.custom_op(f"{NAMESPACE}::moe_decode", mutates_args=())
def moe_decode(kind: str, x: Tensor, ids: Tensor, weights: Tensor, w13: Tensor, s13: Tensor,
               c13: Optional[Tensor], w2: Tensor, s2: Tensor, c2: Optional[Tensor],
               codebook13: Optional[Tensor] = None, codebook2: Optional[Tensor] = None) -> Tensor:
    """[M, H] bfloat16: rows x through their routed experts, one fused launch (kernels.moe_decode); (w13, s13, c13)
    and (w2, s2, c2) are the gate_up and down banks' weight rows, scales and s_channel."""
    banks = (_fields(kind, w13, s13, c13), _fields(kind, w2, s2, c2))
    return kernels.moe_decode(kind, x, ids, weights, banks, (codebook13, codebook2))


@moe_decode.register_fake
def _(kind, x, ids, weights, w13, s13, c13, w2, s2, c2, codebook13=None, codebook2=None):
    return x.new_empty(x.shape, dtype=torch.bfloat16)


# ---- the prompt pass (drama3/offload.py:126-149)

@torch.library.custom_op(f"{NAMESPACE}::prefill_plan", mutates_args=())
def prefill_plan(topk_idx: Tensor, num_experts: int, drop_invalid: bool = False) -> tuple[Tensor, Tensor, Tensor]:
    """(order, pos, groups) of a prompt's routing sorted by expert on the device: kernels.prefill_plan."""
    return kernels.prefill_plan(topk_idx, num_experts, drop_invalid)


@prefill_plan.register_fake
def _(topk_idx, num_experts, drop_invalid=False):
    P = topk_idx.numel()
    return (topk_idx.new_empty((P,), dtype=torch.int64), topk_idx.new_empty((P,), dtype=torch.int64),
            topk_idx.new_empty((num_experts + 1, 5), dtype=torch.int32))


@torch.library.custom_op(f"{NAMESPACE}::grouped_mma", mutates_args=())
def grouped_mma(kind: str, x: Tensor, groups: Tensor, w: Tensor, scale: Tensor, s_channel: Optional[Tensor],
                codebook: Optional[Tensor], n: int, tiles: int, row_index: Optional[Tensor] = None,
                rotate: bool = False, swiglu: bool = False) -> Tensor:
    """[rows, n] float32: the sorted rows through their experts on the tensor cores (kernels.grouped_mma)."""
    return kernels.grouped_mma(kind, x, groups, _fields(kind, w, scale, s_channel), codebook, n, tiles,
                               row_index=row_index, rotate=rotate, swiglu=swiglu)


@grouped_mma.register_fake
def _(kind, x, groups, w, scale, s_channel, codebook, n, tiles, row_index=None, rotate=False, swiglu=False):
    rows = row_index.shape[0] if row_index is not None else x.shape[0]
    return x.new_empty((rows, n), dtype=torch.float32)


@torch.library.custom_op(f"{NAMESPACE}::prefill_combine", mutates_args=())
def prefill_combine(sorted_out: Tensor, pos: Tensor, weights: Tensor, out_f32: bool = False) -> Tensor:
    """[T, H]: the scatter, routing weights and sum over k of a prompt pass (kernels.prefill_combine), bfloat16 or
    float32 with out_f32."""
    return kernels.prefill_combine(sorted_out, pos, weights, dtype=torch.float32 if out_f32 else torch.bfloat16)


@prefill_combine.register_fake
def _(sorted_out, pos, weights, out_f32=False):
    return sorted_out.new_empty((pos.shape[0], sorted_out.shape[1]),
                                dtype=torch.float32 if out_f32 else torch.bfloat16)
