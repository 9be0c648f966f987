"""The reference's expert-module surface (drama3/offload.py) over libdrama3_b200: routed experts held whole on the GPU
(`resident_decode`, `resident_prefill`, `FP8Experts`) or in pinned host memory behind a slot cache on the GPU
(`ExpertStore`, `SlotPool`, `OffloadedExperts`).

Same names, arguments and results as the reference; every expert computation runs in the library's kernels, and a
device they cannot run on raises (there is no torch or CPU fallback). Differences, all on the side of doing less on
the host:
  - `resident_decode` runs the fused decode kernel (`kernels.moe_decode`: gate_up, SwiGLU, down and the weighted sum
    in one launch) instead of four to six launches; `resident_decode_lines` does the same for up to 16 rows at once,
    which is what a batch of lines decoded together needs (drama3/model.py:111-113 loops them one by one);
  - the CPU-expert side (`CpuSide`, `experts_on_cpu`, `kernels.await_cpu`) is not provided: a missed expert is read
    from pinned host memory by the GPU kernels, never run on the host;
  - `ExpertStore.session` sizes the cache from `torch.cuda.mem_get_info` (the reference asks ComfyUI's model
    manager, which is not part of this path).
Quantized banks are recognized by duck typing: any object with `_qdata`, `_params` and `_layout_cls` attributes laid
out like comfy's QuantizedTensor.
"""
import contextlib
import dataclasses
import itertools
import logging

import torch
import torch.nn as nn

from . import kernels

# VRAM a generation keeps free besides the cache (drama3/offload.py:30-31)
RESERVE_BASE = 512 * 1024 ** 2
RESERVE_PER_ROW = 0.3 * 1024 ** 2
FP8_BLOCK = 128
# passes over which an expert's decayed use count halves (drama3/offload.py:42-44)
HALF_LIFE = 128
MAX_EXPERTS_PER_ROW = 8
# slots a decode step may reserve for CPU-run experts (drama3/offload.py:48-50); with no CPU side none are reserved,
# but the budget the resolve kernel reads keeps the reference's values
RESERVE_START, RESERVE_MIN, RESERVE_MAX = 32, 8, 256
ADMIT = 6.0
# the fused decode's limit on rows per call
MAX_DECODE_ROWS = 16
# formats whose activations are ConvRot-rotated; the BASELINE layouts (no reference kernels, fused paths only)
ROTATED_KINDS = ("int8", "w4", "w6")
BASELINE_KINDS = ("fp8c", "w4a8", "w6a8")


def pinned(tensor, pin):
    """tensor in page-locked host memory when `pin` (the kernels read it through its device address), else as is
    (contiguous) (drama3/offload.py:54-58)."""
    if not pin:
        return tensor.contiguous()
    return torch.empty(tensor.shape, dtype=tensor.dtype, pin_memory=True).copy_(tensor)


def tensor_fields(weight):
    """{name: tensor} of a quantized weight's parameter dataclass (drama3/offload.py:61-63)."""
    params = weight._params
    out = {}
    for field in dataclasses.fields(params):
        value = getattr(params, field.name)
        if torch.is_tensor(value):
            out[field.name] = value
    return out


def per_row_fields(weight):
    """The quantized weight's tensors with one entry per weight row, `_qdata` first (drama3/offload.py:66-70)."""
    rows = weight._qdata.shape[0]
    fields = {"_qdata": weight._qdata}
    for name, value in tensor_fields(weight).items():
        if value.ndim >= 1 and value.shape[0] == rows:
            fields[name] = value
    return fields


def _is_quantized(weight):
    return all(hasattr(weight, name) for name in ("_qdata", "_params", "_layout_cls"))


def kernel_bank(weight):
    """(kind, fields) of a flat quantized bank [E * out, ...] the kernels read, or None (drama3/offload.py:73-90):
    "int8" = TensorWiseINT8Layout with ConvRot over 256 columns, fields {_qdata, scale}; "w4" / "w6" =
    AsymW4A8Int8Layout with 16-column groups, ConvRot 256, no correction, not transposed, fields
    {_qdata, scale, s_channel}, 4 bits with a codebook or 6 bits without. K must be at most 2048."""
    if not _is_quantized(weight) or weight._qdata.ndim != 2:
        return None
    params, fields = weight._params, per_row_fields(weight)
    if params.orig_shape[-1] > 2048:
        return None
    names = set(fields)
    if weight._layout_cls == "TensorWiseINT8Layout":
        convrot = getattr(params, "convrot", False) and params.convrot_groupsize == 256
        return ("int8", fields) if convrot and names == {"_qdata", "scale"} else None
    if weight._layout_cls != "AsymW4A8Int8Layout":
        return None
    if (params.group_size != 16 or params.convrot_groupsize != 256 or params.correction is not None
            or params.transposed or names != {"_qdata", "scale", "s_channel"}):
        return None
    bits = weight._qdata.shape[1] * 8 // params.orig_shape[-1]
    has_codebook = params.codebook is not None
    if (bits == 4 and has_codebook) or (bits == 6 and not has_codebook):
        return f"w{bits}", fields
    return None


def quantized_gemv(kind, x, ids, plan, took_over, late, slot_fields, host_fields, rows, codebook):
    """[k, rows] float32 of a decode row's experts in an int8 / W4A8 / W6A8 bank (drama3/offload.py:93-98)."""
    if kind == "int8":
        return kernels.gemv_int8(x, ids, plan, took_over, late, slot_fields, host_fields, rows)
    return kernels.gemv_codes(x, ids, plan, slot_fields, host_fields, codebook, int(kind[1]), rows)


def quantized_grouped(kind, x, groups, slot_fields, host_fields, rows, codebook):
    """quantized_gemv for a prompt's rows grouped by expert (drama3/offload.py:101-105)."""
    if kind == "int8":
        return kernels.grouped_int8(x, groups, slot_fields, host_fields, rows)
    return kernels.grouped_codes(x, groups, slot_fields, host_fields, codebook, int(kind[1]), rows)


# shapes the fused decode kernel is built for (hidden 2048; intermediate 512 as the model, 768 as the benchmark)
FUSED_HIDDEN, FUSED_INTERMEDIATE, FUSED_MAX_PAIRS = 2048, (512, 768), 128


def _decode_banks(banks, rows, kind):
    """(gate_up, down) field dicts checked against the per-expert row counts, and (E, H, I)."""
    gate_up, down = banks
    key = "weight" if kind in ("fp8", "fp8c") else "_qdata"
    if gate_up[key].shape[0] % rows[0] or down[key].shape[0] % rows[1]:
        raise ValueError("bank rows are not a whole number of experts")
    experts = gate_up[key].shape[0] // rows[0]
    if down[key].shape[0] // rows[1] != experts:
        raise ValueError("gate_up and down banks hold different numbers of experts")
    return (gate_up, down), (experts, rows[1], rows[0] // 2)


def fused_decode_fits(hidden, intermediate, rows, k):
    """Whether `rows` rows of top-`k` run in the fused decode kernel (else the per-kernel sequence runs)."""
    return (hidden == FUSED_HIDDEN and intermediate in FUSED_INTERMEDIATE and 1 <= rows <= MAX_DECODE_ROWS
            and rows * k <= FUSED_MAX_PAIRS)


def _decode_sequence(x, ids, weights, banks, rows, kind, codebooks):
    """One row through the reference's kernel sequence (drama3/offload.py:112-123): gemv, SwiGLU [+ rotation], gemv,
    weighted sum; used for shapes the fused kernel is not built for."""
    gate_up, down = banks
    if kind in BASELINE_KINDS:
        raise ValueError(f"{kind} banks decode through the fused kernel only (hidden 2048, intermediate 512 / 768)")
    plan = torch.stack((ids.to(torch.int32), torch.zeros_like(ids, dtype=torch.int32)), dim=-1)
    if kind == "fp8":
        gate, up = kernels.gemv_fp8(x.float(), ids, plan, gate_up, gate_up, rows[0]).chunk(2, dim=-1)
        out = kernels.gemv_fp8(nn.functional.silu(gate) * up, ids, plan, down, down, rows[1])
        return kernels.weighted_sum(out, weights.float())
    took_over, always = torch.arange(2, dtype=torch.int32, device=x.device).split(1)
    hidden = quantized_gemv(kind, kernels.rotate(x, always), ids, plan, took_over, False, gate_up, gate_up, rows[0],
                            codebooks[0])
    out = quantized_gemv(kind, kernels.rotate(hidden, always, swiglu=True), ids, plan, took_over, False, down, down,
                         rows[1], codebooks[1])
    return kernels.weighted_sum(out, weights.float())


def resident_decode_lines(x, ids, weights, banks, rows, kind, codebooks, workspace=None):
    """Rows x [M, H] (each its own line) through their experts ids [M, k] mixed by weights [M, k], banks held whole on
    the GPU (expert e in slot e): [M, H] bfloat16. Shapes the fused kernel is built for run as one launch that reads
    each routed expert once for all M rows; others run the per-kernel sequence row by row."""
    (gate_up, down), (_, hidden, intermediate) = _decode_banks(banks, rows, kind)
    M, k = ids.shape
    if fused_decode_fits(hidden, intermediate, M, k):
        return kernels.moe_decode(kind, x, ids, weights, (gate_up, down), tuple(codebooks), workspace=workspace)
    return torch.cat([_decode_sequence(x[r:r + 1], ids[r], weights[r], (gate_up, down), rows, kind, codebooks)
                      for r in range(M)])


def resident_decode(x, ids, weights, banks, rows, kind, codebooks):
    """One row x [1, H] through experts `ids` [k] of banks held whole on the GPU, `rows` per expert
    (drama3/offload.py:108-123): [1, H] bfloat16, as the reference's weighted_sum returns."""
    return resident_decode_lines(x, ids.reshape(1, -1), weights.reshape(1, -1), banks, rows, kind, codebooks)


def grouped_experts(sorted_x, groups, slot_banks, host_banks, rows, kind, codebooks, always):
    """[rows, H] float32: sorted_x's rows through their experts, one grouped kernel per bank (drama3/offload.py:126-135);
    `always` is an int32 1 on the GPU."""
    if kind == "fp8":
        gate, up = kernels.grouped_fp8(sorted_x.float(), groups, slot_banks[0], host_banks[0], rows[0]).chunk(2, dim=-1)
        return kernels.grouped_fp8(nn.functional.silu(gate) * up, groups, slot_banks[1], host_banks[1], rows[1])
    hidden = quantized_grouped(kind, kernels.rotate(sorted_x.float(), always), groups, slot_banks[0], host_banks[0],
                               rows[0], codebooks[0])
    return quantized_grouped(kind, kernels.rotate(hidden, always, swiglu=True), groups, slot_banks[1], host_banks[1],
                             rows[1], codebooks[1])


def _sort_by_expert(topk_idx, num_experts):
    """(order, counts): the flat (token, rank) pairs sorted by expert, and the pair count of every expert."""
    flat = topk_idx.reshape(-1)
    order = torch.argsort(flat)
    counts = torch.bincount(flat, minlength=num_experts).tolist()
    return order, counts


def capturing(x):
    """Whether the current stream of x's device is capturing a CUDA graph: prompt passes then sort on the device
    (resident_prefill(sync_free=True)), since the host-side sort reads the counts back, which a capture forbids."""
    return x.is_cuda and torch.cuda.is_current_stream_capturing()


def prefill_plan(topk_idx, num_experts, drop_invalid=False):
    """The prompt's (token, rank) pairs sorted by expert on the device, with no host sync, so that a prompt pass can
    be captured in a CUDA graph (the host-side sort of drama3/offload.py:141-145 reads the counts back): a counting
    sort by per-expert prefix sums of the pairs' one-hot rows. Returns (order, pos, groups, tiles):
      order [P] int64: the pairs in expert order, in (token, rank) order within an expert; pos [P] its inverse;
      groups [E + 1, 5] int32 (expert, slot, 0, first, rows): every expert's group, empty ones included (they get no
        tile), then one group for the pairs whose id is outside [0, E), which sort last (slot E: the grouped kernels
        skip its rows and record the bad-slot fault, as they do for such a group of the host-side plan);
      tiles: a host int from the shapes alone that bounds the row tiles of any routing, (P + (t - 1)(E + 1)) // t for
        t rows per tile (the kernels run the number of tiles the groups need, counted on the device).
    drop_invalid: the last group gets no rows, so the pairs of out-of-range ids are left out (not computed, no fault):
    for padding rows."""
    flat = topk_idx.reshape(-1).to(torch.int64)
    E, P = num_experts, flat.numel()
    key = torch.where((flat >= 0) & (flat < E), flat, torch.full_like(flat, E))
    onehot = (key.unsqueeze(1) == torch.arange(E + 1, device=flat.device)).to(torch.int32)
    ranks = torch.cumsum(onehot, dim=0, dtype=torch.int32)
    counts = ranks[-1] if P else torch.zeros((E + 1,), dtype=torch.int32, device=flat.device)
    first = torch.cumsum(counts, dim=0, dtype=torch.int32) - counts
    pos = (first.gather(0, key) + ranks.gather(1, key.unsqueeze(1)).squeeze(1) - 1).to(torch.int64)
    order = torch.empty_like(pos).scatter_(0, pos, torch.arange(P, device=flat.device))
    experts = torch.arange(E + 1, dtype=torch.int32, device=flat.device)
    rows = torch.cat([counts[:E], torch.zeros_like(counts[E:])]) if drop_invalid else counts
    groups = torch.stack([experts, experts, torch.zeros_like(experts), first, rows], dim=1).contiguous()
    t = kernels.grouped_tile_rows()
    return order, pos, groups, (P + (t - 1) * (E + 1)) // t


def _scatter_sum(sorted_out, order, topk_weight, num_tokens, top_k):
    """Undo the sort, weight every pair, and sum each token's k pairs (drama3/offload.py:146-149)."""
    out = torch.empty_like(sorted_out)
    out[order] = sorted_out * topk_weight.reshape(-1)[order].unsqueeze(1).float()
    return out.view(num_tokens, top_k, -1).sum(dim=1)


def _grouped_resident(kind, x, groups, tiles, bank, rows, codebook):
    """One bank's grouped GEMM over banks held whole on the GPU: the tensor-core kernel where the shape allows it,
    else the reference-API grouped kernel (slot = expert)."""
    width = x.shape[1]
    if kernels.grouped_mma_fits(rows, width):
        return kernels.grouped_mma(kind, x, groups, bank, codebook, rows, tiles)
    if kind == "fp8":
        return kernels.grouped_fp8(x, groups, bank, bank, rows)
    return quantized_grouped(kind, x, groups, bank, bank, rows, codebook)


def resident_prefill(x, topk_idx, topk_weight, banks, rows, kind, codebooks, num_experts, sync_free=False):
    """Many rows x [T, H] through banks held whole on the GPU (drama3/offload.py:138-149): rows sorted by expert, one
    grouped GEMM per bank on the tensor cores, SwiGLU between (with the ConvRot rotations for int8/W4/W6), scattered
    back, weighted and summed. Where the shapes allow (N % 128, K % 256), the gather of the sorted rows, SwiGLU and
    the rotations run inside the GEMMs' staging and the scatter / weight / sum is one combine launch. [T, H] in x's
    dtype (bfloat16 or float32).
    sync_free: sort on the device (prefill_plan) instead of reading the expert counts back to the host, so the call
    can be captured in a CUDA graph and replayed with new routing; same results bit for bit (every row's GEMMs and
    its combine are computed alone, whatever tile it shares). Tensor-core shapes only."""
    num_tokens, top_k = topk_idx.shape
    gate_up, down = banks
    rotated = kind in ROTATED_KINDS
    width = x.shape[1]
    fused = (x.dtype in (torch.bfloat16, torch.float32) and kernels.grouped_mma_fits(rows[0], width)
             and kernels.grouped_mma_fits(rows[1], rows[0] // 2))
    if sync_free:
        if not fused:
            raise ValueError("a prompt pass without host syncs runs on the tensor-core kernels only (bfloat16 or "
                             "float32 rows, N % 128 == 0, K % 256 == 0)")
        order, pos, groups, tiles = prefill_plan(topk_idx, num_experts)
    else:
        order, counts = _sort_by_expert(topk_idx, num_experts)
        offsets = [0, *itertools.accumulate(counts)]
        groups = [(e, e, 0, offsets[e], n) for e, n in enumerate(counts) if n]
        groups = torch.tensor(groups, dtype=torch.int32).to(x.device)
        tiles = kernels.grouped_tiles(counts)
    if fused:
        hidden = kernels.grouped_mma(kind, x, groups, gate_up, codebooks[0], rows[0], tiles, row_index=order // top_k,
                                     rotate=rotated)
        sorted_out = kernels.grouped_mma(kind, hidden, groups, down, codebooks[1], rows[1], tiles, rotate=rotated,
                                         swiglu=True)
        if not sync_free:
            pos = torch.empty_like(order)
            pos[order] = torch.arange(order.numel(), device=order.device)
        out = kernels.prefill_combine(sorted_out, pos.view(num_tokens, top_k), topk_weight,
                                      dtype=torch.float32 if x.dtype == torch.float32 else torch.bfloat16)
        return out.to(x.dtype)
    if kind in BASELINE_KINDS:
        raise ValueError(f"{kind} banks run on the tensor-core kernel only (N % 128, K % 256)")
    always = torch.ones((1,), dtype=torch.int32, device=x.device)
    sorted_x = x[order // top_k].float()
    if kind == "fp8":
        gate, up = _grouped_resident(kind, sorted_x, groups, tiles, gate_up, rows[0], None).chunk(2, dim=-1)
        sorted_out = _grouped_resident(kind, nn.functional.silu(gate) * up, groups, tiles, down, rows[1], None)
    else:
        hidden = _grouped_resident(kind, kernels.rotate(sorted_x, always), groups, tiles, gate_up, rows[0],
                                   codebooks[0])
        sorted_out = _grouped_resident(kind, kernels.rotate(hidden, always, swiglu=True), groups, tiles, down,
                                       rows[1], codebooks[1])
    return _scatter_sum(sorted_out, order, topk_weight, num_tokens, top_k).to(x.dtype)


class HostBank:
    """One expert bank in host memory, pinned when asked: tensors whose first dimension holds each expert's rows in
    turn (drama3/offload.py:200-217). `kernel` names the kernel family that reads it."""

    kernel = None

    def __init__(self, num_experts, fields, pin):
        self.num_experts = num_experts
        self.fields = {name: pinned(t, pin) for name, t in fields.items()}

    def rows(self, name):
        return self.fields[name].shape[0] // self.num_experts

    def take(self, fields, first, last):
        """Experts [first, last) of `fields` (host or device), laid out like this bank's."""
        return {name: t[first * self.rows(name):last * self.rows(name)] for name, t in fields.items()}

    def to_device(self, first, last, device):
        return {name: t.to(device, non_blocking=True) for name, t in self.take(self.fields, first, last).items()}


class QuantHostBank(HostBank):
    """A flat quantized expert bank (int8 ConvRot, W4A8, W6A8) of a module with `.weight` and `.num_experts`
    (drama3/offload.py:220-262). Only banks the kernels read are accepted."""

    def __init__(self, module, pin):
        weight = module.weight
        if not _is_quantized(weight) or weight._qdata.ndim != 2:
            raise ValueError("only flat quantized or FP8 expert banks are kept in host memory")
        found = kernel_bank(weight)
        if found is None:
            raise ValueError(f"{weight._layout_cls} bank is not a layout the kernels read")
        fields = per_row_fields(weight)
        super().__init__(module.num_experts, fields, pin)
        self.kernel = found[0]
        self.shared = {name: v for name, v in tensor_fields(weight).items() if name not in fields}
        self.shared_on = {}
        self.in_features = weight._params.orig_shape[-1]

    def codebook(self, device):
        """The bank's 4-bit codebook on `device` (W4A8), else None."""
        device = torch.device(device)
        if device not in self.shared_on:
            self.shared_on[device] = {name: v.to(device) for name, v in self.shared.items()}
        return self.shared_on[device].get("codebook")


class FP8HostBank(HostBank):
    """float8 e4m3 expert rows [E, N, K] and fp32 128 x 128 block scales [E, N/128, K/128]
    (drama3/offload.py:265-273)."""

    kernel = "fp8"

    def __init__(self, weight, scale, pin):
        super().__init__(weight.shape[0], {"weight": weight.view(torch.uint8).flatten(0, 1),
                                           "scale": scale.flatten(0, 1)}, pin)
        self.in_features = weight.shape[-1]

    def codebook(self, device):
        return None


class SlotPool:
    """A fixed number of expert slots on the GPU, filled from host memory, the least used expert out first
    (drama3/offload.py:560-752).

    `table[layer * E + expert]` = its slot, -1 (host only) or -2 - slot (being copied in); `owner[slot]` = its key or
    -1 (free); `score` = decayed use count as of step `at` (clock * layers + layer, -1 never); `clock` ticks at layer
    0 of every pass; `reads` = [hits, fills, CPU runs]. The state lives on the host for host-side calls and on the GPU
    while the decode kernels run (`device_state`), at addresses that never change once made (captured graphs read
    them)."""

    def __init__(self, banks, budget, device):
        self.banks = banks
        first = banks[0]
        self.rows = [{name: bank.rows(name) for name in bank.fields} for bank in first]
        self.expert_bytes = sum(t[:bank.rows(name)].nbytes for bank in first for name, t in bank.fields.items())
        self.layers, self.num_experts = len(banks), first[0].num_experts
        self.count = max(8, min(self.layers * self.num_experts, budget // self.expert_bytes))
        self.fields = [{name: torch.empty((self.count * bank.rows(name), *t.shape[1:]), dtype=t.dtype, device=device)
                        for name, t in bank.fields.items()} for bank in first]
        self.device = torch.device(device)
        keys = self.layers * self.num_experts
        self.table = torch.full((keys,), -1, dtype=torch.int32)
        self.owner = torch.full((self.count,), -1, dtype=torch.int32)
        self.score = torch.zeros((keys,), dtype=torch.float32)
        self.at = torch.full((keys,), -1, dtype=torch.int32)
        self.pending = torch.zeros((self.count,), dtype=torch.int32)
        self.clock = torch.zeros((1,), dtype=torch.int32)
        self.reads = torch.zeros((3,), dtype=torch.int32)
        self.on_device = False
        self.resident = None
        self.reserved, self.copying = [], []
        self.reserve = RESERVE_START
        self.budget = None
        self.copy_stream = None
        # device scalars the kernels read: a layer's step, the took-over flag (always 0 here), a constant 1, the share
        self.step, self.took_over, self.always = torch.tensor([[0], [0], [1]], dtype=torch.int32, device=device)
        self.share = torch.zeros((1,), dtype=torch.float32, device=device)

    def _state(self):
        return self.table, self.owner, self.score, self.at, self.pending, self.clock, self.reads

    def _budget(self):
        """[slots a decode step may reserve, at most per layer] (drama3/offload.py:649-651)."""
        return [self.reserve, max(1, -(-2 * self.reserve // self.layers))]

    def device_state(self):
        """(table, owner, score, at, pending, clock, budget, reads, step, share) on the GPU (drama3/offload.py:598-613)."""
        if not self.on_device:
            budget = torch.tensor(self._budget(), dtype=torch.int32)
            if self.resident is None:
                self.resident = [t.to(self.device) for t in self._state()]
                self.budget = budget.to(self.device)
            else:
                for there, here in zip(self.resident, self._state()):
                    there.copy_(here)
                self.budget.copy_(budget)
            self.table, self.owner, self.score, self.at, self.pending, self.clock, self.reads = self.resident
            self.on_device = True
        return (self.table, self.owner, self.score, self.at, self.pending, self.clock, self.budget, self.reads,
                self.step, self.share)

    def host(self):
        """Bring the state back to the host (after every reserved copy has landed)."""
        if self.on_device:
            self.settle()
            self.table, self.owner, self.score, self.at, self.pending, self.clock, self.reads = (
                t.cpu() for t in self._state())
            self.on_device = False

    def promote(self):
        """Between decode steps: map the slots whose copies landed and start the copies of newly reserved slots on a
        copy stream (drama3/offload.py:624-647). With no CPU side nothing is reserved, so this only keeps the budget."""
        if not self.on_device:
            return
        landed = []
        while self.copying and self.copying[0][0].query():
            landed += self.copying.pop(0)[1]
        self._map(landed)
        lagging = bool(self.copying)
        if self.reserved:
            if self.copy_stream is None:
                self.copy_stream = torch.cuda.Stream(self.device)
            self.copy_stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.copy_stream):
                for layer, expert, slot in self.reserved:
                    self._fill(slot, [bank.take(bank.fields, expert, expert + 1) for bank in self.banks[layer]])
                event = torch.cuda.Event()
                event.record()
            self.copying.append((event, [(layer * self.num_experts + e, slot) for layer, e, slot in self.reserved]))
            self.reserved = []
        if lagging:
            self.reserve = max(RESERVE_MIN, self.reserve * 3 // 4)
        else:
            self.reserve = min(RESERVE_MAX, self.reserve * 5 // 4 + 1)
        self.budget.copy_(torch.tensor(self._budget(), dtype=torch.int32), non_blocking=True)

    def settle(self):
        """Every reserved slot copied in and mapped."""
        self.promote()
        if self.copy_stream is not None:
            self.copy_stream.synchronize()
        self._map([pair for _, pairs in self.copying for pair in pairs])
        self.copying = []

    def _map(self, pairs):
        if not pairs:
            return
        keys, slots = zip(*pairs)
        keys = torch.tensor(keys, dtype=torch.long).to(self.device)
        slots = torch.tensor(slots, dtype=torch.int32).to(self.device)
        self.table[keys] = slots
        self.pending[slots.long()] = 0

    def _now(self, layer):
        """`layer`'s step in this pass; layer 0 starts a new pass (drama3/offload.py:661-665)."""
        if layer == 0:
            self.clock += 1
        return int(self.clock) * self.layers + layer

    def _uses(self, keys, now):
        """Decayed use counts of `keys` at step `now` (drama3/offload.py:667-670)."""
        at = self.at[keys]
        decay = torch.exp2((at - now).float() / (HALF_LIFE * self.layers))
        return torch.where(at < 0, 0.0, self.score[keys] * decay)

    def _fill(self, slot, sources):
        for fields, rows, source in zip(self.fields, self.rows, sources):
            for name, target in fields.items():
                target[slot * rows[name]:(slot + 1) * rows[name]].copy_(source[name], non_blocking=True)

    def slot_fields(self, index, slot):
        """Bank `index`'s fields of the expert in `slot`."""
        return {name: t[slot * self.rows[index][name]:(slot + 1) * self.rows[index][name]]
                for name, t in self.fields[index].items()}

    def use(self, layer, experts):
        """{expert: slot} of the cached ones among `experts`; each counts a use in this pass
        (drama3/offload.py:689-697)."""
        self.host()
        now = self._now(layer)
        keys = torch.tensor(experts, dtype=torch.long) + layer * self.num_experts
        self.score[keys] = self._uses(keys, now) + 1
        self.at[keys] = now
        table = self.table[layer * self.num_experts:(layer + 1) * self.num_experts].tolist()
        return {e: table[e] for e in experts if table[e] >= 0}

    def free_slots(self):
        return (self.owner < 0).nonzero().flatten().tolist()

    def assign(self, slot, layer, expert):
        """Give `slot` to an expert of `layer`; its old expert leaves the table (drama3/offload.py:702-709)."""
        key = layer * self.num_experts + expert
        old = int(self.owner[slot])
        if old >= 0:
            self.table[old] = -1
        self.owner[slot] = key
        self.table[key] = slot
        return slot

    def claim(self, layer, expert):
        """The slot of the least used cached expert (a free one first) that `layer` has not used in this pass; ties go
        to the lower slot (drama3/offload.py:711-717)."""
        keys = self.owner.long()
        held = keys.clamp(min=0)
        now = int(self.clock) * self.layers + layer
        uses = torch.where(keys < 0, -1.0, self._uses(held, now))
        uses[(keys >= 0) & (self.at[held] == now)] = float("inf")
        return self.assign(int(torch.argmin(uses)), layer, expert)

    def room(self, layer):
        """Slots `layer` may still claim in this pass (drama3/offload.py:719-722)."""
        keys = self.owner.long()
        now = int(self.clock) * self.layers + layer
        return int(((keys < 0) | (self.at[keys.clamp(min=0)] != now)).sum())

    def insert(self, layer, expert, sources):
        slot = self.claim(layer, expert)
        self._fill(slot, sources)
        return slot

    def gather(self, index, slots):
        return {name: t.view(self.count, self.rows[index][name], *t.shape[1:]).index_select(0, slots).flatten(0, 1)
                for name, t in self.fields[index].items()}

    def report(self):
        self.host()
        hits, fills, on_cpu = self.reads.tolist()
        total = hits + fills + on_cpu
        if total:
            size = sum(t.nbytes for fields in self.fields for t in fields.values()) / 1024 ** 3
            logging.info("drama3_b200 expert cache: %d experts (%.1f GiB), %.0f%% of %d expert reads hit; %d misses "
                         "read over PCIe", self.count, size, 100 * hits / total, total, fills)


class ExpertStore:
    """Every layer's experts in host memory with one slot cache on the GPU per generation
    (drama3/offload.py:302-552). Decode rows run the slot-plan kernels (resolve, then GEMVs that read misses from
    pinned host memory and fill slots), so a decode step never waits on the host and can be captured as a graph;
    a prompt's rows run the grouped kernels."""

    def __init__(self, cache_bytes, pin):
        self.banks = []
        self.cache = None
        self.cache_bytes = cache_bytes
        self.pin = pin
        self.sync_free = False
        self.cpu_experts = False
        self.cpu_side = None

    def add(self, experts):
        """Take a layer's experts into host memory; returns the module that replaces them."""
        if isinstance(experts, FP8Experts):
            banks = (FP8HostBank(experts.gate_up_weight, experts.gate_up_scale, self.pin),
                     FP8HostBank(experts.down_weight, experts.down_scale, self.pin))
        else:
            banks = (QuantHostBank(experts.gate_up_proj, self.pin), QuantHostBank(experts.down_proj, self.pin))
        self.banks.append(banks)
        return OffloadedExperts(self, len(self.banks) - 1)

    @contextlib.contextmanager
    def session(self, device, patchers=(), cpu_decode=False, rows=0, cpu_experts=True):
        """One generation's expert cache on `device`, sized to the VRAM free at its start less a reserve for `rows`
        rows (and at most `cache_bytes` when set). A session inside another shares its cache. `patchers`,
        `cpu_decode` and `cpu_experts` are accepted for the reference's signature; there is no CPU side."""
        if self.cache is not None:
            yield
            return
        device = torch.device(device)
        if not self.pin:
            raise ValueError("the kernels read missed experts from pinned host memory: build the store with pin=True")
        kernels.available(device)
        reserve = RESERVE_BASE + int(RESERVE_PER_ROW * rows)
        free, _ = torch.cuda.mem_get_info(device)
        budget = max(0, free - reserve)
        if self.cache_bytes:
            budget = min(budget, self.cache_bytes)
        self.cache = SlotPool(self.banks, budget, device)
        self.sync_free = True
        for bank in itertools.chain.from_iterable(self.banks):
            bank.codebook(device)  # before any step is captured: a graph cannot copy it in
        try:
            yield
        finally:
            self.cache.report()
            self.cache = None
            self.sync_free = False

    def between_steps(self):
        """Between decode steps (drama3/offload.py:386-391): land reserved copies; no CPU share to rebalance."""
        self.cache.promote()

    def after_layer(self, layer):
        """The host's part of a decode layer: nothing, with no CPU side."""
        return None

    def forward(self, layer, x, topk_idx, topk_weight):
        if self.cache is None:
            raise RuntimeError("ExpertStore.forward outside a session: open `session(device)` first")
        if x.device != self.cache.device:
            raise RuntimeError(f"rows on {x.device}, expert cache on {self.cache.device}")
        banks = self.banks[layer]
        if x.shape[0] == 1:
            return self.decode(layer, banks, x, topk_idx[0], topk_weight[0])
        return self.prefill(layer, banks, x, topk_idx, topk_weight)

    def decode(self, layer, banks, x, ids, weights):
        """One row x [1, H] through its experts ids [k]: resolve, gate_up, SwiGLU, down, weighted sum
        (drama3/offload.py:403-432 without the CPU side). [1, H] bfloat16."""
        gate_up, down = banks
        cache = self.cache
        plan = kernels.resolve(ids, layer, len(self.banks), gate_up.num_experts, HALF_LIFE, False, ADMIT,
                               *cache.device_state())
        slots_gate_up, slots_down = cache.fields
        weights = weights.float()
        if gate_up.kernel == "fp8":
            hidden = kernels.gemv_fp8(x.float(), ids, plan, slots_gate_up, gate_up.fields, gate_up.rows("weight"))
            gate, up = hidden.chunk(2, dim=-1)
            out = kernels.gemv_fp8(nn.functional.silu(gate) * up, ids, plan, slots_down, down.fields,
                                   down.rows("weight"))
            return kernels.weighted_sum(out, weights)
        kind = gate_up.kernel
        rotated = kernels.rotate(x, cache.always)
        hidden = quantized_gemv(kind, rotated, ids, plan, cache.took_over, False, slots_gate_up, gate_up.fields,
                                gate_up.rows("_qdata"), gate_up.codebook(x.device))
        hidden = kernels.rotate(hidden, cache.always, swiglu=True)
        out = quantized_gemv(kind, hidden, ids, plan, cache.took_over, False, slots_down, down.fields,
                             down.rows("_qdata"), down.codebook(x.device))
        return kernels.weighted_sum(out, weights)

    def prefill(self, layer, banks, x, topk_idx, topk_weight):
        """Many rows: each expert the rows use runs once on its rows (drama3/offload.py:454-466). As there, each
        pair's expert output is in x's dtype before it is weighted and summed over the k pairs."""
        num_tokens, top_k = topk_idx.shape
        order, counts = _sort_by_expert(topk_idx, banks[0].num_experts)
        sorted_out = self.prefill_kernels(layer, banks, x[order // top_k], counts)
        weighted = sorted_out * topk_weight.reshape(-1)[order].unsqueeze(1)
        out = torch.empty_like(weighted)
        out[order] = weighted
        return out.view(num_tokens, top_k, -1).sum(dim=1)

    def prefill_kernels(self, layer, banks, sorted_x, counts):
        """sorted_x's rows (sorted by expert, counts[e] each) through their experts, unweighted: cached experts from
        their slots, the most used uncached ones filled into free slots on the way (at most the layer's share of the
        cache), the rest read from host memory; one grouped kernel per bank (drama3/offload.py:468-512)."""
        gate_up, _ = banks
        cache = self.cache
        device = sorted_x.device
        offsets = [0, *itertools.accumulate(counts)]
        used = [e for e, n in enumerate(counts) if n]
        slots = cache.use(layer, used)
        rest = sorted((e for e in used if e not in slots), key=counts.__getitem__, reverse=True)
        free = cache.free_slots()
        fills = rest[:min(cache.count // len(self.banks), len(free))]
        for e, slot in zip(fills, free):
            slots[e] = cache.assign(slot, layer, e)
        fills = set(fills)
        groups = [(e, slots.get(e, -1), int(e in fills), offsets[e], counts[e]) for e in used]
        if not groups:
            return torch.zeros_like(sorted_x)
        groups = torch.tensor(groups, dtype=torch.int32).to(device)
        key = "weight" if gate_up.kernel == "fp8" else "_qdata"
        bank_rows = [bank.rows(key) for bank in banks]
        codebooks = [bank.codebook(device) for bank in banks]
        always = torch.ones((1,), dtype=torch.int32, device=device)
        out = grouped_experts(sorted_x, groups, cache.fields, [bank.fields for bank in banks], bank_rows,
                              gate_up.kernel, codebooks, always)
        return out.to(sorted_x.dtype)


class FP8Experts(nn.Module):
    """Routed experts as float8 e4m3 weights with a float32 scale per 128 x 128 block, held whole on the GPU
    (drama3/offload.py:755-802). One row, or up to 16 rows of the fused kernel's shapes, run the decode; more run the
    grouped kernels."""

    def __init__(self, num_experts, hidden, intermediate, device=None, dtype=None):
        super().__init__()
        self.num_experts = num_experts
        self.dtype = dtype
        for name, rows, cols in (("gate_up", 2 * intermediate, hidden), ("down", hidden, intermediate)):
            weight = torch.empty((num_experts, rows, cols), dtype=torch.float8_e4m3fn, device=device)
            scale = torch.empty((num_experts, rows // FP8_BLOCK, cols // FP8_BLOCK), dtype=torch.float32,
                                device=device)
            self.register_parameter(f"{name}_weight", nn.Parameter(weight, requires_grad=False))
            self.register_parameter(f"{name}_scale", nn.Parameter(scale, requires_grad=False))
        self._workspace = {}

    def sync_free(self, device):
        """Whether a decode row on `device` runs without waiting on the host."""
        return kernels.available(device)

    def banks(self):
        """(gate_up, down) field dicts in the kernels' flat layout, and the rows per expert of each."""
        banks = [{"weight": getattr(self, f"{name}_weight").view(torch.uint8).flatten(0, 1),
                  "scale": getattr(self, f"{name}_scale").flatten(0, 1)} for name in ("gate_up", "down")]
        rows = [getattr(self, f"{name}_weight").shape[1] for name in ("gate_up", "down")]
        return banks, rows

    def workspace(self, rows, k, device):
        """The fused decode's scratch for `rows` x `k`, made once per (device, shape) and reused."""
        key = (torch.device(device), rows, k)
        if key not in self._workspace:
            self._workspace[key] = kernels.decode_workspace(rows, k, self.down_weight.shape[2], device)
        return self._workspace[key]

    def forward(self, x, topk_idx, topk_weight):
        if not kernels.available(x.device):
            raise RuntimeError(f"FP8Experts runs on the sm_100 kernels only, not on {x.device}")
        banks, rows = self.banks()
        hidden, intermediate = self.down_weight.shape[1:]
        M, k = topk_idx.shape
        if M == 1 or fused_decode_fits(hidden, intermediate, M, k):
            ws = self.workspace(M, k, x.device) if fused_decode_fits(hidden, intermediate, M, k) else None
            return resident_decode_lines(x, topk_idx, topk_weight, banks, rows, "fp8", (None, None), workspace=ws)
        return resident_prefill(x, topk_idx, topk_weight, banks, rows, "fp8", (None, None), self.num_experts,
                                sync_free=capturing(x))


class OffloadedExperts(nn.Module):
    """Stands in for a layer's experts held in an ExpertStore (drama3/offload.py:817-830)."""

    def __init__(self, store, layer):
        super().__init__()
        self.store = store
        self.layer = layer

    def sync_free(self, device):
        """Whether a decode row on `device` runs without waiting on the host, in the current generation."""
        return self.store.sync_free and torch.device(device) == self.store.cache.device

    def forward(self, x, topk_idx, topk_weight):
        return self.store.forward(self.layer, x, topk_idx, topk_weight)
