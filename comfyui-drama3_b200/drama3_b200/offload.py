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
# layout name of the BASELINE int-weight / int8-activation banks dressed as quantized tensors (pack.packed_weight)
WA8_LAYOUT = "Drama3B200GroupInt8ActLayout"
BASELINE_KINDS = ("fp8c", "w4a8", "w6a8")


def pinned(tensor, pin):
    """tensor in page-locked host memory when `pin` (the kernels read it through its device address), else as is
    (contiguous) (drama3/offload.py:54-58). A tensor already page-locked and contiguous is kept, not copied."""
    if not pin or (tensor.is_pinned() and tensor.is_contiguous()):
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
    {_qdata, scale, s_channel}, 4 bits with a codebook or 6 bits without. K must be at most 2048.
    This library's own layout for the BASELINE int8-activation banks, WA8_LAYOUT (int4 two per byte or 6-bit four
    per three bytes along K, bf16 scales per 128 columns, fields {_qdata, scale}), gives "w4a8" / "w6a8"."""
    if not _is_quantized(weight) or weight._qdata.ndim != 2:
        return None
    params, fields = weight._params, per_row_fields(weight)
    if params.orig_shape[-1] > 2048:
        return None
    names = set(fields)
    if weight._layout_cls == "TensorWiseINT8Layout":
        convrot = getattr(params, "convrot", False) and params.convrot_groupsize == 256
        return ("int8", fields) if convrot and names == {"_qdata", "scale"} else None
    if weight._layout_cls == WA8_LAYOUT:
        bits = weight._qdata.shape[1] * 8 // params.orig_shape[-1]
        ok = params.group_size == 128 and bits in (4, 6) and names == {"_qdata", "scale"}
        return (f"w{bits}a8", fields) if ok else None
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


def swiglu(h):
    """SiLU of the first half times the second half (every fused gate_up bank holds its gate rows first)."""
    gate, up = h.chunk(2, dim=-1)
    return nn.functional.silu(gate) * up


def expert_chain(kind, x, project, always):
    """[rows, H] float32: rows x through their experts, unweighted: gate_up, SwiGLU, down. `project(index, rows)` runs
    bank `index`'s kernel (0 = gate_up, 1 = down) on float32 (fp8) or rotated rows. Quantized banks hold their
    weights in the ConvRot basis, so their inputs are rotated first, the SwiGLU fused into the second rotation
    (drama3/offload.py:112-123 for a decode row, :126-135 for grouped rows). `always` is an int32 1 on the GPU."""
    if kind == "fp8":
        return project(1, swiglu(project(0, x.float())))
    hidden = project(0, kernels.rotate(x, always))
    return project(1, kernels.rotate(hidden, always, swiglu=True))


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
    weighted sum; used for shapes the fused kernel is not built for. Expert e sits in slot e (plan code 0)."""
    if kind in BASELINE_KINDS:
        raise ValueError(f"{kind} banks decode through the fused kernel only (hidden 2048, intermediate 512 / 768)")
    plan = torch.stack((ids.to(torch.int32), torch.zeros_like(ids, dtype=torch.int32)), dim=-1)
    took_over, always = torch.arange(2, dtype=torch.int32, device=x.device).split(1)

    def project(index, rows_in):
        if kind == "fp8":
            return kernels.gemv_fp8(rows_in, ids, plan, banks[index], banks[index], rows[index])
        return quantized_gemv(kind, rows_in, ids, plan, took_over, False, banks[index], banks[index], rows[index],
                              codebooks[index])

    return kernels.weighted_sum(expert_chain(kind, x, project, always), weights.float())


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
    """[rows, H] float32: sorted_x's rows through their experts with the reference-API grouped kernels, each group
    reading its expert from its slot or from host memory (drama3/offload.py:126-135); `always` is an int32 1 on the
    GPU."""
    def project(index, rows_in):
        if kind == "fp8":
            return kernels.grouped_fp8(rows_in, groups, slot_banks[index], host_banks[index], rows[index])
        return quantized_grouped(kind, rows_in, groups, slot_banks[index], host_banks[index], rows[index],
                                 codebooks[index])

    return expert_chain(kind, sorted_x.float(), project, always)


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
    be captured in a CUDA graph (the host-side sort of drama3/offload.py:141-145 reads the counts back). Returns
    (order, pos, groups, tiles):
      order [P] int64: the pairs in expert order, in (token, rank) order within an expert; pos [P] its inverse;
      groups [E + 1, 5] int32 (expert, slot, 0, first, rows): every expert's group, empty ones included (they get no
        tile), then one group for the pairs whose id is outside [0, E), which sort last (slot E: the grouped kernels
        skip its rows and record the bad-slot fault, as they do for such a group of the host-side plan);
      tiles: a host int from the shapes alone that bounds the row tiles of any routing, (P + (t - 1)(E + 1)) // t for
        t rows per tile (the kernels run the number of tiles the groups need, counted on the device).
    drop_invalid: the last group gets no rows, so the pairs of out-of-range ids are left out (not computed, no fault):
    for padding rows.
    On a GPU with up to 256 experts the sort is one kernel launch (kernels.prefill_plan, a counting sort); otherwise
    (CPU tensors, more experts) it is the same counting sort in torch ops: per-expert prefix sums of one-hot rows."""
    flat = topk_idx.reshape(-1).to(torch.int64)
    E, P = num_experts, flat.numel()
    t = kernels.grouped_tile_rows()
    tiles = (P + (t - 1) * (E + 1)) // t
    if flat.is_cuda and kernels.prefill_plan_fits(E):
        return (*kernels.prefill_plan(flat, E, drop_invalid), tiles)
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
    return order, pos, groups, tiles


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
    return _unsort_weighted_sum(sorted_out, order, topk_weight.float(), num_tokens, top_k).to(x.dtype)


class HostBank:
    """One expert bank in host memory, pinned when asked: every field's first dimension holds the experts' rows one
    expert after another (drama3/offload.py:200-217). `kernel` names the kernel family that reads it."""

    kernel = None

    def __init__(self, num_experts, fields, pin):
        self.num_experts = num_experts
        self.fields = {name: pinned(t, pin) for name, t in fields.items()}

    def rows(self, name):
        """Rows of field `name` per expert."""
        return self.fields[name].shape[0] // self.num_experts

    def expert_bytes(self):
        """Bytes of one expert over all fields."""
        return sum(t.nbytes for t in self.fields.values()) // self.num_experts

    def take(self, fields, first, last):
        """Experts [first, last) of `fields` (this bank's, or any laid out like them), as views."""
        return {name: t.narrow(0, first * self.rows(name), (last - first) * self.rows(name))
                for name, t in fields.items()}

    def to_device(self, first, last, device):
        """Experts [first, last) copied to `device` (asynchronously from pinned memory)."""
        span = self.take(self.fields, first, last)
        return {name: t.to(device, non_blocking=True) for name, t in span.items()}


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


def host_banks(experts, pin):
    """(gate_up, down) host banks of a layer's expert module: an FP8Experts module's e4m3 block-scaled banks, or the
    quantized banks of an Experts module's gate_up_proj / down_proj."""
    if isinstance(experts, FP8Experts):
        if experts.per_channel:
            raise ValueError("the slot cache reads the reference layouts; per-channel fp8 experts stay resident")
        return tuple(FP8HostBank(getattr(experts, f"{name}_weight"), getattr(experts, f"{name}_scale"), pin)
                     for name in ("gate_up", "down"))
    return tuple(QuantHostBank(getattr(experts, f"{name}_proj"), pin) for name in ("gate_up", "down"))


def decayed_uses(score, at, keys, now, span):
    """float32 use counts of `keys` at step `now`: each count halves every `span` steps after the step `at` it was
    last updated at; a key never used (at < 0) counts 0. The arithmetic is torch's float32 one of the reference's host
    methods: exp2 of the step difference divided by span, times the count (drama3/offload.py:667-670)."""
    last = at[keys]
    return torch.where(last < 0, 0.0, score[keys] * torch.exp2((last - now).float() / span))


class SlotState:
    """The slot cache's bookkeeping as a structure of arrays in one memory (the host's or a GPU's), in the layout the
    resolve kernel reads (kernels.resolve): table [keys], owner [count], score [keys], at [keys], pending [count],
    clock [1], reads [3]; key = layer * experts + expert."""

    NAMES = ("table", "owner", "score", "at", "pending", "clock", "reads")

    def __init__(self, keys, count, device="cpu"):
        def full(n, value, dtype=torch.int32):
            return torch.full((n,), value, dtype=dtype, device=device)
        self.table, self.owner = full(keys, -1), full(count, -1)
        self.score, self.at = full(keys, 0.0, torch.float32), full(keys, -1)
        self.pending, self.clock, self.reads = full(count, 0), full(1, 0), full(3, 0)

    def tensors(self):
        return [getattr(self, name) for name in self.NAMES]

    def copy_from(self, other):
        for mine, theirs in zip(self.tensors(), other.tensors()):
            mine.copy_(theirs)


class SlotPool:
    """A fixed number of expert slots on the GPU, filled from host memory, the least used expert out first
    (drama3/offload.py:560-752).

    Rules (the reference's observable ones):
      - count = max(8, min(layers * experts, budget // expert_bytes)) slots; slot s of bank index i holds rows
        [s * rows_i, (s + 1) * rows_i) of every field.
      - table[key] = the key's slot, -1 (host memory only) or -2 - slot (being copied in); owner[slot] = its key or -1.
      - score / at: a decayed use count (halving every HALF_LIFE passes) as of step at = clock * layers + layer
        (-1: never). clock ticks when layer 0 starts a pass. reads = [hits, fills, CPU runs].
      - A slot's eviction value is -1 when free, +inf while its expert was used by this layer in this pass, else its
        decayed count; a claim takes the lowest (ties: the lower slot), and the old owner leaves the table.
    The state has a host copy (host-side calls: use, assign, claim, room) and a device copy at addresses fixed for
    the pool's life (the resolve kernel, and CUDA graphs recorded over it); `device_state` and `host` move it.
    There is no CPU side here, so no slot is ever reserved for a host copy: between decode steps only the reservation
    budget the resolve kernel reads moves, by the reference's rule."""

    def __init__(self, banks, budget, device):
        self.banks = banks
        layer0 = banks[0]
        self.layers, self.num_experts = len(banks), layer0[0].num_experts
        self.rows = [{name: bank.rows(name) for name in bank.fields} for bank in layer0]
        self.expert_bytes = sum(t.nbytes // bank.num_experts for bank in layer0 for t in bank.fields.values())
        self.count = max(8, min(self.layers * self.num_experts, budget // self.expert_bytes))
        self.device = torch.device(device)
        self.fields = [{name: torch.empty((self.count * rows, *t.shape[1:]), dtype=t.dtype, device=self.device)
                        for (name, t), rows in zip(bank.fields.items(), per.values())}
                       for bank, per in zip(layer0, self.rows)]
        self._span = HALF_LIFE * self.layers
        self._host_state = SlotState(self.layers * self.num_experts, self.count)
        self._device_state = None
        self._state = self._host_state
        self.reserve = RESERVE_START
        self.budget = None
        # device scalars the kernels read: a layer's step, the took-over flag (always 0 here), a constant 1, the share
        self.step, self.took_over, self.always = torch.tensor([[0], [0], [1]], dtype=torch.int32, device=self.device)
        self.share = torch.zeros((1,), dtype=torch.float32, device=self.device)

    # the state arrays of the copy in use
    table = property(lambda self: self._state.table)
    owner = property(lambda self: self._state.owner)
    score = property(lambda self: self._state.score)
    at = property(lambda self: self._state.at)
    pending = property(lambda self: self._state.pending)
    clock = property(lambda self: self._state.clock)
    reads = property(lambda self: self._state.reads)

    @property
    def on_device(self):
        return self._state is self._device_state

    def _budget(self):
        """[slots a decode step may reserve, at most per layer]: the step's reserve spread over the layers, with
        room for twice the even share (drama3/offload.py:649-651)."""
        return [self.reserve, max(1, (2 * self.reserve + self.layers - 1) // self.layers)]

    def device_state(self):
        """(table, owner, score, at, pending, clock, budget, reads, step, share) on the GPU (drama3/offload.py:598-613):
        the host copy moved into the device copy, which is made once and keeps its addresses."""
        if not self.on_device:
            if self._device_state is None:
                self._device_state = SlotState(self.layers * self.num_experts, self.count, self.device)
                self.budget = torch.empty((2,), dtype=torch.int32, device=self.device)
            self._device_state.copy_from(self._host_state)
            self.budget.copy_(torch.tensor(self._budget(), dtype=torch.int32))
            self._state = self._device_state
        s = self._state
        return s.table, s.owner, s.score, s.at, s.pending, s.clock, self.budget, s.reads, self.step, self.share

    def host(self):
        """Bring the state back to the host copy (it waits for the GPU's work on it)."""
        if self.on_device:
            self._host_state.copy_from(self._device_state)
            self._state = self._host_state

    def promote(self):
        """Between decode steps (drama3/offload.py:624-647). Nothing is ever reserved for a host copy here (no CPU
        side), so the copies never lag and the step's reservation budget grows by a quarter plus one, up to
        RESERVE_MAX."""
        if not self.on_device:
            return
        self.reserve = min(RESERVE_MAX, self.reserve + self.reserve // 4 + 1)
        self.budget.copy_(torch.tensor(self._budget(), dtype=torch.int32), non_blocking=True)

    def settle(self):
        """Every reserved slot copied in: there are none here."""

    def _step(self, layer, tick):
        """`layer`'s step in the current pass; with `tick`, layer 0 starts a new pass."""
        if tick and layer == 0:
            self.clock.add_(1)
        return int(self.clock) * self.layers + layer

    def _eviction_values(self, layer):
        """Per slot, the value a claim by `layer` minimizes: -1 free, +inf held by an expert `layer` used in this
        pass, else the holder's decayed use count."""
        now = self._step(layer, tick=False)
        holder = self.owner.long()
        key = holder.clamp(min=0)
        values = torch.where(holder < 0, -1.0, decayed_uses(self.score, self.at, key, now, self._span))
        return values.masked_fill((holder >= 0) & (self.at[key] == now), float("inf"))

    def slot_fields(self, index, slot):
        """Bank `index`'s fields of the expert in `slot`, as views laid out like one expert of a host bank."""
        return {name: t.narrow(0, slot * self.rows[index][name], self.rows[index][name])
                for name, t in self.fields[index].items()}

    def _fill(self, slot, sources):
        for index, source in enumerate(sources):
            for name, view in self.slot_fields(index, slot).items():
                view.copy_(source[name], non_blocking=True)

    def use(self, layer, experts):
        """{expert: slot} of the cached ones among `experts` (distinct); each counts a use in this pass
        (drama3/offload.py:689-697)."""
        self.host()
        now = self._step(layer, tick=True)
        keys = torch.as_tensor(experts, dtype=torch.long) + layer * self.num_experts
        self.score[keys] = decayed_uses(self.score, self.at, keys, now, self._span) + 1
        self.at[keys] = now
        return {e: s for e, s in zip(experts, self.table[keys].tolist()) if s >= 0}

    def free_slots(self):
        """Slots without an expert, ascending."""
        return [s for s, key in enumerate(self.owner.tolist()) if key < 0]

    def assign(self, slot, layer, expert):
        """Give `slot` to an expert of `layer`; its old expert leaves the table. The caller fills it."""
        key = layer * self.num_experts + expert
        evicted = int(self.owner[slot])
        if evicted >= 0:
            self.table[evicted] = -1
        self.owner[slot] = key
        self.table[key] = slot
        return slot

    def claim(self, layer, expert):
        """The slot of the least used cached expert (a free one first) that `layer` has not used in this pass; ties go
        to the lower slot (drama3/offload.py:711-717)."""
        return self.assign(int(torch.argmin(self._eviction_values(layer))), layer, expert)

    def room(self, layer):
        """Slots `layer` may still claim in this pass: those not held by an expert it used (drama3/offload.py:719-722)."""
        return int(torch.isfinite(self._eviction_values(layer)).sum())

    def insert(self, layer, expert, sources):
        """A claimed slot for an expert `layer` uses, filled from `sources` (one expert's fields per bank)."""
        slot = self.claim(layer, expert)
        self._fill(slot, sources)
        return slot

    def slots(self, layer, experts, banks):
        """The host-lookup decode's slots of `experts` (a device tensor), missed ones inserted; counts hits and
        fills (drama3/offload.py:730-740)."""
        found = self.use(layer, experts)
        out = [found[e] if e in found else self.insert(layer, e, [b.take(b.fields, e, e + 1) for b in banks])
               for e in experts]
        self.reads.add_(torch.tensor([len(found), len(experts) - len(found), 0], dtype=torch.int32))
        return torch.tensor(out, device=self.device)

    def gather(self, index, slots):
        """Bank `index`'s fields of the experts in `slots` (a device tensor), one after another."""
        return {name: t.unflatten(0, (self.count, -1)).index_select(0, slots).flatten(0, 1)
                for name, t in self.fields[index].items()}

    def report(self):
        self.host()
        hits, fills, on_cpu = self.reads.tolist()
        total = hits + fills + on_cpu
        if total:
            size = sum(t.nbytes for fields in self.fields for t in fields.values()) / 1024 ** 3
            logging.info("drama3_b200 expert cache: %d experts (%.1f GiB), %.0f%% of %d expert reads hit; %d misses "
                         "read over PCIe", self.count, size, 100 * hits / total, total, fills)


def _unsort_weighted_sum(sorted_out, order, weights, num_tokens, top_k):
    """Pair outputs in expert order back in (token, rank) order, each times its routing weight, summed over a token's
    k pairs (drama3/offload.py:146-149, 461-466); in the dtype of the products (bf16 for bf16 outputs and weights,
    as the reference's model passes them)."""
    weighted = sorted_out * weights.reshape(-1)[order].unsqueeze(1)
    out = torch.empty_like(weighted)
    out[order] = weighted
    return out.view(num_tokens, top_k, -1).sum(dim=1)


class ExpertStore:
    """Every layer's experts in host memory with one slot cache on the GPU per generation
    (drama3/offload.py:302-552). Decode rows run the slot-plan kernels (resolve, then GEMVs that read misses from
    pinned host memory and fill slots), so a decode step never waits on the host and can be captured as a graph;
    a prompt's rows run the grouped kernels over slots the host chooses."""

    def __init__(self, cache_bytes, pin):
        self.banks = []
        self.cache = None
        self.cache_bytes = cache_bytes
        self.pin = pin
        self.sync_free = False
        # the reference's CPU side (experts run on the host beside the GPU): never used here
        self.cpu_experts = False
        self.cpu_side = None

    def add(self, experts):
        """Take a layer's experts into host memory; returns the module that replaces them."""
        self.banks.append(host_banks(experts, self.pin))
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
        free, _ = torch.cuda.mem_get_info(device)
        budget = max(0, free - RESERVE_BASE - int(RESERVE_PER_ROW * rows))
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
        """Between decode steps (drama3/offload.py:386-391): no CPU share to rebalance; the pool's budget moves."""
        self.cache.promote()

    def after_layer(self, layer):
        """The host's part of a decode layer: nothing, with no CPU side."""
        return None

    def forward(self, layer, x, topk_idx, topk_weight):
        if self.cache is None:
            raise RuntimeError("ExpertStore.forward outside a session: open `session(device)` first")
        if x.device != self.cache.device:
            raise RuntimeError(f"rows on {x.device}, expert cache on {self.cache.device}")
        if x.shape[0] == 1:
            return self.decode(layer, self.banks[layer], x, topk_idx[0], topk_weight[0])
        return self.prefill(layer, self.banks[layer], x, topk_idx, topk_weight)

    def decode(self, layer, banks, x, ids, weights):
        """One row x [1, H] through its experts ids [k]: resolve, gate_up, SwiGLU, down, weighted sum
        (drama3/offload.py:403-432 without the CPU side). [1, H] bfloat16."""
        cache = self.cache
        kind = banks[0].kernel
        plan = kernels.resolve(ids, layer, len(self.banks), banks[0].num_experts, HALF_LIFE, False, ADMIT,
                               *cache.device_state())

        def project(index, rows_in):
            bank = banks[index]
            if kind == "fp8":
                return kernels.gemv_fp8(rows_in, ids, plan, cache.fields[index], bank.fields, bank.rows("weight"))
            return quantized_gemv(kind, rows_in, ids, plan, cache.took_over, False, cache.fields[index], bank.fields,
                                  bank.rows("_qdata"), bank.codebook(x.device))

        return kernels.weighted_sum(expert_chain(kind, x, project, cache.always), weights.float())

    def prefill(self, layer, banks, x, topk_idx, topk_weight):
        """Many rows: each expert the rows use runs once on its rows (drama3/offload.py:454-466). As there, each
        pair's expert output is in x's dtype before it is weighted and summed over the k pairs."""
        num_tokens, top_k = topk_idx.shape
        order, counts = _sort_by_expert(topk_idx, banks[0].num_experts)
        sorted_out = self.prefill_kernels(layer, banks, x[order // top_k], counts)
        return _unsort_weighted_sum(sorted_out, order, topk_weight, num_tokens, top_k)

    def prompt_groups(self, layer, counts):
        """(expert, slot, fill, first row, rows) for every expert with rows in a prompt sorted by expert (counts[e]
        rows each): a cached expert reads its slot; of the others, those with the most rows (ties: the lower expert)
        take free slots in ascending order, at most the layer's share of the cache (count // layers), and are filled
        on the way (fill 1); the rest read host memory (slot -1) (drama3/offload.py:468-485)."""
        cache = self.cache
        used = [e for e, n in enumerate(counts) if n]
        slot_of = cache.use(layer, used)
        uncached = sorted((e for e in used if e not in slot_of), key=lambda e: (-counts[e], e))
        free = cache.free_slots()
        filled = uncached[:min(cache.count // len(self.banks), len(free))]
        for e, slot in zip(filled, free):
            slot_of[e] = cache.assign(slot, layer, e)
        first = [0, *itertools.accumulate(counts)]
        return [(e, slot_of.get(e, -1), int(e in filled), first[e], counts[e]) for e in used]

    def prefill_kernels(self, layer, banks, sorted_x, counts):
        """sorted_x's rows (sorted by expert, counts[e] each) through their experts, unweighted, one grouped kernel per
        bank over the groups of prompt_groups (drama3/offload.py:468-512). In sorted_x's dtype."""
        groups = self.prompt_groups(layer, counts)
        if not groups:
            return torch.zeros_like(sorted_x)
        device = sorted_x.device
        groups = torch.tensor(groups, dtype=torch.int32).to(device)
        key = "weight" if banks[0].kernel == "fp8" else "_qdata"
        out = grouped_experts(sorted_x, groups, self.cache.fields, [bank.fields for bank in banks],
                              [bank.rows(key) for bank in banks], banks[0].kernel,
                              [bank.codebook(device) for bank in banks], self.cache.always)
        return out.to(sorted_x.dtype)


class FP8Experts(nn.Module):
    """Routed experts as float8 e4m3 weights held whole on the GPU (drama3/offload.py:755-802): by default with a
    float32 scale per 128 x 128 block, the reference's layout ({gate_up,down}_scale [E, N/128, K/128]); with
    `per_channel` one float32 scale per output row ({gate_up,down}_scale [E, N]), the per-channel layout the fused
    tensor-core decode reads fastest. Up to 16 rows of the fused kernel's shapes run the decode (one launch for all
    rows); more run the grouped tensor-core GEMMs."""

    def __init__(self, num_experts, hidden, intermediate, device=None, dtype=None, per_channel=False):
        super().__init__()
        self.num_experts = num_experts
        self.dtype = dtype
        self.per_channel = per_channel
        for name, rows, cols in (("gate_up", 2 * intermediate, hidden), ("down", hidden, intermediate)):
            weight = torch.empty((num_experts, rows, cols), dtype=torch.float8_e4m3fn, device=device)
            shape = (num_experts, rows) if per_channel else (num_experts, rows // FP8_BLOCK, cols // FP8_BLOCK)
            scale = torch.empty(shape, dtype=torch.float32, device=device)
            self.register_parameter(f"{name}_weight", nn.Parameter(weight, requires_grad=False))
            self.register_parameter(f"{name}_scale", nn.Parameter(scale, requires_grad=False))
        self._workspace = {}

    @property
    def kind(self):
        return "fp8c" if self.per_channel else "fp8"

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
        fits = fused_decode_fits(hidden, intermediate, M, k)
        if M == 1 or fits:
            ws = self.workspace(M, k, x.device) if fits else None
            return resident_decode_lines(x, topk_idx, topk_weight, banks, rows, self.kind, (None, None), workspace=ws)
        return resident_prefill(x, topk_idx, topk_weight, banks, rows, self.kind, (None, None), self.num_experts,
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
