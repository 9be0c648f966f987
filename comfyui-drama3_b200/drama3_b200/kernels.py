"""The reference's kernel module surface (drama3/kernels.py:604-724), backed by libdrama3_b200.so instead of NVRTC.

Same function names, arguments, output shapes and dtypes; every output is allocated with torch on the input's device
and every launch goes on the device's current stream, so calls can be captured in CUDA graphs. Differences:
  - `available` returns False only for non-CUDA devices (as the reference does); on a CUDA device it raises if the
    library is missing or the device is not an sm_100 GPU: there is no fallback implementation;
  - `route` and `weighted_sum` also take several rows at once;
  - `await_cpu` (the CPU-expert handshake) is not provided: this path has no CPU side;
  - `moe_decode` is new: the whole resident decode (gate_up, SwiGLU, down, combine) for 1..16 rows in one pass;
  - `grouped_mma` is new: the grouped kernels on the tensor cores for banks held whole on the GPU.
"""
import functools

import torch

from . import _lib
from ._lib import check, lib

ROWS_PER_BLOCK = 16


def _ptr(t):
    return None if t is None else t.data_ptr()


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


@functools.cache
def _device_ok(index):
    with torch.cuda.device(index):
        check(lib().d3_device_check(), f"cuda:{index}")
    return True


def available(device):
    """Whether `device` runs these kernels: a CUDA device that is an sm_100 GPU, with the library built. Raises on a
    CUDA device where that is not so (no fallback); False for other devices."""
    device = torch.device(device)
    if device.type != "cuda":
        return False
    index = device.index if device.index is not None else torch.cuda.current_device()
    return _device_ok(index)


def _on(device):
    available(device)
    return torch.cuda.device(device)


def resolve(ids, layer, layers, num_experts, half_life, cpu, admit, table, owner, score, at, pending, clock, budget,
            reads, step, share):
    """plan [k, 2] int32 for the row's experts `ids` [k] (int64) of `layer` (drama3/kernels.py:618-625)."""
    plan = torch.empty((ids.shape[0], 2), dtype=torch.int32, device=ids.device)
    with _on(ids.device):
        check(lib().d3_resolve(_ptr(ids), ids.shape[0], int(layer), int(layers), int(num_experts), _ptr(table),
                               _ptr(owner), _ptr(score), _ptr(at), _ptr(pending), owner.shape[0], _ptr(clock),
                               _ptr(budget), _ptr(plan), _ptr(reads), _ptr(step), _ptr(share), float(half_life),
                               int(cpu), float(admit), _stream(ids.device)), "resolve")
    return plan


def await_cpu(plan, flag, step, result, timeout_us, took_over):
    raise NotImplementedError("drama3_b200 has no CPU-expert side: every expert runs on the GPU")


def rotate(x, only_if, swiglu=False):
    """Rows of x [rows, K] (float32 or bfloat16; float32 [rows, 2K] gate | up with `swiglu`, SiLU(gate) * up first)
    in the ConvRot basis: float32 [rows, K]; left unset when `only_if` (an int32 on the GPU) is 0
    (drama3/kernels.py:636-644)."""
    rows, width = x.shape
    k = width // 2 if swiglu else width
    mode = 2 if swiglu else (1 if x.dtype == torch.bfloat16 else 0)
    if mode != 1 and x.dtype != torch.float32:
        raise TypeError(f"rotate takes float32 or bfloat16 rows, not {x.dtype}")
    x = x.contiguous()
    out = torch.empty((rows, k), dtype=torch.float32, device=x.device)
    with _on(x.device):
        check(lib().d3_rotate(_ptr(x), mode, rows, k, _ptr(out), _ptr(only_if), _stream(x.device)), "rotate")
    return out


def route(logits, k):
    """(ids [rows, k] int64, weights [rows, k] float32) of router logits [rows, n] (bfloat16): the k largest, by
    descending logit (ties: lower index first), and their softmax weights renormalized over them, rounded to
    bfloat16 (drama3/kernels.py:647-653, for any number of rows)."""
    if logits.dtype != torch.bfloat16:
        raise TypeError("route takes bfloat16 logits")
    logits = logits.contiguous()
    rows, n = logits.shape
    ids = torch.empty((rows, k), dtype=torch.int64, device=logits.device)
    weights = torch.empty((rows, k), dtype=torch.float32, device=logits.device)
    with _on(logits.device):
        check(lib().d3_route(_ptr(logits), rows, n, int(k), _ptr(ids), _ptr(weights), _stream(logits.device)), "route")
    return ids, weights


def _aligned16(t):
    """t, or a copy of it where its data does not start on a 16-byte boundary (the bulk copies' rule)."""
    return t if t.data_ptr() % 16 == 0 else t.clone()


def router(x, weight, k, logits=False):
    """(ids [rows, k] int64, weights [rows, k] float32[, logits [rows, E] bfloat16]) of decode rows x [rows, H]
    (bfloat16, rows <= 16) through a bias-free bf16 router linear `weight` [E, H] and the decode routing, in one launch:
    route(x @ weight.T, k) with the logits as the bf16 rounding of fp32 sums of the exact products."""
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("router takes bfloat16 rows and weight")
    x, weight = _aligned16(x.contiguous()), _aligned16(weight.contiguous())
    rows, H = x.shape
    E = weight.shape[0]
    ids = torch.empty((rows, k), dtype=torch.int64, device=x.device)
    w = torch.empty((rows, k), dtype=torch.float32, device=x.device)
    lg = torch.empty((rows, E), dtype=torch.bfloat16, device=x.device) if logits else None
    with _on(x.device):
        check(lib().d3_router(_ptr(x), rows, H, _ptr(weight), E, int(k), _ptr(ids), _ptr(w), _ptr(lg),
                              _stream(x.device)), "router")
    return (ids, w, lg) if logits else (ids, w)


def router_fits(rows, hidden, experts, k):
    """Whether `router` takes these shapes."""
    return 1 <= rows <= 16 and hidden == 2048 and experts % 64 == 0 and 64 <= experts <= 256 and k <= min(32, experts)


_SHARED_SCRATCH = {}


def shared_expert(x, gate_up, down, gate, out):
    """out [rows, H] bfloat16 += sigmoid(x @ gate.T) * down(SwiGLU(gate_up(x))) for decode rows x [rows, H] (bfloat16,
    rows <= 16), in place, in two launches; gate_up [2I, H], down [H, I], gate [1, H] or [H], all bfloat16 (the
    reference's SharedExpert and shared_expert_gate linears, drama3/model.py:40-47,123). Returns out."""
    for t in (x, gate_up, down, gate, out):
        if t.dtype != torch.bfloat16:
            raise TypeError("shared_expert takes bfloat16 tensors")
    x, gate_up, down, gate = (_aligned16(t.contiguous()) for t in (x, gate_up, down, gate))
    if not out.is_contiguous():
        raise ValueError("out must be contiguous (it is updated in place)")
    rows, H = x.shape
    I = down.shape[1]
    # scratch: the SwiGLU rows [rows, I] bf16, then the gate [rows] fp32
    key = (x.device, torch.cuda.current_stream(x.device).cuda_stream, rows, I)
    if torch.cuda.is_current_stream_capturing():
        scratch = torch.empty(rows * (I + 2), dtype=torch.bfloat16, device=x.device)
    else:
        scratch = _SHARED_SCRATCH.get(key)
        if scratch is None:
            scratch = _SHARED_SCRATCH[key] = torch.empty(rows * (I + 2), dtype=torch.bfloat16, device=x.device)
    with _on(x.device):
        check(lib().d3_shared_expert(_ptr(x), rows, H, _ptr(gate_up), _ptr(down), _ptr(gate), I, _ptr(scratch),
                                     _ptr(out), _stream(x.device)), "shared_expert")
    return out


def shared_expert_fits(rows, hidden, intermediate):
    """Whether `shared_expert` takes these shapes."""
    return 1 <= rows <= 16 and hidden == 2048 and intermediate in (256, 512, 768, 1024)


def prefill_plan(topk_idx, num_experts, drop_invalid=False):
    """(order [P] int64, pos [P] int64, groups [E + 1, 5] int32) of a prompt's routing [T, k] sorted by expert on the
    device in one launch, no host sync: order holds the (token, rank) pairs by expert id, within an expert in index
    order, ids outside [0, E) last; pos its inverse; groups (expert, slot, 0, first, rows) for every expert and one
    last group for the out-of-range ids (0 rows when drop_invalid). num_experts <= 256 (drama3/offload.py:141-145
    sorts on the host)."""
    flat = topk_idx.reshape(-1).to(torch.int64).contiguous()
    P = flat.numel()
    order = torch.empty(P, dtype=torch.int64, device=flat.device)
    pos = torch.empty(P, dtype=torch.int64, device=flat.device)
    groups = torch.empty((num_experts + 1, 5), dtype=torch.int32, device=flat.device)
    with _on(flat.device):
        check(lib().d3_prefill_plan(_ptr(flat), P, int(num_experts), int(bool(drop_invalid)), _ptr(order), _ptr(pos),
                                    _ptr(groups), _stream(flat.device)), "prefill_plan")
    return order, pos, groups


def prefill_plan_fits(num_experts):
    """Whether `prefill_plan` takes this many experts."""
    return 1 <= num_experts <= 256


def weighted_sum(parts, weights):
    """[rows, H] bfloat16: parts [rows * k, H] (float32) summed per row by weights [rows, k] or [k] (float32), in
    rank order (drama3/kernels.py:656-661; there rows == 1)."""
    weights = weights.reshape(-1, weights.shape[-1]).float().contiguous()
    rows, k = weights.shape
    parts = parts.contiguous()
    H = parts.shape[-1]
    if parts.numel() != rows * k * H:
        raise ValueError("parts must hold rows * k rows")
    out = torch.empty((rows, H), dtype=torch.bfloat16, device=parts.device)
    with _on(parts.device):
        check(lib().d3_weighted_sum(_ptr(parts), _ptr(weights), rows, k, H, _ptr(out), _stream(parts.device)),
              "weighted_sum")
    return out


def _bank_rows(fields, key, n):
    return fields[key].shape[0] // n


def gemv_int8(x, ids, plan, took_over, late, slot_fields, host_fields, n):
    """[k, n] float32: each expert's int8 rows against x [1 or k, K] (float32, rotated); fields are
    {"_qdata", "scale"} (drama3/kernels.py:664-671)."""
    k, width = ids.shape[0], x.shape[1]
    out = torch.empty((k, n), dtype=torch.float32, device=x.device)
    with _on(x.device):
        check(lib().d3_gemv_int8(_ptr(x), x.shape[0], _ptr(ids), _ptr(plan), _ptr(took_over), int(late), k,
                                 _ptr(slot_fields["_qdata"]), _ptr(slot_fields["scale"]), _ptr(host_fields["_qdata"]),
                                 _ptr(host_fields["scale"]), _ptr(out), n, width,
                                 _bank_rows(host_fields, "_qdata", n), _bank_rows(slot_fields, "_qdata", n),
                                 _stream(x.device)), "gemv_int8")
    return out


def gemv_fp8(x, ids, plan, slot_fields, host_fields, n):
    """[k, n] float32: each expert's float8 rows against x [1 or k, K] float32; fields are {"weight", "scale"}
    (drama3/kernels.py:674-681)."""
    k, width = ids.shape[0], x.shape[1]
    out = torch.empty((k, n), dtype=torch.float32, device=x.device)
    with _on(x.device):
        check(lib().d3_gemv_fp8(_ptr(x), x.shape[0], _ptr(ids), _ptr(plan), k, _ptr(slot_fields["weight"]),
                                _ptr(slot_fields["scale"]), _ptr(host_fields["weight"]), _ptr(host_fields["scale"]),
                                _ptr(out), n, width, _bank_rows(host_fields, "weight", n),
                                _bank_rows(slot_fields, "weight", n), _stream(x.device)), "gemv_fp8")
    return out


def gemv_codes(x, ids, plan, slot_fields, host_fields, codebook, bits, n):
    """gemv_int8 for W4A8/W6A8 banks; fields are {"_qdata", "scale" (e4m3), "s_channel"}, codebook [16] at 4 bits
    (drama3/kernels.py:703-713)."""
    k, width = ids.shape[0], x.shape[1]
    out = torch.empty((k, n), dtype=torch.float32, device=x.device)
    with _on(x.device):
        check(lib().d3_gemv_codes(_ptr(x), x.shape[0], _ptr(ids), _ptr(plan), k, _ptr(slot_fields["_qdata"]),
                                  _ptr(slot_fields["scale"]), _ptr(slot_fields["s_channel"]),
                                  _ptr(host_fields["_qdata"]), _ptr(host_fields["scale"]),
                                  _ptr(host_fields["s_channel"]), _ptr(codebook), int(bits), _ptr(out), n, width,
                                  _bank_rows(host_fields, "_qdata", n), _bank_rows(slot_fields, "_qdata", n),
                                  _stream(x.device)), "gemv_codes")
    return out


def grouped_int8(x, groups, slot_fields, host_fields, n):
    """[rows, n] float32 for x's rows (float32, rotated, sorted by expert) through their experts; groups [g, 5] int32
    (expert, slot, fill, first, rows). Rows outside every group are left unset (drama3/kernels.py:684-691)."""
    out = torch.empty((x.shape[0], n), dtype=torch.float32, device=x.device)
    with _on(x.device):
        check(lib().d3_grouped_int8(_ptr(x), x.shape[0], _ptr(groups), groups.shape[0], _ptr(slot_fields["_qdata"]),
                                    _ptr(slot_fields["scale"]), _ptr(host_fields["_qdata"]),
                                    _ptr(host_fields["scale"]), _ptr(out), n, x.shape[1],
                                    _bank_rows(host_fields, "_qdata", n), _bank_rows(slot_fields, "_qdata", n),
                                    _stream(x.device)), "grouped_int8")
    return out


def grouped_fp8(x, groups, slot_fields, host_fields, n):
    """grouped_int8 for float8 experts, against float32 rows x (drama3/kernels.py:694-700)."""
    out = torch.empty((x.shape[0], n), dtype=torch.float32, device=x.device)
    with _on(x.device):
        check(lib().d3_grouped_fp8(_ptr(x), x.shape[0], _ptr(groups), groups.shape[0], _ptr(slot_fields["weight"]),
                                   _ptr(slot_fields["scale"]), _ptr(host_fields["weight"]),
                                   _ptr(host_fields["scale"]), _ptr(out), n, x.shape[1],
                                   _bank_rows(host_fields, "weight", n), _bank_rows(slot_fields, "weight", n),
                                   _stream(x.device)), "grouped_fp8")
    return out


def grouped_codes(x, groups, slot_fields, host_fields, codebook, bits, n):
    """grouped_int8 for W4A8/W6A8 banks (drama3/kernels.py:716-724)."""
    out = torch.empty((x.shape[0], n), dtype=torch.float32, device=x.device)
    with _on(x.device):
        check(lib().d3_grouped_codes(_ptr(x), x.shape[0], _ptr(groups), groups.shape[0], _ptr(slot_fields["_qdata"]),
                                     _ptr(slot_fields["scale"]), _ptr(slot_fields["s_channel"]),
                                     _ptr(host_fields["_qdata"]), _ptr(host_fields["scale"]),
                                     _ptr(host_fields["s_channel"]), _ptr(codebook), int(bits), _ptr(out), n,
                                     x.shape[1], _bank_rows(host_fields, "_qdata", n),
                                     _bank_rows(slot_fields, "_qdata", n), _stream(x.device)), "grouped_codes")
    return out


@functools.cache
def grouped_tile_rows():
    """Rows per tile of the tensor-core grouped kernel (its MMA N at most)."""
    return int(lib().d3_grouped_mma_tile_rows())


def grouped_tiles(counts):
    """Row tiles the tensor-core grouped kernel runs for groups of these row counts."""
    t = grouped_tile_rows()
    return sum((int(n) + t - 1) // t for n in counts)


def grouped_mma_fits(n, k):
    """Whether an [n, k] bank runs on the tensor-core grouped kernel (n % 128 == 0, k % 256 == 0)."""
    return n % 128 == 0 and k % 256 == 0 and k >= 256


GM_ROTATE, GM_SWIGLU = 1, 2


def grouped_mma(kind, x, groups, fields, codebook, n, tiles, row_index=None, rotate=False, swiglu=False):
    """[rows, n] float32 for the sorted rows through their experts, on the tensor cores, for a bank held whole on the
    GPU: the grouped_fp8 / grouped_int8 / grouped_codes results with every group's slot = its expert's index in
    `fields` (drama3/offload.py:126-149). groups [g, 5] int32 on the GPU; tiles = grouped_tiles(row counts), or any
    bound on it (the kernels count the tiles the groups need on the device; offload.prefill_plan gives one). Sorted
    row s is x[row_index[s]] (x float32 or bfloat16; row_index int64, or None for x itself), optionally through
    SwiGLU (x holds gate | up) and the ConvRot rotation first, as kernels.rotate would give it. Rows outside every
    group are left unset."""
    fmt = _lib.FORMATS[kind]
    w = fields[_lib.WEIGHT_KEY[kind]]
    scale = fields["scale"]
    if x.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"grouped_mma takes float32 or bfloat16 rows, not {x.dtype}")
    x = x.contiguous()
    K = x.shape[1] // 2 if swiglu else x.shape[1]
    rows = row_index.shape[0] if row_index is not None else x.shape[0]
    mode = (GM_ROTATE if rotate else 0) | (GM_SWIGLU if swiglu else 0)
    out = torch.empty((rows, n), dtype=torch.float32, device=x.device)
    size = lib().d3_grouped_mma_workspace(int(tiles), K)
    ws = torch.empty((max(size, 256),), dtype=torch.uint8, device=x.device)
    if row_index is not None:
        row_index = row_index.to(torch.int64).contiguous()
    with _on(x.device):
        check(lib().d3_grouped_mma(fmt, _ptr(x), int(x.dtype == torch.bfloat16), _ptr(row_index), mode, _ptr(groups),
                                   groups.shape[0], int(tiles), _ptr(w), _ptr(scale), _ptr(fields.get("s_channel")),
                                   _ptr(codebook), w.shape[0], _ptr(out), n, K, _ptr(ws), ws.numel(),
                                   _stream(x.device)), "grouped_mma")
    return out


def prefill_combine(sorted_out, pos, weights, dtype=torch.bfloat16):
    """[T, H] `dtype` (bfloat16 or float32): out[t] = sum over k' of weights[t, k'] * sorted_out[pos[t, k']] in rank
    order (the scatter, weighting and sum of drama3/offload.py:146-149 in one launch); pos [T, k] int64, weights
    [T, k] fp32 or bf16."""
    T, k = pos.shape
    H = sorted_out.shape[1]
    if dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"prefill_combine writes bfloat16 or float32, not {dtype}")
    out = torch.empty((T, H), dtype=dtype, device=sorted_out.device)
    weights = weights.contiguous()
    if weights.dtype not in (torch.float32, torch.bfloat16):
        weights = weights.float()
    with _on(sorted_out.device):
        check(lib().d3_prefill_combine(_ptr(sorted_out.contiguous()), _ptr(pos.to(torch.int64).contiguous()),
                                       _ptr(weights), int(weights.dtype == torch.bfloat16), T, k, H, _ptr(out),
                                       int(dtype == torch.float32), _stream(sorted_out.device)), "prefill_combine")
    return out


def moe_decode_ep(kind, x, ids, weights, banks, e_first, num_experts, codebooks=(None, None), workspace=None,
                  partial=None, exchange=None):
    """[M, H] float32: moe_decode over this rank's experts only (expert parallelism). `banks` hold experts
    [e_first, e_first + E_local) of the num_experts routed ones (bank expert 0 = expert e_first); pairs routed to other
    ranks' experts are skipped. The result is the routing-weighted sum over this rank's pairs, in rank order;
    summing the ranks' results and rounding to bf16 gives moe_decode's output. With `exchange` (the device struct
    of an ep.PeerExchange) the partial is pushed into every rank's exchange area instead and None is returned;
    ep_reduce then finishes the layer."""
    fmt = _lib.FORMATS[kind]
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"moe_decode_ep takes bfloat16 or float32 rows, not {x.dtype}")
    gate_up, down = banks
    wkey = _lib.WEIGHT_KEY[kind]
    M, H = x.shape
    k = ids.shape[-1]
    w13, w2 = gate_up[wkey], down[wkey]
    e_local = w2.shape[0] // H
    I = w13.shape[0] // (2 * e_local)
    if partial is None and exchange is None:
        partial = torch.empty((M, H), dtype=torch.float32, device=x.device)
    if workspace is None:
        workspace = _default_workspace(M, k, I, x.device)
    x = x.contiguous()
    ids = ids.reshape(M, k).contiguous()
    weights = weights.reshape(M, k).float().contiguous()
    with _on(x.device):
        check(lib().d3_moe_decode_ep(fmt, _ptr(x), int(x.dtype == torch.bfloat16), M, k, int(num_experts),
                                     int(e_first), e_local, H, I, _ptr(ids), _ptr(weights), _ptr(w13),
                                     _ptr(gate_up["scale"]), _ptr(gate_up.get("s_channel")), _ptr(w2),
                                     _ptr(down["scale"]), _ptr(down.get("s_channel")), _ptr(codebooks[0]),
                                     _ptr(codebooks[1]), _ptr(partial), _ptr(exchange), _ptr(workspace),
                                     workspace.numel(), _stream(x.device)), "moe_decode_ep")
    return partial


def ep_reduce(exchange, M, H, out=None):
    """[M, H] bfloat16: waits (bounded) until every rank has pushed its partial for this call into this rank's
    exchange area, then sums them in rank order. `exchange` is the device struct of an ep.PeerExchange."""
    if out is None:
        out = torch.empty((M, H), dtype=torch.bfloat16, device=exchange.device)
    with _on(exchange.device):
        check(lib().d3_ep_reduce(_ptr(exchange), M, H, _ptr(out), _stream(exchange.device)), "ep_reduce")
    return out


def decode_workspace(rows, k, intermediate, device):
    """The workspace moe_decode needs, allocated once by the caller and reused by every call (graph-captured steps
    included). It must start zeroed: its last bytes are the kernel's grid-barrier ticket counter, which each call
    advances by a whole number of rounds, so it never needs resetting. Calls that share one workspace must not overlap
    on the GPU."""
    size = lib().d3_moe_decode_workspace(rows, k, intermediate)
    return torch.zeros((size,), dtype=torch.uint8, device=device)


_WORKSPACES = {}


def _default_workspace(rows, k, intermediate, device):
    """The workspace of a decode call made without one: one per (device, stream, rows, k, intermediate), made on first
    use and kept, so repeated calls allocate and clear nothing (calls on one stream never overlap; calls on different
    streams get different workspaces). During a CUDA-graph capture a fresh one is made (and zeroed) inside the
    graph instead, which owns it."""
    device = torch.device(device)
    if torch.cuda.is_current_stream_capturing():
        return decode_workspace(rows, k, intermediate, device)
    key = (device, torch.cuda.current_stream(device).cuda_stream, rows, k, intermediate)
    if key not in _WORKSPACES:
        _WORKSPACES[key] = decode_workspace(rows, k, intermediate, device)
    return _WORKSPACES[key]


def moe_decode(kind, x, ids, weights, banks, codebooks=(None, None), workspace=None, out=None):
    """[M, H] bfloat16: rows x [M, H] (bfloat16 or float32, M <= 16) through their routed experts ids [M, k] (int64)
    mixed by weights [M, k], with banks (gate_up, down) held whole on the GPU in the reference layouts:
    fp8 {"weight" uint8 [E*2I, H] / [E*H, I], "scale" fp32 block scales}; int8 {"_qdata", "scale"};
    w4/w6 {"_qdata", "scale" (e4m3 bytes), "s_channel"} and a codebook per bank for w4; the BASELINE layouts fp8c
    {"weight", "scale" fp32 [E*N]} and w4a8 / w6a8 {"_qdata", "scale" bf16 [E*N, K/128]}. Each routed expert is read
    once for all M rows."""
    fmt = _lib.FORMATS[kind]
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"moe_decode takes bfloat16 or float32 rows, not {x.dtype}")
    gate_up, down = banks
    wkey = _lib.WEIGHT_KEY[kind]
    M, H = x.shape
    k = ids.shape[-1]
    w13, w2 = gate_up[wkey], down[wkey]
    E = w2.shape[0] // H
    I = w13.shape[0] // (2 * E)
    if out is None:
        out = torch.empty((M, H), dtype=torch.bfloat16, device=x.device)
    if workspace is None:
        workspace = _default_workspace(M, k, I, x.device)
    x = x.contiguous()
    ids = ids.reshape(M, k).contiguous()
    weights = weights.reshape(M, k).float().contiguous()
    scale13, scale2 = gate_up["scale"], down["scale"]
    with _on(x.device):
        check(lib().d3_moe_decode(fmt, _ptr(x), int(x.dtype == torch.bfloat16), M, k, E, H, I, _ptr(ids),
                                  _ptr(weights), _ptr(w13), _ptr(scale13), _ptr(gate_up.get("s_channel")), _ptr(w2),
                                  _ptr(scale2), _ptr(down.get("s_channel")), _ptr(codebooks[0]), _ptr(codebooks[1]),
                                  _ptr(out), _ptr(workspace), workspace.numel(), _stream(x.device)), "moe_decode")
    return out
