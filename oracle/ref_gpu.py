"""TEST INFRASTRUCTURE ONLY. The reference's own CUDA kernels (oracle/_ref/ref_kernels.cubin, built by
oracle/build_ref.py from drama3/kernels.py) launched on the current GPU through the CUDA driver API.

The launchers restate the reference's Python launchers (drama3/kernels.py:618-724) and drivers
(drama3/offload.py:108-149): same grids, blocks, shared memory and argument order, and torch for the glue the
reference does in torch. Used by the GPU tests as the bit-exact pin for decode routing, slot resolve and rotation,
and by bench.py to time the reference's GPU path beside this library's.
"""
import ctypes
import functools
import itertools
from pathlib import Path

import torch
import torch.nn as nn

CUBIN = Path(__file__).resolve().parent / "_ref" / "ref_kernels.cubin"
ROWS_PER_BLOCK = 16  # drama3/kernels.py:590


class _Driver:
    def __init__(self):
        self.cu = ctypes.CDLL("libcuda.so.1")
        for name in ("cuInit", "cuModuleLoadData", "cuModuleGetFunction", "cuLaunchKernel", "cuCtxGetCurrent",
                     "cuDevicePrimaryCtxRetain", "cuCtxSetCurrent", "cuDeviceGet", "cuFuncSetAttribute"):
            getattr(self.cu, name).restype = ctypes.c_int
        self.check(self.cu.cuInit(0), "cuInit")
        self.modules = {}

    @staticmethod
    def check(status, what):
        if status != 0:
            raise RuntimeError(f"{what}: CUresult {status}")

    def function(self, name, device_index):
        if device_index not in self.modules:
            dev = ctypes.c_int()
            self.check(self.cu.cuDeviceGet(ctypes.byref(dev), device_index), "cuDeviceGet")
            ctx = ctypes.c_void_p()
            self.check(self.cu.cuDevicePrimaryCtxRetain(ctypes.byref(ctx), dev), "cuDevicePrimaryCtxRetain")
            self.check(self.cu.cuCtxSetCurrent(ctx), "cuCtxSetCurrent")
            image = CUBIN.read_bytes()
            module = ctypes.c_void_p()
            self.check(self.cu.cuModuleLoadData(ctypes.byref(module), image), "cuModuleLoadData")
            self.modules[device_index] = (module, {})
        module, funcs = self.modules[device_index]
        if name not in funcs:
            fn = ctypes.c_void_p()
            self.check(self.cu.cuModuleGetFunction(ctypes.byref(fn), module, name.encode()), f"function {name}")
            funcs[name] = fn
        return funcs[name]


@functools.cache
def _driver():
    if not CUBIN.exists():
        raise FileNotFoundError(f"{CUBIN} is missing: run oracle/build_ref.py where the reference is checked out")
    return _Driver()


def available():
    return CUBIN.exists() and torch.cuda.is_available()


def _arg(v):
    if isinstance(v, torch.Tensor):
        return ctypes.c_void_p(v.data_ptr())
    if isinstance(v, bool):
        return ctypes.c_int(int(v))
    if isinstance(v, int):
        return ctypes.c_int(v)
    if isinstance(v, float):
        return ctypes.c_double(v)
    raise TypeError(type(v))


def _launch(name, device, grid, block, args, shared_mem=0):
    """drama3/kernels.py:599-601 (_launch), through cuLaunchKernel."""
    drv = _driver()
    fn = drv.function(name, device.index if device.index is not None else torch.cuda.current_device())
    cargs = [_arg(a) for a in args]
    params = (ctypes.c_void_p * len(cargs))(*[ctypes.cast(ctypes.pointer(a), ctypes.c_void_p) for a in cargs])
    stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
    drv.check(drv.cu.cuLaunchKernel(fn, *grid, *block, shared_mem, stream, params, None), f"launch {name}")


# ---------------------------------------------------------------------------------------------------------------
# launchers: drama3/kernels.py:618-724
def resolve(ids, layer, layers, num_experts, half_life, cpu, admit, table, owner, score, at, pending, clock, budget,
            reads, step, share):
    plan = torch.empty((ids.shape[0], 2), dtype=torch.int32, device=ids.device)
    _launch("resolve_experts", ids.device, (1, 1, 1), (1024, 1, 1),
            [ids, ids.shape[0], layer, layers, num_experts, table, owner, score, at, pending, owner.shape[0], clock,
             budget, plan, reads, step, share, float(half_life), int(cpu), float(admit)])
    return plan


def rotate(x, only_if, swiglu=False):
    rows, width = x.shape
    k = width // 2 if swiglu else width
    out = torch.empty((rows, k), dtype=torch.float32, device=x.device)
    _launch("rotate_rows", x.device, (rows, 1, 1), (256, 1, 1),
            [x, int(x.dtype == torch.bfloat16), int(swiglu), k, out, only_if])
    return out


def route(logits, k):
    ids = torch.empty((1, k), dtype=torch.int64, device=logits.device)
    weights = torch.empty((1, k), dtype=torch.float32, device=logits.device)
    _launch("route_experts", logits.device, (1, 1, 1), (256, 1, 1), [logits, logits.shape[1], k, ids, weights])
    return ids, weights


def weighted_sum(parts, weights):
    out = torch.empty((1, parts.shape[1]), dtype=torch.bfloat16, device=parts.device)
    _launch("weighted_sum", parts.device, ((parts.shape[1] + 255) // 256, 1, 1), (256, 1, 1),
            [parts, weights, parts.shape[0], parts.shape[1], out])
    return out


def gemv_int8(x, ids, plan, took_over, late, slot_fields, host_fields, n):
    k, width = ids.shape[0], x.shape[1]
    out = torch.empty((k, n), dtype=torch.float32, device=x.device)
    _launch("gemv_int8", x.device, (n // ROWS_PER_BLOCK, k, 1), (256, 1, 1),
            [x, x.shape[0], ids, plan, took_over, int(late), slot_fields["_qdata"], slot_fields["scale"],
             host_fields["_qdata"], host_fields["scale"], out, n, width], shared_mem=4 * width)
    return out


def gemv_fp8(x, ids, plan, slot_fields, host_fields, n):
    k, width = ids.shape[0], x.shape[1]
    out = torch.empty((k, n), dtype=torch.float32, device=x.device)
    _launch("gemv_fp8", x.device, (n // ROWS_PER_BLOCK, k, 1), (256, 1, 1),
            [x, x.shape[0], ids, plan, slot_fields["weight"], slot_fields["scale"], host_fields["weight"],
             host_fields["scale"], out, n, width], shared_mem=4 * width)
    return out


def gemv_codes(x, ids, plan, slot_fields, host_fields, codebook, bits, n):
    k, width = ids.shape[0], x.shape[1]
    if codebook is None:
        codebook = host_fields["s_channel"]
    out = torch.empty((k, n), dtype=torch.float32, device=x.device)
    _launch("gemv_codes", x.device, (n // ROWS_PER_BLOCK, k, 1), (256, 1, 1),
            [x, x.shape[0], ids, plan, slot_fields["_qdata"], slot_fields["scale"], slot_fields["s_channel"],
             host_fields["_qdata"], host_fields["scale"], host_fields["s_channel"], codebook, bits, out, n, width],
            shared_mem=4 * width)
    return out


def grouped_int8(x, groups, slot_fields, host_fields, n):
    out = torch.empty((x.shape[0], n), dtype=torch.float32, device=x.device)
    _launch("grouped_int8", x.device, (n // ROWS_PER_BLOCK, groups.shape[0], 1), (256, 1, 1),
            [x, groups, slot_fields["_qdata"], slot_fields["scale"], host_fields["_qdata"], host_fields["scale"], out,
             n, x.shape[1]])
    return out


def grouped_fp8(x, groups, slot_fields, host_fields, n):
    out = torch.empty((x.shape[0], n), dtype=torch.float32, device=x.device)
    _launch("grouped_fp8", x.device, (n // ROWS_PER_BLOCK, groups.shape[0], 1), (256, 1, 1),
            [x, groups, slot_fields["weight"], slot_fields["scale"], host_fields["weight"], host_fields["scale"], out,
             n, x.shape[1]])
    return out


def grouped_codes(x, groups, slot_fields, host_fields, codebook, bits, n):
    out = torch.empty((x.shape[0], n), dtype=torch.float32, device=x.device)
    if codebook is None:
        codebook = host_fields["s_channel"]
    _launch("grouped_codes", x.device, (n // ROWS_PER_BLOCK, groups.shape[0], 1), (256, 1, 1),
            [x, groups, slot_fields["_qdata"], slot_fields["scale"], slot_fields["s_channel"], host_fields["_qdata"],
             host_fields["scale"], host_fields["s_channel"], codebook, bits, out, n, x.shape[1]])
    return out


# ---------------------------------------------------------------------------------------------------------------
# drivers: drama3/offload.py:93-149
def quantized_gemv(kind, x, ids, plan, took_over, late, slot_fields, host_fields, rows, codebook):
    if kind == "int8":
        return gemv_int8(x, ids, plan, took_over, late, slot_fields, host_fields, rows)
    return gemv_codes(x, ids, plan, slot_fields, host_fields, codebook, int(kind[1]), rows)


def quantized_grouped(kind, x, groups, slot_fields, host_fields, rows, codebook):
    if kind == "int8":
        return grouped_int8(x, groups, slot_fields, host_fields, rows)
    return grouped_codes(x, groups, slot_fields, host_fields, codebook, int(kind[1]), rows)


def resident_decode(x, ids, weights, banks, rows, kind, codebooks):
    (gate_up, down), (gate_up_rows, down_rows) = banks, rows
    plan = torch.stack((ids.to(torch.int32), torch.zeros_like(ids, dtype=torch.int32)), dim=-1)
    if kind == "fp8":
        gate, up = gemv_fp8(x.float(), ids, plan, gate_up, gate_up, gate_up_rows).chunk(2, dim=-1)
        out = gemv_fp8(nn.functional.silu(gate) * up, ids, plan, down, down, down_rows)
        return weighted_sum(out, weights.float())
    took_over, always = torch.arange(2, dtype=torch.int32, device=x.device).split(1)
    hidden = quantized_gemv(kind, rotate(x, always), ids, plan, took_over, False, gate_up, gate_up, gate_up_rows,
                            codebooks[0])
    out = quantized_gemv(kind, rotate(hidden, always, swiglu=True), ids, plan, took_over, False, down, down,
                         down_rows, codebooks[1])
    return weighted_sum(out, weights.float())


def lines_decode(x, ids, weights, banks, rows, kind, codebooks):
    """M rows decoded together, one resident_decode per row (drama3/model.py:111-113)."""
    return torch.cat([resident_decode(x[t:t + 1], ids[t], weights[t], banks, rows, kind, codebooks)
                      for t in range(x.shape[0])])


def grouped_experts(sorted_x, groups, slot_banks, host_banks, rows, kind, codebooks, always):
    if kind == "fp8":
        gate, up = grouped_fp8(sorted_x.float(), groups, slot_banks[0], host_banks[0], rows[0]).chunk(2, dim=-1)
        return grouped_fp8(nn.functional.silu(gate) * up, groups, slot_banks[1], host_banks[1], rows[1])
    hidden = quantized_grouped(kind, rotate(sorted_x.float(), always), groups, slot_banks[0], host_banks[0], rows[0],
                               codebooks[0])
    return quantized_grouped(kind, rotate(hidden, always, swiglu=True), groups, slot_banks[1], host_banks[1], rows[1],
                             codebooks[1])


def resident_prefill(x, topk_idx, topk_weight, banks, rows, kind, codebooks, num_experts):
    num_tokens, top_k = topk_idx.shape
    order = torch.argsort(topk_idx.reshape(-1))
    counts = torch.bincount(topk_idx.reshape(-1), minlength=num_experts).tolist()
    offsets = [0, *itertools.accumulate(counts)]
    groups = torch.tensor([(expert, expert, 0, offsets[expert], n) for expert, n in enumerate(counts) if n],
                          dtype=torch.int32)
    always = torch.ones((1,), dtype=torch.int32, device=x.device)
    sorted_out = grouped_experts(x[order // top_k], groups.to(x.device), banks, banks, rows, kind, codebooks, always)
    out = torch.empty_like(sorted_out)
    out[order] = sorted_out * topk_weight.reshape(-1)[order].unsqueeze(1).float()
    return out.view(num_tokens, top_k, -1).sum(dim=1).to(x.dtype)
