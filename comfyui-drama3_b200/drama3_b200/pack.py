"""Packing float experts into the BASELINE layouts the kernels read, on the host cores (the C++ packers in
csrc/pack.cpp): banks as torch tensors in the fields moe_decode / grouped_mma / resident_prefill take."""
import torch

from . import _lib
from ._lib import check, lib


def _rows(w):
    w = torch.as_tensor(w)
    if w.device.type != "cpu":
        raise ValueError("the packers run on host memory")
    w = w.detach().to(torch.float32).contiguous()
    return w, w.reshape(-1, w.shape[-1])


def pack_fp8c(w, threads=0):
    """Experts w [E, N, K] (or rows [R, K]) -> {"weight": uint8 [E*N, K] e4m3, "scale": fp32 [E*N]}: per-row
    absmax / 448 scales, nearest e4m3 with ties to even."""
    w, flat = _rows(w)
    rows, K = flat.shape
    codes = torch.empty((rows, K), dtype=torch.uint8)
    scale = torch.empty((rows,), dtype=torch.float32)
    check(lib().d3_pack_fp8c(flat.data_ptr(), rows, K, codes.data_ptr(), scale.data_ptr(), int(threads)), "pack_fp8c")
    return {"weight": codes, "scale": scale}


def pack_wa8(w, bits, threads=0):
    """Experts w [E, N, K] (or rows [R, K]) -> {"_qdata": uint8 [E*N, K*bits/8], "scale": bf16 [E*N, K/128]}: W4A8
    (bits 4, two codes per byte) or W6A8 (bits 6, four codes per three bytes) with absmax / qmax scales per 128
    columns ([3])."""
    w, flat = _rows(w)
    rows, K = flat.shape
    packed = torch.empty((rows, K * bits // 8), dtype=torch.uint8)
    scale = torch.empty((rows, K // 128), dtype=torch.int16)
    check(lib().d3_pack_wa8(flat.data_ptr(), rows, K, int(bits), packed.data_ptr(), scale.data_ptr(), int(threads)),
          "pack_wa8")
    return {"_qdata": packed, "scale": scale.view(torch.bfloat16)}


def pack_bank(kind, w, threads=0):
    """pack_fp8c / pack_wa8 by layout name ("fp8c", "w4a8", "w6a8")."""
    if kind == "fp8c":
        return pack_fp8c(w, threads)
    if kind in ("w4a8", "w6a8"):
        return pack_wa8(w, int(kind[1]), threads)
    raise ValueError(f"no packer for {kind}")
