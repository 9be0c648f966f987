"""Packing float experts into the layouts the kernels read, on the host cores (the C++ packers in csrc/pack.cpp):
the converter step of the reference (tools/convert.py:48-82,179-215) with plain nearest rounding, for the reference's
layouts (fp8 block-scaled, int8 ConvRot, w4 / w6 codes) and the BASELINE ones (fp8c, w4a8, w6a8). Banks come back as
host torch tensors in the fields moe_decode / grouped_mma / resident_prefill and the offload store take, flat over
experts ([E * N, ...], expert e's rows contiguous)."""
import torch

from ._lib import check, lib

# the 16-entry codebook the w4 packer uses when none is given: a symmetric nonuniform grid on [-1, 1]
CODEBOOK4 = (-1.0, -0.6962, -0.5251, -0.3949, -0.2844, -0.1848, -0.0911, 0.0, 0.0796, 0.1609, 0.2461, 0.3379, 0.4407,
             0.5626, 0.7230, 1.0)


def _rows(w):
    w = torch.as_tensor(w)
    if w.device.type != "cpu":
        raise ValueError("the packers run on host memory")
    w = w.detach().to(torch.float32).contiguous()
    return w.reshape(-1, w.shape[-1])


def pack_fp8_blocks(w, threads=0):
    """Experts w [E, N, K] (or rows [R, K]) -> {"weight": uint8 [E*N, K] e4m3, "scale": fp32 [E*N/128, K/128]}: block
    absmax / 448 per 128 x 128 block (the fp8 layout, tools/convert.py:179-189)."""
    flat = _rows(w)
    rows, K = flat.shape
    codes = torch.empty((rows, K), dtype=torch.uint8)
    scale = torch.empty((rows // 128, K // 128), dtype=torch.float32)
    check(lib().d3_pack_fp8_blocks(flat.data_ptr(), rows, K, codes.data_ptr(), scale.data_ptr(), int(threads)),
          "pack_fp8_blocks")
    return {"weight": codes, "scale": scale}


def pack_int8_convrot(w, threads=0):
    """Experts w [E, N, K] -> {"_qdata": int8 [E*N, K], "scale": fp32 [E*N]}: rows in the ConvRot basis (times the
    normalized 256-point Hadamard matrix per 256 columns), absmax / 127 row scales (tools/convert.py:48-53)."""
    flat = _rows(w)
    rows, K = flat.shape
    q = torch.empty((rows, K), dtype=torch.int8)
    scale = torch.empty((rows,), dtype=torch.float32)
    check(lib().d3_pack_int8_convrot(flat.data_ptr(), rows, K, q.data_ptr(), scale.data_ptr(), int(threads)),
          "pack_int8_convrot")
    return {"_qdata": q, "scale": scale}


def pack_codes(w, bits, codebook=CODEBOOK4, threads=0):
    """Experts w [E, N, K] -> {"_qdata": uint8 [E*N, K*bits/8], "scale": uint8 e4m3 [E*N, K/16], "s_channel": fp32
    [E*N]}: the reference's w4 (codebook, bits 4) / w6 (bits 6) planes in the ConvRot basis (tools/convert.py:61-82,
    decoded by drama3/kernels.py:466-483). codebook: 16 values (bits 4; the kernels read it as fp32 [16])."""
    flat = _rows(w)
    rows, K = flat.shape
    book = torch.as_tensor(codebook, dtype=torch.float32).contiguous()
    if bits == 4 and book.numel() != 16:
        raise ValueError("a w4 codebook has 16 entries")
    codes = torch.empty((rows, K * bits // 8), dtype=torch.uint8)
    group = torch.empty((rows, K // 16), dtype=torch.uint8)
    chan = torch.empty((rows,), dtype=torch.float32)
    check(lib().d3_pack_codes(flat.data_ptr(), rows, K, int(bits), book.data_ptr(), codes.data_ptr(), group.data_ptr(),
                              chan.data_ptr(), int(threads)), "pack_codes")
    return {"_qdata": codes, "scale": group, "s_channel": chan}


def pack_fp8c(w, threads=0):
    """Experts w [E, N, K] (or rows [R, K]) -> {"weight": uint8 [E*N, K] e4m3, "scale": fp32 [E*N]}: per-row
    absmax / 448 scales, nearest e4m3 with ties to even."""
    flat = _rows(w)
    rows, K = flat.shape
    codes = torch.empty((rows, K), dtype=torch.uint8)
    scale = torch.empty((rows,), dtype=torch.float32)
    check(lib().d3_pack_fp8c(flat.data_ptr(), rows, K, codes.data_ptr(), scale.data_ptr(), int(threads)), "pack_fp8c")
    return {"weight": codes, "scale": scale}


def pack_wa8(w, bits, threads=0):
    """Experts w [E, N, K] (or rows [R, K]) -> {"_qdata": uint8 [E*N, K*bits/8], "scale": bf16 [E*N, K/128]}: W4A8
    (bits 4, two codes per byte) or W6A8 (bits 6, four codes per three bytes) with absmax / qmax scales per 128
    columns ([3])."""
    flat = _rows(w)
    rows, K = flat.shape
    packed = torch.empty((rows, K * bits // 8), dtype=torch.uint8)
    scale = torch.empty((rows, K // 128), dtype=torch.int16)
    check(lib().d3_pack_wa8(flat.data_ptr(), rows, K, int(bits), packed.data_ptr(), scale.data_ptr(), int(threads)),
          "pack_wa8")
    return {"_qdata": packed, "scale": scale.view(torch.bfloat16)}


def pack_bank(kind, w, threads=0, codebook=CODEBOOK4):
    """The packer of layout `kind` ("fp8", "int8", "w4", "w6", "fp8c", "w4a8", "w6a8") on float experts w."""
    if kind == "fp8":
        return pack_fp8_blocks(w, threads)
    if kind == "int8":
        return pack_int8_convrot(w, threads)
    if kind in ("w4", "w6"):
        return pack_codes(w, int(kind[1]), codebook, threads)
    if kind == "fp8c":
        return pack_fp8c(w, threads)
    if kind in ("w4a8", "w6a8"):
        return pack_wa8(w, int(kind[1]), threads)
    raise ValueError(f"no packer for {kind}")
