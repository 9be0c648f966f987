"""Packing float experts into the layouts the kernels read, on the host cores (the C++ packers in csrc/pack.cpp):
the converter step of the reference (tools/convert.py:48-82,179-215) with plain nearest rounding, for the reference's
layouts (fp8 block-scaled, int8 ConvRot, w4 / w6 codes) and the BASELINE ones (fp8c, w4a8, w6a8). Banks come back as
host torch tensors in the fields moe_decode / grouped_mma / resident_prefill and the offload store take, flat over
experts ([E * N, ...], expert e's rows contiguous)."""
import dataclasses
import json

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


# ---------------------------------------------------------------------------------------------------------------
# The converter's on-disk expert layout (tools/convert.py:179-215): state-dict entries per layer, and back to banks.
# The file's "drama3_format" metadata value of each reference layout (tools/convert.py:287).
DRAMA3_FORMAT = {"fp8": "fp8", "int8": "int8_convrot", "w4": "w4a8", "w6": "w6a8"}
CONVROT_GROUP = 256
CODES_GROUP = 16


def _comfy_quant(conf):
    """The layout's config as the uint8 tensor of its JSON text (tools/convert.py:56-58,74-75)."""
    return torch.tensor(list(json.dumps(conf).encode()), dtype=torch.uint8)


def expert_state(kind, layer, gate_up, down, threads=0, codebook=CODEBOOK4):
    """One layer's float experts, gate_up [E, 2I, H] (gate rows then up rows, tools/convert.py:195) and down [E, H, I],
    packed into the converter's state-dict entries for `kind` ("fp8", "int8", "w4", "w6"):
      fp8:  model.layers.{layer}.mlp.experts.{gate_up,down}_{weight [E, N, K] float8_e4m3fn, scale [E, N/128, K/128]
            fp32} (tools/convert.py:181-189);
      int8: model.layers.{layer}.mlp.experts.{gate_up,down}_proj.{weight [E, N, K] int8, weight_scale [E, N, 1] fp32,
            comfy_quant} (:207-213);
      w4 / w6: ....{gate_up,down}_proj.{weight [E, N, K*bits/8] uint8, weight_s_rel [E, N, K/16] uint8 (e4m3),
            weight_s_channel [E, N] fp32, comfy_quant, weight_codebook fp32 [16] (w4 only)} (:61-82, :199-205).
    The rounding is this module's plain nearest rounding, so the codes are not comfy_kitchen's; the layout is."""
    out = {}
    for bank, w in (("gate_up", gate_up), ("down", down)):
        w = torch.as_tensor(w)
        E, N, K = w.shape
        fields = pack_bank(kind, w, threads, codebook)
        if kind == "fp8":
            prefix = f"model.layers.{layer}.mlp.experts.{bank}"
            out[f"{prefix}_weight"] = fields["weight"].view(E, N, K).view(torch.float8_e4m3fn)
            out[f"{prefix}_scale"] = fields["scale"].view(E, N // 128, K // 128)
            continue
        module = f"model.layers.{layer}.mlp.experts.{bank}_proj"
        if kind == "int8":
            out[f"{module}.weight"] = fields["_qdata"].view(E, N, K)
            out[f"{module}.weight_scale"] = fields["scale"].view(E, N, 1)
            out[f"{module}.comfy_quant"] = _comfy_quant({"format": "int8_tensorwise", "convrot": True,
                                                         "convrot_groupsize": CONVROT_GROUP, "num_experts": E})
            continue
        bits = int(kind[1])
        out[f"{module}.weight"] = fields["_qdata"].view(E, N, K * bits // 8)
        out[f"{module}.weight_s_rel"] = fields["scale"].view(E, N, K // CODES_GROUP)
        out[f"{module}.weight_s_channel"] = fields["s_channel"].view(E, N)
        out[f"{module}.comfy_quant"] = _comfy_quant({"format": "asym_w4a8_int8" if bits == 4 else "w6a8_int8",
                                                     "group_size": CODES_GROUP, "convrot_groupsize": CONVROT_GROUP,
                                                     "num_experts": E})
        if bits == 4:
            out[f"{module}.weight_codebook"] = torch.as_tensor(codebook, dtype=torch.float32).clone()
    return out


def banks_from_state(kind, state, layer):
    """The converter's entries of one layer (expert_state's keys) -> (gate_up fields, down fields, codebooks): flat
    banks [E * N, ...] in the fields the kernels and the offload store take (drama3/offload.py:72-90,755-766), and
    each bank's fp32 codebook for w4 (a bank holds one table, tools/convert.py:62-63), else (None, None)."""
    banks = []
    for bank in ("gate_up", "down"):
        if kind == "fp8":
            prefix = f"model.layers.{layer}.mlp.experts.{bank}"
            w, s = state[f"{prefix}_weight"], state[f"{prefix}_scale"]
            E, N, K = w.shape
            banks.append({"weight": w.view(torch.uint8).reshape(E * N, K), "scale": s.reshape(E * N // 128, K // 128)})
            continue
        module = f"model.layers.{layer}.mlp.experts.{bank}_proj"
        conf = json.loads(bytes(state[f"{module}.comfy_quant"].tolist()).decode())
        q = state[f"{module}.weight"]
        E, N = q.shape[:2]
        if kind == "int8":
            if conf.get("format") != "int8_tensorwise" or conf.get("convrot_groupsize") != CONVROT_GROUP:
                raise ValueError(f"{module}: not an int8 ConvRot bank ({conf})")
            banks.append({"_qdata": q.reshape(E * N, -1), "scale": state[f"{module}.weight_scale"].reshape(E * N)})
            continue
        want = "asym_w4a8_int8" if kind == "w4" else "w6a8_int8"
        if conf.get("format") != want or conf.get("group_size") != CODES_GROUP:
            raise ValueError(f"{module}: not a {kind} bank ({conf})")
        banks.append({"_qdata": q.reshape(E * N, -1),
                      "scale": state[f"{module}.weight_s_rel"].reshape(E * N, -1),
                      "s_channel": state[f"{module}.weight_s_channel"].reshape(E * N)})
    codebooks = (None, None)
    if kind == "w4":
        codebooks = tuple(state[f"model.layers.{layer}.mlp.experts.{bank}_proj.weight_codebook"].float()
                          for bank in ("gate_up", "down"))
    return banks[0], banks[1], codebooks


# ---------------------------------------------------------------------------------------------------------------
# Packed banks dressed as comfy's quantized tensors, for the modules that recognize those (offload.kernel_bank).
@dataclasses.dataclass
class PackedParams:
    """The parameter fields of comfy's TensorWiseINT8Layout / AsymW4A8Int8Layout that the expert path reads."""
    orig_shape: tuple
    scale: torch.Tensor
    s_channel: torch.Tensor = None
    codebook: torch.Tensor = None
    convrot: bool = True
    convrot_groupsize: int = CONVROT_GROUP
    group_size: int = CODES_GROUP
    correction: object = None
    transposed: bool = False


class PackedWeight:
    """A flat packed bank [E * N, ...] with the attributes of comfy's QuantizedTensor (`_qdata`, `_params`,
    `_layout_cls`), so that offload.kernel_bank, model.Experts and offload.ExpertStore take it as they take a
    converted checkpoint's expert weight."""

    def __init__(self, layout, qdata, params):
        self._layout_cls, self._qdata, self._params = layout, qdata, params

    def to(self, device):
        """The same bank with every tensor on `device`."""
        moved = {f.name: (v.to(device) if torch.is_tensor(v) else v)
                 for f in dataclasses.fields(self._params) for v in [getattr(self._params, f.name)]}
        return PackedWeight(self._layout_cls, self._qdata.to(device), PackedParams(**moved))


def packed_weight(kind, w, threads=0, codebook=CODEBOOK4):
    """Float experts w [E, N, K] -> a PackedWeight of layout `kind` on the host: the reference's "int8" (ConvRot),
    "w4", "w6", or the BASELINE "w4a8" / "w6a8" (layout name offload.WA8_LAYOUT)."""
    if kind not in ("int8", "w4", "w6", "w4a8", "w6a8"):
        raise ValueError(f"no quantized-tensor form for {kind}: fp8 banks are FP8Experts parameters")
    w = torch.as_tensor(w)
    K = w.shape[-1]
    fields = pack_bank(kind, w, threads, codebook)
    rows = fields["_qdata"].shape[0]
    if kind == "int8":
        return PackedWeight("TensorWiseINT8Layout", fields["_qdata"],
                            PackedParams((rows, K), scale=fields["scale"].view(rows, 1)))
    if kind in ("w4a8", "w6a8"):
        from .offload import WA8_LAYOUT
        return PackedWeight(WA8_LAYOUT, fields["_qdata"],
                            PackedParams((rows, K), scale=fields["scale"], convrot=False, convrot_groupsize=0,
                                         group_size=128))
    book = torch.as_tensor(codebook, dtype=torch.float32).clone() if kind == "w4" else None
    return PackedWeight("AsymW4A8Int8Layout", fields["_qdata"],
                        PackedParams((rows, K), scale=fields["scale"], s_channel=fields["s_channel"], codebook=book))
