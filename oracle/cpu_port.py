"""TEST INFRASTRUCTURE ONLY. The reference's CPU path for a decode row, ported to torch on the host cores: the CPU
baseline of bench.py and its `--impl reference` arm (the reference's Python cannot travel to the GPU box).

It follows drama3/offload.py:771-784 (FP8Experts.experts / forward without the kernels): the row's k experts are
gathered and dequantized to the model dtype (dequantize_fp8, :163-167), then experts_decode (:192-199) runs two
matmuls (down as k x k blocks keeping the diagonal) and the weighted sum; lines decoded together run one row at a
time (drama3/model.py:111-113).
"""
import torch


def dequantize_fp8(weight_u8, scale, dtype):
    rows, cols = weight_u8.shape
    blocks = weight_u8.view(torch.float8_e4m3fn).float().view(rows // 128, 128, cols // 128, 128)
    return (blocks * scale[:, None, :, None]).view(rows, cols).to(dtype)


def experts(weight, scale, ids, dtype):
    """weight u8 [E, N, K], scale [E, N/128, K/128] -> the k experts' rows [k*N, K] in dtype."""
    w = weight.index_select(0, ids).flatten(0, 1)
    s = scale.index_select(0, ids).flatten(0, 1)
    return dequantize_fp8(w, s, dtype)


def experts_decode(x, gate_up, down, weights):
    k = weights.shape[0]
    h = torch.nn.functional.linear(x, gate_up).view(k, -1)
    gate, up = h.chunk(2, dim=-1)
    hidden = torch.nn.functional.silu(gate) * up
    out = torch.nn.functional.linear(hidden, down).view(k, k, -1).diagonal(dim1=0, dim2=1).T
    return (out * weights[:, None].to(out.dtype)).sum(0, keepdim=True)


def fp8_decode_lines(x, ids, weights, gate_up_w, gate_up_s, down_w, down_s, dtype=torch.bfloat16):
    """[M, H]: M rows, one at a time, through their fp8 experts (banks [E, N, K] uint8 + block scales)."""
    out = []
    for t in range(x.shape[0]):
        gu = experts(gate_up_w, gate_up_s, ids[t], dtype)
        dn = experts(down_w, down_s, ids[t], dtype)
        out.append(experts_decode(x[t:t + 1].to(dtype), gu, dn, weights[t]))
    return torch.cat(out)


# ---------------------------------------------------------------------------------------------------------------
# int8 ConvRot experts on the CPU: the reference's own CPU int8 path (drama3/offload.py:170-189, 245-249, 448-450)
def hadamard(size=256):
    """ConvRot's normalized regular Hadamard matrix (h4 Kronecker powers / sqrt(size), drama3/offload.py:170-176)."""
    h4 = torch.tensor([[1.0, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]])
    h = h4
    while h.shape[0] < size:
        h = torch.kron(h, h4)
    return h / size ** 0.5


def int8_linear(x_bf16, qdata, scale_bf16):
    """bf16 rows through int8 rows with bf16 per-row scales: QuantHostBank.cpu_linear (drama3/offload.py:245-249)."""
    return torch._weight_int8pack_mm(x_bf16, qdata, scale_bf16)


def int8_decode_row(x, ids, weights, gate_up_q, gate_up_s, down_q, down_s, rotation):
    """One row x [1, H] through its k int8 ConvRot experts on the CPU (experts_on_cpu, drama3/offload.py:179-189):
    the row rotated and rounded to bf16, each expert's gate_up, SwiGLU (float), the hidden row rotated and rounded
    to bf16, down; then the routing-weighted sum (drama3/offload.py:448-450). Banks: qdata int8 [E, N, K], scale
    [E, N] fp32 (the matmul takes bf16 scales). [1, H] float32."""
    k = ids.shape[0]
    H = x.shape[1]
    row = (x.float().view(1, -1, 256) @ rotation).flatten(1).to(torch.bfloat16)
    parts = []
    for e in ids.tolist():
        h = int8_linear(row, gate_up_q[e], gate_up_s[e].to(torch.bfloat16)).float()
        gate, up = h.chunk(2, dim=-1)
        hidden = torch.nn.functional.silu(gate) * up
        hidden = (hidden.view(1, -1, 256) @ rotation).flatten(1).to(torch.bfloat16)
        parts.append(int8_linear(hidden, down_q[e], down_s[e].to(torch.bfloat16)).float())
    return weights.float().view(1, k) @ torch.cat(parts).view(k, H)


# ---------------------------------------------------------------------------------------------------------------
# w4 / w6 code banks on the CPU. The reference runs these through comfy_kitchen's quantized matmuls, which are not
# available: this is a RESTATEMENT, labelled so wherever it is timed. Codes are decoded as drama3/kernels.py:466-483
# decodes them (the int8 grid, times s_channel), rounded to bf16 weights, then the decode's matmuls.
def decode_codes(qdata, group_scale, s_channel, K, bits, codebook):
    """Rows of a w4 / w6 bank -> bf16 weights [N, K] (rotated basis): value on the int8 grid times s_channel."""
    q = qdata.to(torch.int32)
    nib = torch.stack((q[:, :K // 2] & 0xF, q[:, :K // 2] >> 4), dim=-1).reshape(q.shape[0], K)
    if bits == 6:
        hi = q[:, K // 2:K // 2 + K // 4]
        top = torch.stack([(hi >> (2 * j)) & 3 for j in range(4)], dim=-1).reshape(q.shape[0], K)
        value = ((nib | (top << 4)) - 32).float()
    else:
        value = codebook[nib]
    s = group_scale.view(torch.float8_e4m3fn).float().repeat_interleave(16, dim=1)
    grid = torch.clamp(torch.round(value * s), -127, 127)
    return (grid * s_channel.view(-1, 1)).to(torch.bfloat16)


def codes_decode_row(x, ids, weights, bank13, bank2, bits, codebooks, rotation):
    """One row through its k w4 / w6 experts on the CPU (restatement): rotation, decoded bf16 weights, SwiGLU, the
    hidden row rotated, down, routing-weighted sum. bank = (qdata u8 [E, N, K*bits/8], group scales u8 [E, N, K/16],
    s_channel [E, N]). [1, H] float32."""
    H = x.shape[1]
    row = (x.float().view(1, -1, 256) @ rotation).flatten(1).to(torch.bfloat16)
    q13, g13, c13 = bank13
    q2, g2, c2 = bank2
    K2 = q2.shape[2] * 8 // bits
    parts = []
    for e in ids.tolist():
        h = torch.nn.functional.linear(row, decode_codes(q13[e], g13[e], c13[e], H, bits, codebooks[0])).float()
        gate, up = h.chunk(2, dim=-1)
        hidden = ((torch.nn.functional.silu(gate) * up).view(1, -1, 256) @ rotation).flatten(1).to(torch.bfloat16)
        parts.append(torch.nn.functional.linear(hidden, decode_codes(q2[e], g2[e], c2[e], K2, bits,
                                                                     codebooks[1])).float())
    return weights.float().view(1, -1) @ torch.cat(parts).view(len(parts), H)
