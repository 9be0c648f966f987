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
