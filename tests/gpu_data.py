"""Seeded synthetic inputs for the GPU tests and the bench: banks in the reference layouts, rows, routing."""
import numpy as np
import torch

from oracle import moe

KINDS = ("fp8", "int8", "w4", "w6")
BASELINE_KINDS = ("fp8c", "w4a8", "w6a8")
WKEY = {"fp8": "weight", "int8": "_qdata", "w4": "_qdata", "w6": "_qdata", "fp8c": "weight", "w4a8": "_qdata",
        "w6a8": "_qdata"}


def _rand_e4m3(gen, shape, lo, hi, device):
    """e4m3 bytes in [lo, hi) (positive, never the NaN code)."""
    return torch.randint(lo, hi, shape, generator=gen, dtype=torch.int32).to(device=device, dtype=torch.uint8)


def rand_bank(kind, E, N, K, seed, device):
    """A flat bank [E * N, ...] of random valid codes in `kind`'s layout (fields as drama3/offload.py keys them)."""
    gen = torch.Generator().manual_seed(seed)
    if kind == "fp8":
        w = torch.randint(0, 254, (E * N, K), generator=gen, dtype=torch.int32)
        w = torch.where(w >= 0x7F, w + 1, w).to(torch.uint8)  # skip 0x7F; 0xFF is out of range
        s = torch.rand((E * N // 128, K // 128), generator=gen) * 1e-4 + 5e-5
        return {"weight": w.to(device), "scale": s.to(device)}
    if kind == "int8":
        q = torch.randint(-127, 128, (E * N, K), generator=gen, dtype=torch.int8)
        s = torch.rand((E * N,), generator=gen) * 2e-4 + 1e-4
        return {"_qdata": q.to(device), "scale": s.to(device)}
    if kind == "fp8c":
        w = torch.randint(0, 254, (E * N, K), generator=gen, dtype=torch.int32)
        w = torch.where(w >= 0x7F, w + 1, w).to(torch.uint8)
        s = torch.rand((E * N,), generator=gen) * 1e-4 + 5e-5
        return {"weight": w.to(device), "scale": s.to(device)}
    if kind in ("w4a8", "w6a8"):
        q = torch.randint(0, 256, (E * N, K * int(kind[1]) // 8), generator=gen, dtype=torch.int32).to(torch.uint8)
        s = (torch.rand((E * N, K // 128), generator=gen) * 2e-3 + 1e-3).to(torch.bfloat16)
        return {"_qdata": q.to(device), "scale": s.to(device)}
    bits = int(kind[1])
    q = torch.randint(0, 256, (E * N, K * bits // 8), generator=gen, dtype=torch.int32).to(torch.uint8)
    lo, hi = (0x50, 0x70) if bits == 4 else (0x30, 0x50)
    g = _rand_e4m3(gen, (E * N, K // 16), lo, hi, "cpu")
    c = torch.rand((E * N,), generator=gen) * 2e-4 + 1e-4
    return {"_qdata": q.to(device), "scale": g.to(device), "s_channel": c.to(device)}


def codebooks(kind, device):
    if kind != "w4":
        return (None, None)
    cb = torch.from_numpy(moe.CODEBOOK4).to(device)
    return (cb, cb.clone())


def rand_rows(M, H, seed, device):
    gen = torch.Generator().manual_seed(seed)
    return torch.randn((M, H), generator=gen).to(torch.bfloat16).to(device)


def rand_routing(M, E, k, seed, device, skew=None):
    """Distinct top-k experts per row and bf16-valued softmax weights; `skew` biases expert popularity."""
    gen = torch.Generator().manual_seed(seed)
    logits = torch.randn((M, E), generator=gen)
    if skew is not None:
        logits = logits + torch.as_tensor(skew, dtype=torch.float32)
    w, ids = torch.softmax(logits, dim=-1).topk(k, dim=-1)
    w = (w / w.sum(-1, keepdim=True)).to(torch.bfloat16).float()
    return ids.to(device), w.to(device)


def to_np(t):
    t = t.cpu()
    return t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()


def to_np_bank(bank):
    return {n: to_np(t) for n, t in bank.items()}


def baseline_oracle_decode(kind, x, ids, weights, banks):
    """oracle.baseline_decode on the whole (small) banks."""
    return moe.baseline_decode(kind, x.float().cpu().numpy(), ids.cpu().numpy(), weights.cpu().numpy(),
                               tuple(to_np_bank(b) for b in banks))


def subset(kind, bank, experts, rows):
    """numpy fields of the listed experts only (expert i of the subset = experts[i])."""
    out = {}
    for n, t in bank.items():
        per = t.shape[0] // (bank[WKEY[kind]].shape[0] // rows)
        idx = torch.as_tensor(experts, device=t.device)
        out[n] = t.view(-1, per, *t.shape[1:]).index_select(0, idx).reshape(-1, *t.shape[1:]).cpu().numpy()
    return out


def oracle_decode(kind, x, ids, weights, banks, cbs, H):
    """oracle.moe_decode on the used experts only."""
    used = sorted(set(ids.reshape(-1).tolist()))
    remap = {e: i for i, e in enumerate(used)}
    gate_up, down = banks
    n1 = gate_up[WKEY[kind]].shape[0] // (down[WKEY[kind]].shape[0] // H)
    sub = (subset(kind, gate_up, used, n1), subset(kind, down, used, H))
    local = np.vectorize(remap.get)(ids.cpu().numpy())
    cbn = tuple(None if c is None else c.cpu().numpy() for c in cbs)
    return moe.moe_decode(kind, x.float().cpu().numpy(), local, weights.cpu().numpy(), sub, cbn)


def rel_l2(a, b):
    a = torch.as_tensor(a).double().cpu()
    b = torch.as_tensor(b).double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))
