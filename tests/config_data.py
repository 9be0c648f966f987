"""The BASELINE configurations' seeded inputs, drawn the same way on every machine (test infrastructure).

Each config n draws from torch.Generator("cpu").manual_seed(seed_n), in this order: the router weight [E, H]
(N(0, 0.02), stored bf16), the gate_up experts [E, 2I, H] and the down experts [E, H, I] (N(0, 0.02), fp32), the
rows x [rows, H] (N(0, 1), stored bf16), then, for config 4 only, a permutation r of the ranks 1..E for the Zipf(1.1)
bias -1.1 ln(r_e) added to every row's router logits. The float experts are packed into each layout the config
names by the library's packers (byte-identical to the oracle's quantizers, tests/test_pack_cpu.py), and the routing
comes from the router logits bf16(x W_r^T + bias) computed in float64: the decode rule (oracle.moe.route, the
reference's route_experts) for decode rows, the prompt rule (oracle.moe.route_prefill) for a prompt's rows.

  config 1  seed 0  int8 ConvRot (per-row fp32 scales)                      1 row (decode)
  config 2  seed 1  fp8 128x128 block scales (reference) and fp8c (per-row)  1, 4, 16 rows (decode)
  config 3  seed 2  w4 codes (reference) and w4a8 (int4, bf16 g128 scales)   1, 16 rows (decode)
  config 4  seed 3  w6 codes (reference) and w6a8 (6-bit, bf16 g128 scales)  2048 rows (prompt pass), Zipf-skewed

tests/golden/make_configs.py writes the oracle's outputs on these inputs to tests/golden/configs.npz, with a
sha256 of every packed bank (so that a test can first check it packed the same bytes).
"""
import hashlib

import numpy as np
import torch

from oracle import moe

E, H, I, TOP_K = 128, 2048, 768, 8
CONFIGS = {
    1: {"seed": 0, "kinds": ("int8",), "rows": 1, "lines": (1,)},
    2: {"seed": 1, "kinds": ("fp8", "fp8c"), "rows": 16, "lines": (1, 4, 16)},
    3: {"seed": 2, "kinds": ("w4", "w4a8"), "rows": 16, "lines": (1, 16)},
    4: {"seed": 3, "kinds": ("w6", "w6a8"), "rows": 2048, "lines": None},
}
ZIPF = 1.1


def draw(n):
    """The float draws of config n: router (bf16), gate_up, down (fp32), x (bf16) and the bias (config 4), or None."""
    c = CONFIGS[n]
    gen = torch.Generator().manual_seed(c["seed"])
    router = (torch.randn((E, H), generator=gen) * 0.02).to(torch.bfloat16)
    gate_up = torch.randn((E, 2 * I, H), generator=gen) * 0.02
    down = torch.randn((E, H, I), generator=gen) * 0.02
    x = torch.randn((c["rows"], H), generator=gen).to(torch.bfloat16)
    bias = None
    if n == 4:
        ranks = torch.randperm(E, generator=gen) + 1
        bias = -ZIPF * torch.log(ranks.to(torch.float64))
    return {"router": router, "gate_up": gate_up, "down": down, "x": x, "bias": bias}


def logits(d):
    """Router logits bf16 [rows, E] as uint16 bits: bf16(x W_r^T + bias), the product and sum in float64."""
    z = d["x"].double() @ d["router"].double().T
    if d["bias"] is not None:
        z = z + d["bias"]
    return moe.f32_to_bf16(z.float().numpy())


def routing(n, d):
    """(ids [rows, k] int64, weights [rows, k] float32 bf16-valued): the decode rule for configs 1-3, the prompt
    rule for config 4."""
    bits = logits(d)
    if n == 4:
        ids, w = moe.route_prefill(bits, TOP_K)
    else:
        ids, w = moe.route(bits, TOP_K)
    return np.asarray(ids, np.int64), np.asarray(w, np.float32)


def pack(kind, d, threads=0):
    """(gate_up fields, down fields) of `kind`, host torch tensors flat over experts."""
    from drama3_b200 import pack as packer
    return (packer.pack_bank(kind, d["gate_up"], threads), packer.pack_bank(kind, d["down"], threads))


def bank_hash(banks):
    """sha256 hex digest of every field's bytes, gate_up then down, fields by name."""
    h = hashlib.sha256()
    for bank in banks:
        for name in sorted(bank):
            t = bank[name].contiguous()
            h.update(name.encode())
            h.update(t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.uint8 else t.numpy().tobytes())
    return h.hexdigest()


def codebooks(kind):
    """The w4 packer's codebook per bank (both banks use the default one), else (None, None)."""
    if kind != "w4":
        return (None, None)
    from drama3_b200 import pack as packer
    cb = torch.tensor(packer.CODEBOOK4, dtype=torch.float32)
    return (cb, cb.clone())


def prompt_sample(rows=2048, count=32):
    """The prompt rows the config-4 fixture keeps the oracle's output of: every (rows // count)-th row."""
    return np.arange(0, rows, rows // count)[:count]
