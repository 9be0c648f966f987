"""Write tests/golden/configs.npz: the oracle's outputs on the BASELINE configurations' seeded inputs
(tests/config_data.py), for every layout each config names, with a sha256 of every packed bank.

    python tests/golden/make_configs.py

Test infrastructure. Contents, per config n and layout kind:
  c{n}_{kind}_hash      sha256 of the packed (gate_up, down) banks, as 32 bytes
  c{n}_logits           router logits of the decode rows (configs 1-3), bf16 bits [rows, E]
  c{n}_ids, c{n}_w      the routing: ids int16 [rows, k], weights float32 (bf16 values)
  c{n}_{kind}_M{m}      configs 1-3: the oracle's decode of the first m rows, bf16-valued float32 [m, H]
  c4_sample             config 4: the prompt rows kept; c4_{kind}_out the oracle's prompt pass of those rows [32, H]
  c4_counts             config 4: the realized pairs per expert of the whole 2048-row prompt
The oracle's prompt pass computes every row on its own, so a sample of rows gives exactly those rows' outputs.
"""
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
for p in (ROOT, ROOT / "comfyui-drama3_b200", ROOT / "tests"):
    sys.path.insert(0, str(p))

import config_data as cd  # noqa: E402
import gpu_data as gd  # noqa: E402
from oracle import moe  # noqa: E402

OUT = Path(__file__).resolve().parent / "configs.npz"


def main():
    g = {}
    for n, c in cd.CONFIGS.items():
        started = time.time()
        d = cd.draw(n)
        ids, w = cd.routing(n, d)
        g[f"c{n}_ids"], g[f"c{n}_w"] = ids.astype(np.int16), w
        x = d["x"].float().numpy()
        if n != 4:
            g[f"c{n}_logits"] = cd.logits(d)
        else:
            g["c4_counts"] = np.bincount(ids.reshape(-1), minlength=cd.E).astype(np.int32)
            g["c4_sample"] = cd.prompt_sample(c["rows"])
        for kind in c["kinds"]:
            banks = cd.pack(kind, d)
            g[f"c{n}_{kind}_hash"] = np.frombuffer(bytes.fromhex(cd.bank_hash(banks)), np.uint8)
            npb = tuple(gd.to_np_bank(b) for b in banks)
            cbs = tuple(None if t is None else t.numpy() for t in cd.codebooks(kind))
            baseline = kind in ("fp8c", "w4a8", "w6a8")
            if n == 4:
                s = g["c4_sample"]
                if baseline:
                    out = moe.baseline_prefill(kind, x[s], ids[s], w[s], npb)
                else:
                    out = moe.resident_prefill(kind, x[s], ids[s], w[s], npb, cbs)
                g[f"c4_{kind}_out"] = np.asarray(out, np.float32)
            else:
                for m in c["lines"]:
                    if baseline:
                        out = moe.baseline_decode(kind, x[:m], ids[:m], w[:m], npb)
                    else:
                        out = moe.moe_decode(kind, x[:m], ids[:m], w[:m], npb, cbs)
                    g[f"c{n}_{kind}_M{m}"] = np.asarray(out, np.float32)
            print(f"config {n} {kind}: {time.time() - started:.0f} s", flush=True)
    np.savez_compressed(OUT, **g)
    print(f"{OUT}: {OUT.stat().st_size} bytes, {len(g)} arrays")


if __name__ == "__main__":
    main()
