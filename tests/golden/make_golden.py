"""Generate tests/golden/golden.npz from the reference's own Python CPU functions.

    python tests/golden/make_golden.py [/path/to/ComfyUI-Drama3]   (default: as oracle/build_ref.py finds it)

Runs only where the reference checkout exists (it is read, never copied). drama3/offload.py imports ComfyUI
modules that are not installed; a minimal stand-in provides the three names it touches at import time and the one
it calls on the CPU path: comfy.ops._swiglu_eager, restated as SiLU(first half) * second half (the gate rows come
first in every fused bank, tools/convert.py:195). Every array is seeded; the file is small and committed.

Cases:
  rotation     offload.hadamard(256) applied as the reference applies it ((x.view(-1, 256) @ H).flatten),
               drama3/offload.py:170-176, 185, 491
  dequant      offload.dequantize_fp8 on seeded e4m3 bytes and block scales, drama3/offload.py:163-167
  fp8_decode   offload.FP8Experts CPU forward for one row (experts_decode), fp32, drama3/offload.py:775-784
  fp8_prefill  offload.FP8Experts CPU forward for 24 rows (the per-expert loop), fp32, drama3/offload.py:785-802
  int8_cpu     offload.experts_on_cpu with QuantHostBank.cpu_linear (int8 ConvRot on the CPU),
               drama3/offload.py:179-189, 245-249
  prefill_route  the prompt-routing expression of drama3/model.py:120-121, run through torch
  slotpool     offload.SlotPool host methods (use / free_slots / assign / claim / room) on a fixed call sequence,
               drama3/offload.py:689-722
  config1      BASELINE config 1 (tests/config_data.py: seed 0, int8 ConvRot, one decode row) through the
               reference's CPU int8 decode: the row rotated (hadamard) and rounded to bf16, experts_on_cpu over its
               8 routed experts, the routing-weighted sum, bf16 (drama3/offload.py:170-189, 403-450)
"""
import sys
import types
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent / "golden.npz"


def import_reference(root):
    comfy = types.ModuleType("comfy")
    ops = types.ModuleType("comfy.ops")

    def _swiglu_eager(h):
        gate, up = h.chunk(2, dim=-1)
        return torch.nn.functional.silu(gate) * up

    ops._swiglu_eager = _swiglu_eager
    mm = types.ModuleType("comfy.model_management")
    qo = types.ModuleType("comfy.quant_ops")

    class QuantizedTensor:  # never constructed on these paths
        pass

    qo.QuantizedTensor = QuantizedTensor
    comfy.ops, comfy.model_management, comfy.quant_ops = ops, mm, qo
    for name, module in (("comfy", comfy), ("comfy.ops", ops), ("comfy.model_management", mm),
                         ("comfy.quant_ops", qo)):
        sys.modules[name] = module
    sys.path.insert(0, str(root))
    from drama3 import offload  # noqa: E402
    return offload


def e4m3_bytes(gen, shape):
    """Seeded e4m3 bytes without the two NaN codes."""
    b = torch.randint(0, 254, shape, generator=gen, dtype=torch.int32)
    b = torch.where(b >= 0x7F, b + 1, b)  # skip 0x7F
    return b.to(torch.uint8)


def main(root):
    offload = import_reference(root)
    gen = torch.Generator().manual_seed(1234)
    g = {}

    # rotation
    x = torch.randn((3, 768), generator=gen)
    g["rot_in"] = x.numpy()
    g["rot_out"] = (x.view(3, -1, 256) @ offload.hadamard(256)).flatten(1).numpy()

    # fp8 block dequantization
    w = e4m3_bytes(gen, (256, 384))
    s = torch.rand((2, 3), generator=gen) * 0.01 + 1e-4
    g["dq_w"], g["dq_s"] = w.numpy(), s.numpy()
    g["dq_out"] = offload.dequantize_fp8(w.view(torch.float8_e4m3fn), s, torch.float32).numpy()

    # FP8Experts CPU forward, fp32 (E=8, hidden 256, intermediate 128)
    E, H, I, k = 8, 256, 128, 4
    experts = offload.FP8Experts(E, H, I, device="cpu", dtype=torch.float32)
    with torch.no_grad():
        experts.gate_up_weight.copy_(e4m3_bytes(gen, (E, 2 * I, H)).view(torch.float8_e4m3fn))
        experts.down_weight.copy_(e4m3_bytes(gen, (E, H, I)).view(torch.float8_e4m3fn))
        experts.gate_up_scale.copy_(torch.rand((E, 2 * I // 128, H // 128), generator=gen) * 1e-3)
        experts.down_scale.copy_(torch.rand((E, H // 128, I // 128), generator=gen) * 1e-3)
    g["fp8_gu_w"] = experts.gate_up_weight.view(torch.uint8).numpy()
    g["fp8_gu_s"] = experts.gate_up_scale.numpy()
    g["fp8_dn_w"] = experts.down_weight.view(torch.uint8).numpy()
    g["fp8_dn_s"] = experts.down_scale.numpy()
    x1 = torch.randn((1, H), generator=gen).to(torch.bfloat16).float()
    ids = torch.tensor([[5, 0, 3, 6]])
    wts = torch.tensor([[0.4, 0.3, 0.2, 0.1]]).to(torch.bfloat16).float()
    with torch.no_grad():
        g["fp8_decode_out"] = experts(x1, ids, wts).numpy()
    g["fp8_decode_x"], g["fp8_decode_ids"], g["fp8_decode_w"] = x1.numpy(), ids.numpy(), wts.numpy()
    T = 24
    xt = torch.randn((T, H), generator=gen).to(torch.bfloat16).float()
    idx = torch.stack([torch.randperm(E, generator=gen)[:k] for _ in range(T)])
    wt = torch.softmax(torch.randn((T, k), generator=gen), dim=-1).to(torch.bfloat16).float()
    with torch.no_grad():
        g["fp8_prefill_out"] = experts(xt, idx, wt).numpy()
    g["fp8_prefill_x"], g["fp8_prefill_ids"], g["fp8_prefill_w"] = xt.numpy(), idx.numpy(), wt.numpy()

    # experts_on_cpu: int8 ConvRot experts through QuantHostBank.cpu_linear (E=4, hidden 256, intermediate 256)
    E2, H2, I2 = 4, 256, 256

    class Bank:
        cpu_linear = offload.QuantHostBank.cpu_linear

        def __init__(self, rows, cols):
            self.num_experts = E2
            self.fields = {"_qdata": torch.randint(-127, 128, (E2 * rows, cols), generator=gen, dtype=torch.int8),
                           "scale": torch.rand((E2 * rows, 1), generator=gen) * 1e-3 + 1e-4}
            self.scale_bf16 = self.fields["scale"].view(-1).to(torch.bfloat16)

        def rows(self, name):
            return self.fields[name].shape[0] // self.num_experts

    gate_up, down = Bank(2 * I2, H2), Bank(H2, I2)
    rot = offload.hadamard(256)
    xr = (torch.randn((3, H2), generator=gen).view(3, -1, 256) @ rot).flatten(1).to(torch.bfloat16)
    ex = [2, 0, 3]
    with torch.no_grad():
        g["int8_cpu_out"] = offload.experts_on_cpu((gate_up, down), ex, [1, 1, 1], xr, rot).numpy()
    g["int8_gu_q"], g["int8_gu_s"] = gate_up.fields["_qdata"].numpy(), gate_up.fields["scale"].numpy()
    g["int8_dn_q"], g["int8_dn_s"] = down.fields["_qdata"].numpy(), down.fields["scale"].numpy()
    g["int8_cpu_x"] = xr.float().numpy()
    g["int8_cpu_ids"] = np.array(ex)

    # prompt routing (drama3/model.py:120-121), 32 rows of 128 bf16 logits
    logits = (torch.randn((32, 128), generator=gen) * 0.9).to(torch.bfloat16)
    tw, ti = torch.softmax(logits.float(), dim=-1).topk(8, dim=-1)
    tw = (tw / tw.sum(dim=-1, keepdim=True)).to(torch.bfloat16)
    g["route_logits"] = logits.view(torch.int16).numpy().view(np.uint16)
    g["route_ids"], g["route_w"] = ti.numpy(), tw.float().numpy()

    # SlotPool host methods: 3 layers x 16 experts, 10 slots, one fp8-like bank of 128-row experts
    class HostBankStub:
        def __init__(self):
            self.num_experts = 16
            self.fields = {"weight": torch.zeros((16 * 128, 16), dtype=torch.uint8),
                           "scale": torch.zeros((16, 1), dtype=torch.float32)}

        def rows(self, name):
            return self.fields[name].shape[0] // self.num_experts

    banks = [(HostBankStub(), HostBankStub()) for _ in range(3)]
    expert_bytes = sum(t[:b.rows(n)].nbytes for b in banks[0] for n, t in b.fields.items())
    pool = offload.SlotPool(banks, 10 * expert_bytes, "cpu")
    trace, sgen = [], torch.Generator().manual_seed(99)
    for step in range(12):
        for layer in range(3):
            used = sorted(torch.randperm(16, generator=sgen)[:5].tolist())
            cached = pool.use(layer, used)
            for expert in used:
                if expert not in cached:
                    free = pool.free_slots()
                    slot = pool.assign(free[0], layer, expert) if free else pool.claim(layer, expert)
                    trace.append((step, layer, expert, slot, pool.room(layer)))
    g["slot_trace"] = np.array(trace, np.int64)
    g["slot_table"], g["slot_owner"] = pool.table.numpy(), pool.owner.numpy()
    g["slot_score"], g["slot_at"] = pool.score.numpy(), pool.at.numpy()
    g["slot_clock"] = pool.clock.numpy()

    # BASELINE config 1 through the reference's CPU int8 decode
    import config_data as cd
    d = cd.draw(1)
    ids, wts = cd.routing(1, d)
    packed = cd.pack("int8", d)

    class ConfigBank:
        cpu_linear = offload.QuantHostBank.cpu_linear

        def __init__(self, fields):
            self.num_experts = cd.E
            self.fields = {"_qdata": fields["_qdata"], "scale": fields["scale"].view(-1, 1)}
            self.scale_bf16 = fields["scale"].view(-1).to(torch.bfloat16)

        def rows(self, name):
            return self.fields[name].shape[0] // self.num_experts

    rot = offload.hadamard(256)
    row = (d["x"].float().view(1, -1, 256) @ rot).flatten(1).to(torch.bfloat16)
    k = ids.shape[1]
    with torch.no_grad():
        parts = offload.experts_on_cpu((ConfigBank(packed[0]), ConfigBank(packed[1])), ids[0].tolist(), [1] * k,
                                       row.expand(k, -1), rot)
        g["c1_ref_cpu_out"] = (torch.from_numpy(wts[0]) @ parts).to(torch.bfloat16).float().numpy().reshape(1, -1)

    np.savez_compressed(OUT, **g)
    print(f"{OUT}: {OUT.stat().st_size} bytes, {len(g)} arrays")


if __name__ == "__main__":
    for path in ("", "comfyui-drama3_b200", "tests"):
        sys.path.insert(0, str(Path(__file__).resolve().parents[2] / path))
    from oracle.build_ref import reference_root
    root = Path(sys.argv[1]) if len(sys.argv) > 1 else reference_root()
    if root is None:
        sys.exit("name the reference checkout: an argument, DRAMA3_REFERENCE, or BASELINE.json's reference_path")
    main(root)
