"""The drop-in expert modules on the GPU: FP8Experts against the reference's own CPU forward (golden.npz), the fused
lines decode against the oracle and the per-kernel sequence, the slot-cache ExpertStore against the same experts held
whole (bit for bit: the same kernels read a slot, or host memory, and fill), and the MoE block's batched decode."""
import numpy as np
import pytest
import torch

import gpu_data as gd
from drama3_b200 import kernels, offload
from drama3_b200.model import Experts, SparseMoeBlock, block_config
from oracle import moe
from test_offload_host import FakeQuantized, Params

pytestmark = pytest.mark.gpu
E, H, I = 16, 2048, 768


def fp8_module(E_, H_, I_, seed, device):
    ex = offload.FP8Experts(E_, H_, I_, device=device, dtype=torch.bfloat16)
    gu, dn = gd.rand_bank("fp8", E_, 2 * I_, H_, seed, device), gd.rand_bank("fp8", E_, H_, I_, seed + 1, device)
    with torch.no_grad():
        ex.gate_up_weight.copy_(gu["weight"].view(E_, 2 * I_, H_).view(torch.float8_e4m3fn))
        ex.gate_up_scale.copy_(gu["scale"].view(E_, 2 * I_ // 128, H_ // 128))
        ex.down_weight.copy_(dn["weight"].view(E_, H_, I_).view(torch.float8_e4m3fn))
        ex.down_scale.copy_(dn["scale"].view(E_, H_ // 128, I_ // 128))
    return ex, (gu, dn)


def quant_module(kind, E_, N, K, seed, device):
    """A module whose .weight is a duck-typed quantized bank the kernels read."""
    bank = gd.rand_bank(kind, E_, N, K, seed, device)
    if kind == "int8":
        w = FakeQuantized("TensorWiseINT8Layout", bank["_qdata"], Params((E_ * N, K), scale=bank["scale"]))
    else:
        cb = gd.codebooks(kind, device)[0]
        w = FakeQuantized("AsymW4A8Int8Layout", bank["_qdata"],
                          Params((E_ * N, K), scale=bank["scale"], s_channel=bank["s_channel"], codebook=cb))
    return type("Bank", (), {"weight": w, "num_experts": E_})(), bank


def test_fp8_experts_match_reference_cpu_forward(golden, cuda):
    """FP8Experts (E 8, hidden 256, intermediate 128: the per-kernel sequence) against the reference's own fp32 CPU
    forward: one row (drama3/offload.py:782-784) and a 24-row prompt (:785-802)."""
    ex = offload.FP8Experts(8, 256, 128, device=cuda, dtype=torch.float32)
    with torch.no_grad():
        for name in ("gu", "dn"):
            full = "gate_up" if name == "gu" else "down"
            getattr(ex, f"{full}_weight").copy_(torch.from_numpy(golden[f"fp8_{name}_w"]).view(torch.float8_e4m3fn))
            getattr(ex, f"{full}_scale").copy_(torch.from_numpy(golden[f"fp8_{name}_s"]))
    x = torch.from_numpy(golden["fp8_decode_x"]).to(cuda)
    out = ex(x, torch.from_numpy(golden["fp8_decode_ids"]).to(cuda), torch.from_numpy(golden["fp8_decode_w"]).to(cuda))
    ref = torch.from_numpy(golden["fp8_decode_out"]).to(torch.bfloat16)
    assert out.dtype == torch.bfloat16 and gd.rel_l2(out.float(), ref.float()) <= 1e-3
    xt = torch.from_numpy(golden["fp8_prefill_x"]).to(cuda)
    out = ex(xt, torch.from_numpy(golden["fp8_prefill_ids"]).to(cuda),
             torch.from_numpy(golden["fp8_prefill_w"]).to(cuda))
    assert out.dtype == torch.float32 and gd.rel_l2(out, golden["fp8_prefill_out"]) <= 1e-5


@pytest.mark.parametrize("M", [1, 4, 16])
def test_fp8_experts_lines_fused(cuda, M):
    """M lines through FP8Experts at the benchmark's layer shape: one fused launch, against the oracle and against
    the per-kernel sequence row by row."""
    ex, banks = fp8_module(E, H, I, 30 + M, cuda)
    x = gd.rand_rows(M, H, 40 + M, cuda)
    ids, w = gd.rand_routing(M, E, 8, 50 + M, cuda)
    out = ex(x, ids, w)
    ref = gd.oracle_decode("fp8", x, ids, w, banks, (None, None), H)
    assert gd.rel_l2(out.float(), ref) <= 1e-3
    seq = torch.cat([offload._decode_sequence(x[r:r + 1], ids[r], w[r], banks, (2 * I, H), "fp8", (None, None))
                     for r in range(M)])
    assert gd.rel_l2(out.float(), seq.float()) <= 1e-3


@pytest.mark.parametrize("kind", ["int8", "w4", "w6"])
def test_quantized_experts_lines_and_prompt(cuda, kind):
    """Experts over quantized banks: 4 lines (fused) and a 40-row prompt (grouped kernels) against the oracle."""
    gu, gu_bank = quant_module(kind, E, 2 * I, H, 60, cuda)
    dn, dn_bank = quant_module(kind, E, H, I, 61, cuda)
    ex = Experts(E, H, I, device=cuda, dtype=torch.bfloat16)  # the reference's argument list
    ex.gate_up_proj.weight, ex.down_proj.weight = gu.weight, dn.weight
    cbs = gd.codebooks(kind, cuda)
    x = gd.rand_rows(4, H, 62, cuda)
    ids, w = gd.rand_routing(4, E, 8, 63, cuda)
    ref = gd.oracle_decode(kind, x, ids, w, (gu_bank, dn_bank), cbs, H)
    assert gd.rel_l2(ex(x, ids, w).float(), ref) <= 1e-3
    xt = gd.rand_rows(40, H, 64, cuda)
    idt, wt = gd.rand_routing(40, E, 8, 65, cuda)
    out = ex(xt, idt, wt)
    npb = (gd.to_np_bank(gu_bank), gd.to_np_bank(dn_bank))
    cbn = tuple(None if c is None else c.cpu().numpy() for c in cbs)
    ref = moe.resident_prefill(kind, xt.float().cpu().numpy(), idt.cpu().numpy(), wt.cpu().numpy(), npb, cbn)
    assert out.dtype == torch.bfloat16 and gd.rel_l2(out.float(), ref) <= 1e-3


def device_state_consistent(pool):
    pool.host()
    owner, table = pool.owner.numpy(), pool.table.numpy()
    for slot, key in enumerate(owner):
        if key >= 0:
            assert table[key] == slot
    for key, slot in enumerate(table):
        if slot >= 0:
            assert owner[slot] == key


@pytest.mark.parametrize("kind", ["fp8", "int8", "w4"])
def test_expert_store_matches_resident(cuda, kind):
    """Two layers of 16 experts in pinned host memory behind a 24-slot cache: 6 decode steps and a 40-row prompt pass,
    bit for bit against the same experts held whole on the GPU (hits read a slot, misses read host memory and fill a
    slot, all through the same kernels); every slot then holds its owner's bytes."""
    store = offload.ExpertStore(cache_bytes=0, pin=True)
    layers, device_banks = [], []
    for layer in range(2):
        if kind == "fp8":
            module, banks = fp8_module(E, H, I, 70 + 2 * layer, cuda)
            host = offload.FP8Experts(E, H, I, device="cpu", dtype=torch.bfloat16)
            with torch.no_grad():
                for name in ("gate_up_weight", "gate_up_scale", "down_weight", "down_scale"):
                    getattr(host, name).copy_(getattr(module, name).cpu())
            layers.append(store.add(host))
        else:
            gu, gu_bank = quant_module(kind, E, 2 * I, H, 70 + 2 * layer, "cpu")
            dn, dn_bank = quant_module(kind, E, H, I, 71 + 2 * layer, "cpu")
            banks = ({n: t.to(cuda) for n, t in gu_bank.items()}, {n: t.to(cuda) for n, t in dn_bank.items()})
            layers.append(store.add(type("X", (), {"gate_up_proj": gu, "down_proj": dn})()))
        device_banks.append(banks)
    store.cache_bytes = 24 * sum(t[:b.rows(n)].nbytes for b in store.banks[0] for n, t in b.fields.items())
    cbs = gd.codebooks(kind, cuda)
    with store.session(cuda):
        assert store.cache.count == 24 and all(m.sync_free(cuda) for m in layers)
        for step in range(6):
            x = gd.rand_rows(1, H, 80 + step, cuda)
            for layer, module in enumerate(layers):
                ids, w = gd.rand_routing(1, E, 8, 90 + 10 * step + layer, cuda)
                got = module(x, ids, w)
                want = offload._decode_sequence(x, ids[0], w[0], device_banks[layer], (2 * I, H), kind, cbs)
                assert torch.equal(got, want), (step, layer)
            store.between_steps()
        torch.cuda.synchronize()
        hits, fills, on_cpu = store.cache.reads.tolist()
        assert hits + fills == 6 * 2 * 8 and on_cpu == 0 and hits > 0
        xt = gd.rand_rows(40, H, 99, cuda)
        for layer, module in enumerate(layers):
            idt, wt = gd.rand_routing(40, E, 8, 120 + layer, cuda)
            got = module(xt, idt, wt)
            # the store's prompt pass rounds each pair's output to the rows' dtype before weighting
            # (drama3/offload.py:462-466, 512)
            order, counts = offload._sort_by_expert(idt, E)
            offsets = np.concatenate([[0], np.cumsum(counts)])
            groups = torch.tensor([(e, e, 0, offsets[e], n) for e, n in enumerate(counts) if n],
                                  dtype=torch.int32).to(cuda)
            always = torch.ones((1,), dtype=torch.int32, device=cuda)
            so = offload.grouped_experts(xt[order // 8], groups, device_banks[layer], device_banks[layer], (2 * I, H),
                                         kind, cbs, always).to(xt.dtype)
            weighted = so * wt.reshape(-1)[order].unsqueeze(1)
            want = torch.empty_like(weighted)
            want[order] = weighted
            assert torch.equal(got, want.view(40, 8, -1).sum(dim=1)), layer
        torch.cuda.synchronize()
        pool = store.cache
        device_state_consistent(pool)
        key_field = "weight" if kind == "fp8" else "_qdata"
        for slot, key in enumerate(pool.owner.tolist()):
            if key < 0:
                continue
            layer, expert = divmod(key, E)
            for index, bank in enumerate(store.banks[layer]):
                rows = bank.rows(key_field)
                got = pool.fields[index][key_field][slot * rows:(slot + 1) * rows].cpu()
                assert torch.equal(got, bank.fields[key_field][expert * rows:(expert + 1) * rows])


def test_moe_block_batched_lines(cuda):
    """[B, 1, H] decode rows of lines batched together: routed by one route launch and run as one fused decode,
    against the block run row by row."""
    torch.manual_seed(5)
    block = SparseMoeBlock(block_config(num_experts=E), device=cuda, dtype=torch.bfloat16)
    ex, _ = fp8_module(E, H, I, 140, cuda)
    block.experts = ex
    with torch.no_grad():
        for lin in (block.gate, block.shared_expert.gate_up_proj, block.shared_expert.down_proj,
                    block.shared_expert_gate):
            lin.weight.normal_(0, 0.02)
        x = gd.rand_rows(8, H, 141, cuda).view(8, 1, H)
        together = block(x)
        alone = torch.cat([block(x[r:r + 1]) for r in range(8)])
        logits = block.gate(x.view(8, H))
    ids, _ = kernels.route(logits, 8)
    for r in range(8):
        ids_r, _ = kernels.route(logits[r:r + 1], 8)
        assert torch.equal(ids[r], ids_r[0])
    assert together.shape == x.shape and gd.rel_l2(together.float(), alone.float()) <= 1e-3


@pytest.mark.parametrize("kind, bound", [("int8", 0.03), ("w6", 0.07), ("w4", 0.25)])
def test_packed_float_experts_through_the_module(cuda, kind, bound):
    """Float experts N(0, 0.02) packed on the host (pack.packed_weight), moved to the GPU and run by Experts for 4
    lines: against the oracle on the packed fields (rel-L2 1e-3) and against the float experts themselves (the
    packing's own error, layout by layout)."""
    from drama3_b200 import pack
    Ef = 8
    gen = torch.Generator().manual_seed(150)
    gu_f = torch.randn((Ef, 2 * I, H), generator=gen) * 0.02
    dn_f = torch.randn((Ef, H, I), generator=gen) * 0.02
    ex = Experts(Ef, H, I, device=cuda, dtype=torch.bfloat16)
    ex.gate_up_proj.weight = pack.packed_weight(kind, gu_f).to(cuda)
    ex.down_proj.weight = pack.packed_weight(kind, dn_f).to(cuda)
    mods = (ex.gate_up_proj, ex.down_proj)
    x = gd.rand_rows(4, H, 151, cuda)
    ids, w = gd.rand_routing(4, Ef, 8, 152, cuda)
    out = ex(x, ids, w).float()
    banks = tuple(offload.kernel_bank(m.weight)[1] for m in mods)
    cbs = tuple(m.weight._params.codebook for m in mods)
    assert gd.rel_l2(out, gd.oracle_decode(kind, x, ids, w, banks, cbs, H)) <= 1e-3
    xf, idc, wc = x.double().cpu(), ids.cpu(), w.double().cpu()
    ref = torch.zeros((4, H), dtype=torch.float64)
    for t in range(4):
        for j in range(8):
            e = int(idc[t, j])
            h = gu_f[e].double() @ xf[t]
            ref[t] += wc[t, j] * (dn_f[e].double() @ (torch.nn.functional.silu(h[:I]) * h[I:]))
    assert gd.rel_l2(out, ref) <= bound
