"""Host-side logic of the drop-in expert modules, on the CPU: the slot pool's bookkeeping against the reference's own
SlotPool run on a fixed call sequence (golden.npz), bank-layout recognition, host banks, and the prompt routing
expression of the MoE block."""
import dataclasses

import numpy as np
import pytest
import torch

from drama3_b200 import offload
from drama3_b200.model import SparseMoeBlock, block_config


class HostBankStub:
    """An fp8-like bank of 16 experts with 128 rows each: the stand-in bank the golden slot trace was made with."""

    def __init__(self):
        self.num_experts = 16
        self.fields = {"weight": torch.zeros((16 * 128, 16), dtype=torch.uint8),
                       "scale": torch.zeros((16, 1), dtype=torch.float32)}

    def rows(self, name):
        return self.fields[name].shape[0] // self.num_experts


def test_slot_pool_matches_reference_trace(golden):
    """use / free_slots / assign / claim / room over 12 passes x 3 layers reproduce the reference's slots, room counts
    and final state bit for bit (drama3/offload.py:689-722)."""
    banks = [(HostBankStub(), HostBankStub()) for _ in range(3)]
    expert_bytes = sum(t[:b.rows(n)].nbytes for b in banks[0] for n, t in b.fields.items())
    pool = offload.SlotPool(banks, 10 * expert_bytes, "cpu")
    assert pool.count == 10 and pool.expert_bytes == expert_bytes
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
    np.testing.assert_array_equal(np.array(trace, np.int64), golden["slot_trace"])
    np.testing.assert_array_equal(pool.table.numpy(), golden["slot_table"])
    np.testing.assert_array_equal(pool.owner.numpy(), golden["slot_owner"])
    np.testing.assert_array_equal(pool.score.numpy().view(np.uint32), golden["slot_score"].view(np.uint32))
    np.testing.assert_array_equal(pool.at.numpy(), golden["slot_at"])
    np.testing.assert_array_equal(pool.clock.numpy(), golden["slot_clock"])


def test_slot_pool_count_bounds():
    """count = max(8, min(layers * experts, budget // expert_bytes)) (drama3/offload.py:575)."""
    banks = [(HostBankStub(), HostBankStub()) for _ in range(2)]
    per = offload.SlotPool(banks, 0, "cpu").expert_bytes
    assert offload.SlotPool(banks, 0, "cpu").count == 8
    assert offload.SlotPool(banks, 13 * per + per // 2, "cpu").count == 13
    assert offload.SlotPool(banks, 10 ** 12, "cpu").count == 32


def test_slot_pool_assign_and_claim_rules():
    """assign evicts the old owner from the table; claim takes free slots first, never a slot this layer used in this
    pass, and the least used of the rest (ties: the lower slot)."""
    banks = [(HostBankStub(), HostBankStub()) for _ in range(2)]
    pool = offload.SlotPool(banks, 0, "cpu")
    assert pool.use(0, [1, 2, 3]) == {}
    for slot, expert in enumerate((1, 2, 3)):
        pool.assign(slot, 0, expert)
    assert pool.use(1, [4]) == {}
    assert pool.claim(1, 4) == 3  # the first free slot scores -1
    for slot in range(4, 8):
        pool.assign(slot, 1, slot + 1)
    assert pool.free_slots() == []
    # next pass: layer 0 uses expert 2 (slot 1, excluded); slots 4-7 hold experts never counted as used (score 0),
    # below the decayed counts of slots 0, 2 and 3: the lowest of them goes
    assert pool.use(0, [2]) == {2: 1}
    slot = pool.claim(0, 9)
    assert slot == 4 and int(pool.table[16 + 5]) == -1 and int(pool.table[9]) == 4 and int(pool.owner[4]) == 9
    assert pool.room(0) == 7


@dataclasses.dataclass
class Params:
    orig_shape: tuple
    scale: torch.Tensor = None
    s_channel: torch.Tensor = None
    codebook: torch.Tensor = None
    convrot: bool = True
    convrot_groupsize: int = 256
    group_size: int = 16
    correction: object = None
    transposed: bool = False


class FakeQuantized:
    """Duck-typed stand-in for comfy's QuantizedTensor: `_qdata`, `_params`, `_layout_cls`."""

    def __init__(self, layout, qdata, params):
        self._layout_cls, self._qdata, self._params = layout, qdata, params


def int8_weight(rows=64, K=256, **kw):
    return FakeQuantized("TensorWiseINT8Layout", torch.zeros((rows, K), dtype=torch.int8),
                         Params((rows, K), scale=torch.ones((rows, 1)), **kw))


def codes_weight(bits, rows=64, K=256, codebook=True, **kw):
    return FakeQuantized("AsymW4A8Int8Layout", torch.zeros((rows, K * bits // 8), dtype=torch.uint8),
                         Params((rows, K), scale=torch.zeros((rows, K // 16), dtype=torch.uint8),
                                s_channel=torch.ones((rows,)), codebook=torch.zeros(16) if codebook else None, **kw))


def test_kernel_bank_recognition():
    """The layouts the kernels read, and the near misses they do not (drama3/offload.py:73-90)."""
    kind, fields = offload.kernel_bank(int8_weight())
    assert kind == "int8" and set(fields) == {"_qdata", "scale"}
    assert offload.kernel_bank(int8_weight(convrot=False)) is None
    assert offload.kernel_bank(int8_weight(convrot_groupsize=128)) is None
    assert offload.kernel_bank(int8_weight(K=4096)) is None
    assert offload.kernel_bank(codes_weight(4))[0] == "w4"
    assert offload.kernel_bank(codes_weight(6, codebook=False))[0] == "w6"
    assert offload.kernel_bank(codes_weight(4, codebook=False)) is None
    assert offload.kernel_bank(codes_weight(6, codebook=True)) is None
    assert offload.kernel_bank(codes_weight(4, group_size=32)) is None
    assert offload.kernel_bank(codes_weight(4, transposed=True)) is None
    assert offload.kernel_bank(codes_weight(4, correction=torch.zeros(1))) is None
    assert offload.kernel_bank(torch.zeros((4, 4))) is None
    assert set(offload.per_row_fields(codes_weight(4))) == {"_qdata", "scale", "s_channel"}
    assert set(offload.tensor_fields(codes_weight(4))) == {"scale", "s_channel", "codebook"}


def test_host_banks_layout():
    """FP8HostBank flattens [E, N, K] experts to [E * N, K] rows and [E, N/128, K/128] scales to rows of blocks;
    take() slices whole experts (drama3/offload.py:200-273)."""
    w = torch.arange(4 * 256 * 128, dtype=torch.int32).remainder(120).to(torch.uint8).view(4, 256, 128)
    s = torch.rand((4, 2, 1))
    bank = offload.FP8HostBank(w.view(torch.float8_e4m3fn), s, pin=False)
    assert bank.num_experts == 4 and bank.rows("weight") == 256 and bank.rows("scale") == 2
    part = bank.take(bank.fields, 1, 3)
    assert torch.equal(part["weight"], w[1:3].reshape(512, 128))
    assert torch.equal(part["scale"], s[1:3].reshape(4, 1))
    module = type("M", (), {"weight": codes_weight(4, rows=4 * 64), "num_experts": 4})()
    qbank = offload.QuantHostBank(module, pin=False)
    assert qbank.kernel == "w4" and qbank.rows("_qdata") == 64 and qbank.rows("s_channel") == 64
    with pytest.raises(ValueError):
        offload.QuantHostBank(type("M", (), {"weight": int8_weight(convrot=False), "num_experts": 1})(), pin=False)


def test_prompt_routing_matches_reference(golden):
    """A prompt's rows route by the reference's softmax / top-k / renormalization expression (drama3/model.py:120-121)."""
    block = SparseMoeBlock(block_config(hidden=64, num_experts=128, intermediate=128, shared_intermediate=64),
                           device="meta", dtype=torch.bfloat16)
    logits = torch.from_numpy(golden["route_logits"].view(np.int16)).view(torch.bfloat16)
    ids, weights = block.route(logits, decode=False)
    np.testing.assert_array_equal(ids.numpy(), golden["route_ids"])
    np.testing.assert_array_equal(weights.float().numpy(), golden["route_w"])


def test_prompt_pass_sorts_on_the_device_under_graph_capture(monkeypatch):
    """A prompt pass reached while a CUDA graph is being captured asks resident_prefill for the device-side sort (the
    host-side one reads counts back, which a capture forbids); outside a capture it keeps the host-side plan."""
    from drama3_b200 import offload
    calls = []
    monkeypatch.setattr(offload.kernels, "available", lambda device: True)
    monkeypatch.setattr(offload, "resident_prefill", lambda *args, **kw: calls.append(kw.get("sync_free")))
    ex = offload.FP8Experts(4, 256, 128, dtype=torch.float32)
    x = torch.zeros((40, 256))
    ids = torch.zeros((40, 8), dtype=torch.int64)
    w = torch.full((40, 8), 0.125)
    assert offload.capturing(x) is False
    ex(x, ids, w)
    monkeypatch.setattr(offload, "capturing", lambda t: True)
    ex(x, ids, w)
    assert calls == [False, True]


def test_modules_take_the_reference_argument_lists():
    """Experts(num_experts, hidden, intermediate, device, dtype, ops) and SparseMoeBlock(config, device, dtype, ops)
    build as drama3/model.py:62,95 builds them: with a ComfyUI-like `ops` namespace its factories are used, without one
    the library's own (torch Linear, MoEBank)."""
    from types import SimpleNamespace
    from drama3_b200.model import Experts, MoEBank, SharedExpert

    made = []

    class Linear(torch.nn.Linear):
        def __init__(self, *a, **kw):
            made.append(("Linear", a))
            super().__init__(*a, **kw)

    class MoEExperts(MoEBank):
        def __init__(self, *a, **kw):
            made.append(("MoEExperts", a))
            super().__init__(*a, **kw)

    ops = SimpleNamespace(Linear=Linear, MoEExperts=MoEExperts)
    ex = Experts(16, 256, 128, "meta", torch.bfloat16, ops)
    assert ex.num_experts == 16 and isinstance(ex.gate_up_proj, MoEExperts)
    assert made[:2] == [("MoEExperts", (16, 256, 256)), ("MoEExperts", (16, 128, 256))]
    block = SparseMoeBlock(block_config(hidden=256, num_experts=16, intermediate=128, shared_intermediate=64,
                                        fp8=False), "meta", torch.bfloat16, ops)
    assert isinstance(block.experts, Experts) and isinstance(block.gate, Linear)
    assert isinstance(block.shared_expert, SharedExpert) and block.gate.weight.shape == (16, 256)
    fp8 = SparseMoeBlock(block_config(hidden=256, num_experts=16, intermediate=128, shared_intermediate=64),
                         "meta", torch.bfloat16)
    assert isinstance(fp8.experts, offload.FP8Experts) and fp8.experts.kind == "fp8"
    assert fp8.experts.gate_up_scale.shape == (16, 2, 2)
    chan = SparseMoeBlock(block_config(hidden=256, num_experts=16, intermediate=128, shared_intermediate=64,
                                       per_channel=True), "meta", torch.bfloat16)
    assert chan.experts.kind == "fp8c" and chan.experts.gate_up_scale.shape == (16, 256)
    with pytest.raises(ValueError):
        MoEBank(4, 8, 8, bias=True)


@pytest.mark.parametrize("kind", ["w4a8", "w6a8"])
def test_baseline_banks_dressed_as_quantized_tensors(kind):
    """pack.packed_weight of the BASELINE int8-activation layouts is recognized by kernel_bank, with the packer's
    fields."""
    from drama3_b200 import pack
    w = torch.randn((2, 128, 256), generator=torch.Generator().manual_seed(3)) * 0.02
    packed = pack.packed_weight(kind, w)
    found, fields = offload.kernel_bank(packed)
    direct = pack.pack_bank(kind, w)
    assert found == kind and set(fields) == {"_qdata", "scale"}
    assert torch.equal(fields["_qdata"], direct["_qdata"]) and torch.equal(fields["scale"], direct["scale"])
