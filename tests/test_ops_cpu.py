"""The torch.library custom ops (drama3_b200.ops) on the CPU: every op is registered under torch.ops.drama3_b200
with the schema its kernels function needs; each fake implementation gives the kernel's output shapes and dtypes on
meta tensors (what graph builders trace with); and each op hands its arguments, with the banks rebuilt field by field
in the reference's names, to the kernels function it wraps (checked with that function replaced by a recorder)."""
import pytest
import torch

from drama3_b200 import kernels, ops

M = "meta"


def test_every_op_is_registered():
    for name in ops.OPS:
        packet = getattr(torch.ops.drama3_b200, name)
        assert packet.default._schema.name == f"drama3_b200::{name}"
    schema = str(torch.ops.drama3_b200.moe_decode.default._schema)
    assert "str kind" in schema and "Tensor? c13" in schema and "-> Tensor" in schema
    assert "Tensor(a4!) out" in str(torch.ops.drama3_b200.shared_expert.default._schema)


def test_fake_shapes_on_meta_tensors():
    o = torch.ops.drama3_b200
    ids, w = o.route(torch.empty((5, 128), dtype=torch.bfloat16, device=M), 8)
    assert ids.shape == (5, 8) and ids.dtype == torch.int64 and w.dtype == torch.float32
    out = o.weighted_sum(torch.empty((40, 2048), device=M), torch.empty((5, 8), device=M))
    assert out.shape == (5, 2048) and out.dtype == torch.bfloat16
    only = torch.empty(1, dtype=torch.int32, device=M)
    assert o.rotate(torch.empty((3, 3072), device=M), only, True).shape == (3, 1536)
    ids, w = o.router(torch.empty((16, 2048), dtype=torch.bfloat16, device=M),
                      torch.empty((128, 2048), dtype=torch.bfloat16, device=M), 8)
    assert ids.shape == (16, 8) and w.shape == (16, 8)
    x = torch.empty((4, 2048), dtype=torch.bfloat16, device=M)
    u8 = dict(dtype=torch.uint8, device=M)
    y = o.moe_decode("fp8c", x, torch.empty((4, 8), dtype=torch.int64, device=M), torch.empty((4, 8), device=M),
                     torch.empty((128 * 1536, 2048), **u8), torch.empty(128 * 1536, device=M), None,
                     torch.empty((128 * 2048, 768), **u8), torch.empty(128 * 2048, device=M), None)
    assert y.shape == (4, 2048) and y.dtype == torch.bfloat16
    order, pos, groups = o.prefill_plan(torch.empty((2048, 8), dtype=torch.int64, device=M), 128)
    assert order.shape == (16384,) and pos.dtype == torch.int64 and groups.shape == (129, 5)
    g = o.grouped_mma("w6a8", x, groups, torch.empty((128 * 1536, 1536), **u8),
                      torch.empty((128 * 1536, 16), dtype=torch.bfloat16, device=M), None, None, 1536, 226,
                      torch.empty(16384, dtype=torch.int64, device=M))
    assert g.shape == (16384, 1536) and g.dtype == torch.float32
    c = o.prefill_combine(torch.empty((16384, 2048), device=M), torch.empty((2048, 8), dtype=torch.int64, device=M),
                          torch.empty((2048, 8), device=M), True)
    assert c.shape == (2048, 2048) and c.dtype == torch.float32


def test_ops_pass_their_arguments_through(monkeypatch):
    seen = {}

    def fake_decode(kind, x, ids, weights, banks, codebooks=(None, None), workspace=None, out=None):
        seen["decode"] = (kind, banks, codebooks)
        return torch.zeros(x.shape, dtype=torch.bfloat16)

    def fake_grouped(kind, x, groups, fields, codebook, n, tiles, row_index=None, rotate=False, swiglu=False):
        seen["grouped"] = (kind, fields, codebook, n, tiles, row_index, rotate, swiglu)
        return torch.zeros((x.shape[0], n))

    def fake_combine(sorted_out, pos, weights, dtype=torch.bfloat16):
        seen["combine"] = dtype
        return torch.zeros((pos.shape[0], sorted_out.shape[1]), dtype=dtype)

    monkeypatch.setattr(kernels, "moe_decode", fake_decode)
    monkeypatch.setattr(kernels, "grouped_mma", fake_grouped)
    monkeypatch.setattr(kernels, "prefill_combine", fake_combine)
    x = torch.zeros((2, 8), dtype=torch.bfloat16)
    w13, s13, c13, w2, s2, c2, cb = (torch.full((1,), float(i)) for i in range(7))
    torch.ops.drama3_b200.moe_decode("w4", x, torch.zeros((2, 1), dtype=torch.int64), torch.ones((2, 1)),
                                     w13, s13, c13, w2, s2, c2, cb, None)
    kind, (gu, dn), cbs = seen["decode"]
    assert kind == "w4" and set(gu) == {"_qdata", "scale", "s_channel"} and gu["s_channel"] is c13
    assert dn["_qdata"] is w2 and cbs[0] is cb and cbs[1] is None
    torch.ops.drama3_b200.moe_decode("fp8", x, torch.zeros((2, 1), dtype=torch.int64), torch.ones((2, 1)),
                                     w13, s13, None, w2, s2, None)
    assert set(seen["decode"][1][0]) == {"weight", "scale"}
    out = torch.ops.drama3_b200.grouped_mma("w6a8", torch.zeros((3, 8)), torch.zeros((1, 5), dtype=torch.int32),
                                            w13, s13, None, None, 16, 4, None, False, True)
    assert out.shape == (3, 16)
    kind, fields, codebook, n, tiles, row_index, rot, swi = seen["grouped"]
    assert kind == "w6a8" and set(fields) == {"_qdata", "scale"}
    assert (n, tiles, row_index, rot, swi) == (16, 4, None, False, True)
    assert torch.ops.drama3_b200.prefill_combine(torch.zeros((4, 8)), torch.zeros((2, 2), dtype=torch.int64),
                                                 torch.ones((2, 2)), True).dtype == torch.float32
    assert seen["combine"] == torch.float32


def test_ops_have_no_fallback_off_the_gpu():
    """On CPU tensors an op is refused before the library is called (no CPU or torch path exists)."""
    with pytest.raises(ValueError, match="cuda device"):
        torch.ops.drama3_b200.route(torch.zeros((2, 128), dtype=torch.bfloat16), 8)


def test_ops_trace_into_an_exported_program():
    """torch.export traces a module that calls the ops through their fake implementations (nothing runs), and the
    exported graph holds the ops themselves."""

    class Block(torch.nn.Module):
        def forward(self, logits, parts):
            ids, w = torch.ops.drama3_b200.route(logits, 8)
            return ids, torch.ops.drama3_b200.weighted_sum(parts, w)

    ep = torch.export.export(Block(), (torch.zeros((4, 128), dtype=torch.bfloat16), torch.zeros((32, 2048))))
    targets = {str(n.target) for n in ep.graph.nodes if n.op == "call_function"}
    assert {"drama3_b200.route.default", "drama3_b200.weighted_sum.default"} <= targets
    out = [n for n in ep.graph.nodes if n.op == "output"][0].args[0]
    assert tuple(out[1].meta["val"].shape) == (4, 2048) and out[1].meta["val"].dtype == torch.bfloat16
