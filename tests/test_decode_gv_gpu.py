"""The one-line streaming decode of per-channel e4m3 experts (moe_decode_gv_kernel: phase-1 rows streamed through a
ring, every pair's down rows prefetched into shared memory, one grid barrier, each CTA's output rows combined over
the pairs in rank order) against the oracle and against the tensor-core decode of the same call (D3_DECODE_GV=0
selects it): both expert widths, bf16 and fp32 rows, fewer than 8 pairs, a repeated expert, an out-of-range id, a row
of wide dynamic range, a zero row, and repeated calls on one workspace."""
import pytest
import torch

import gpu_data as gd
from drama3_b200 import _lib, kernels

pytestmark = pytest.mark.gpu
H, E = 2048, 32


def banks_for(I, seed, device):
    return (gd.rand_bank("fp8c", E, 2 * I, H, seed, device), gd.rand_bank("fp8c", E, H, I, seed + 1, device))


def close_to_oracle(got, ref):
    """Within rel-L2 1e-4 of the oracle, or else only bf16 rounding flips apart: every element within one bf16 step of
    the oracle's (plus 2^-20 of the row's rms, for elements that are small by cancellation) and fewer than 0.5 %
    differing. The fp32 sums differ from the oracle's float64 ones by ~1e-7, which flips the bf16 rounding of the odd
    element sitting on a rounding boundary."""
    got = got.float().cpu()
    ref = torch.as_tensor(ref).float()
    if gd.rel_l2(got, ref) <= 1e-4:
        return True
    step = ref.abs() * 2.0 ** -7 + ref.pow(2).mean().sqrt() * 2.0 ** -20
    return bool(((got - ref).abs() <= step * 1.0001).all()) and float((got != ref).float().mean()) < 0.005


def both(monkeypatch, x, ids, w, banks, **kw):
    """(streaming decode, tensor-core decode) of the same call."""
    monkeypatch.delenv("D3_DECODE_GV", raising=False)
    gv = kernels.moe_decode("fp8c", x, ids, w, banks, **kw)
    monkeypatch.setenv("D3_DECODE_GV", "0")
    tc = kernels.moe_decode("fp8c", x, ids, w, banks, **kw)
    monkeypatch.delenv("D3_DECODE_GV")
    return gv, tc


@pytest.mark.parametrize("I", [768, 512])
@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("k", [8, 6, 1])
def test_gv_decode_matches_oracle(cuda, monkeypatch, I, bf16, k):
    banks = banks_for(I, 40 + k, cuda)
    x = gd.rand_rows(1, H, 50 + k, cuda)
    if not bf16:
        x = torch.randn((1, H), generator=torch.Generator().manual_seed(60 + k)).to(cuda)
    ids, w = gd.rand_routing(1, E, k, 70 + k, cuda)
    _lib.take_fault()
    gv, tc = both(monkeypatch, x, ids, w, banks)
    assert _lib.take_fault() == 0
    ref = gd.baseline_oracle_decode("fp8c", x, ids, w, banks)
    assert close_to_oracle(gv, ref)
    assert gd.rel_l2(gv.float(), tc.float()) <= 1e-3


def test_gv_decode_wide_range_row_and_repeated_expert(cuda, monkeypatch):
    """One element 1000x the rest (the f16 terms keep the small ones), and an expert routed twice."""
    I = 768
    banks = banks_for(I, 80, cuda)
    x = torch.randn((1, H), generator=torch.Generator().manual_seed(81))
    x[0, 77] = 1000.0
    x = x.to(torch.bfloat16).to(cuda)
    ids = torch.tensor([[3, 9, 3, 20, 1, 0, 31, 17]], device=cuda)
    w = torch.full((1, 8), 0.125, device=cuda)
    _lib.take_fault()
    gv, _ = both(monkeypatch, x, ids, w, banks)
    assert _lib.take_fault() == 0
    assert close_to_oracle(gv, gd.baseline_oracle_decode("fp8c", x, ids, w, banks))


def test_gv_decode_bad_id_zero_row_and_repeats(cuda):
    """An out-of-range id: its pair is skipped (fault bit 2) and the rest equals the oracle without it; a zero row gives
    zeros; repeated calls sharing one workspace are bit-identical."""
    I = 768
    banks = banks_for(I, 90, cuda)
    x = gd.rand_rows(1, H, 91, cuda)
    ids, w = gd.rand_routing(1, E, 8, 92, cuda)
    bad = ids.clone()
    bad[0, 5] = E + 7
    _lib.take_fault()
    got = kernels.moe_decode("fp8c", x, bad, w, banks)
    torch.cuda.synchronize()
    assert _lib.take_fault() == 2
    w0 = w.clone()
    w0[0, 5] = 0.0
    ok_ids = bad.clone()
    ok_ids[0, 5] = 0
    assert close_to_oracle(got, gd.baseline_oracle_decode("fp8c", x, ok_ids, w0, banks))
    zero = kernels.moe_decode("fp8c", torch.zeros_like(x), ids, w, banks)
    assert not zero.float().abs().any()
    ws = kernels.decode_workspace(1, 8, I, cuda)
    first = kernels.moe_decode("fp8c", x, ids, w, banks, workspace=ws)
    for _ in range(5):
        assert torch.equal(kernels.moe_decode("fp8c", x, ids, w, banks, workspace=ws), first)
    assert _lib.take_fault() == 0


@pytest.mark.parametrize("I", [768, 512])
@pytest.mark.parametrize("bf16", [True, False])
def test_gv_decode_block_scaled_fp8(cuda, monkeypatch, I, bf16):
    """The reference's fp8 layout (128 x 128 block scales) through the streaming kernel: against the oracle of the
    reference's chain and against the mma.sync decode (D3_DECODE_GV=0) of the same call."""
    banks = (gd.rand_bank("fp8", E, 2 * I, H, 130, cuda), gd.rand_bank("fp8", E, H, I, 131, cuda))
    x = gd.rand_rows(1, H, 132, cuda)
    if not bf16:
        x = torch.randn((1, H), generator=torch.Generator().manual_seed(133)).to(cuda)
    ids, w = gd.rand_routing(1, E, 8, 134, cuda)
    _lib.take_fault()
    monkeypatch.delenv("D3_DECODE_GV", raising=False)
    gv = kernels.moe_decode("fp8", x, ids, w, banks)
    monkeypatch.setenv("D3_DECODE_GV", "0")
    old = kernels.moe_decode("fp8", x, ids, w, banks)
    monkeypatch.delenv("D3_DECODE_GV")
    torch.cuda.synchronize()
    assert _lib.take_fault() == 0
    assert close_to_oracle(gv, gd.oracle_decode("fp8", x, ids, w, banks, (None, None), H))
    assert gd.rel_l2(gv.float(), old.float()) <= 1e-3


@pytest.mark.parametrize("I", [768, 512])
@pytest.mark.parametrize("bf16", [True, False])
@pytest.mark.parametrize("k", [8, 5])
def test_gv_decode_w4a8(cuda, monkeypatch, I, bf16, k):
    """W4A8 (int4 codes, bf16 group scales, int8 per-row activations) through the streaming kernel: against the oracle
    of the format's definition (exact integer dots, so only the fp32 sums of the group partials and the output's bf16
    rounding can differ) and against the tensor-core decode (D3_DECODE_GV=0)."""
    banks = (gd.rand_bank("w4a8", E, 2 * I, H, 140 + k, cuda), gd.rand_bank("w4a8", E, H, I, 141 + k, cuda))
    x = gd.rand_rows(1, H, 142 + k, cuda)
    if not bf16:
        x = torch.randn((1, H), generator=torch.Generator().manual_seed(143 + k)).to(cuda)
    ids, w = gd.rand_routing(1, E, k, 144 + k, cuda)
    _lib.take_fault()
    monkeypatch.delenv("D3_DECODE_GV", raising=False)
    gv = kernels.moe_decode("w4a8", x, ids, w, banks)
    monkeypatch.setenv("D3_DECODE_GV", "0")
    tc = kernels.moe_decode("w4a8", x, ids, w, banks)
    monkeypatch.delenv("D3_DECODE_GV")
    torch.cuda.synchronize()
    assert _lib.take_fault() == 0
    assert close_to_oracle(gv, gd.baseline_oracle_decode("w4a8", x, ids, w, banks))
    assert gd.rel_l2(gv.float(), tc.float()) <= 1e-3


@pytest.mark.parametrize("I", [768, 512])
@pytest.mark.parametrize("bf16", [True, False])
def test_gv_decode_int8_convrot(cuda, monkeypatch, I, bf16):
    """The reference's int8 ConvRot layout through the streaming kernel: the row and each pair's
    SwiGLU row rotated in registers and written as three int8 terms; against the oracle of the reference's chain
    (rotate, gemv, rotate(SwiGLU), gemv, weighted sum) and against the mma.sync decode (D3_DECODE_GV=0)."""
    banks = (gd.rand_bank("int8", E, 2 * I, H, 150, cuda), gd.rand_bank("int8", E, H, I, 151, cuda))
    x = gd.rand_rows(1, H, 152, cuda)
    if not bf16:
        x = torch.randn((1, H), generator=torch.Generator().manual_seed(153)).to(cuda)
    ids, w = gd.rand_routing(1, E, 8, 154, cuda)
    _lib.take_fault()
    monkeypatch.delenv("D3_DECODE_GV", raising=False)
    gv = kernels.moe_decode("int8", x, ids, w, banks)
    monkeypatch.setenv("D3_DECODE_GV", "0")
    old = kernels.moe_decode("int8", x, ids, w, banks)
    monkeypatch.delenv("D3_DECODE_GV")
    torch.cuda.synchronize()
    assert _lib.take_fault() == 0
    ref = gd.oracle_decode("int8", x, ids, w, banks, (None, None), H)
    assert gd.rel_l2(gv.float(), ref) <= 1e-3
    assert gd.rel_l2(gv.float(), old.float()) <= 1e-3
