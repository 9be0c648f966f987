"""The BASELINE layouts (per-channel fp8, W4A8, W6A8 with int8 activations) through the fused decode, against the
oracle's restatement; the quantizers' banks through it end to end."""
import numpy as np
import pytest
import torch

import gpu_data as gd
from drama3_b200 import kernels
from oracle import moe

pytestmark = pytest.mark.gpu
E, H, I = 16, 2048, 768


@pytest.mark.parametrize("kind", gd.BASELINE_KINDS)
@pytest.mark.parametrize("M", [1, 4, 16])
def test_baseline_decode_matches_oracle(cuda, kind, M):
    banks = (gd.rand_bank(kind, E, 2 * I, H, 200 + M, cuda), gd.rand_bank(kind, E, H, I, 300 + M, cuda))
    x = gd.rand_rows(M, H, 400 + M, cuda)
    ids, w = gd.rand_routing(M, E, 8, 500 + M, cuda)
    out = kernels.moe_decode(kind, x, ids, w, banks)
    ref = gd.baseline_oracle_decode(kind, x, ids, w, banks)
    assert out.dtype == torch.bfloat16 and gd.rel_l2(out.float(), ref) <= 1e-3


def test_fp8c_float32_rows(cuda):
    """fp32 rows take the hi + lo activation path."""
    banks = (gd.rand_bank("fp8c", E, 2 * I, H, 31, cuda), gd.rand_bank("fp8c", E, H, I, 32, cuda))
    x = torch.randn((4, H), generator=torch.Generator().manual_seed(33)).to(cuda)
    ids, w = gd.rand_routing(4, E, 8, 34, cuda)
    out = kernels.moe_decode("fp8c", x, ids, w, banks)
    assert gd.rel_l2(out.float(), gd.baseline_oracle_decode("fp8c", x, ids, w, banks)) <= 1e-3


@pytest.mark.parametrize("kind", gd.BASELINE_KINDS)
def test_quantized_banks_end_to_end(cuda, kind):
    """Banks from the restated quantizers (N(0, 0.02) experts, BASELINE configs[1..3]) decode to what the oracle gives
    for the same bytes, and near the unquantized experts."""
    rng = np.random.default_rng(9)
    w13 = rng.normal(0, 0.02, size=(4, 2 * I, H)).astype(np.float32)
    w2 = rng.normal(0, 0.02, size=(4, H, I)).astype(np.float32)
    npb = (moe.make_baseline_bank(kind, w13), moe.make_baseline_bank(kind, w2))

    def dev(b):
        out = {}
        for n, v in b.items():
            t = torch.from_numpy(v)
            out[n] = (t.view(torch.bfloat16) if v.dtype == np.uint16 else t).to(cuda)
        return out

    banks = tuple(dev(b) for b in npb)
    x = gd.rand_rows(2, H, 40, cuda)
    ids = torch.tensor([[0, 1, 2, 3, 0, 1, 2, 3][:4], [3, 2, 1, 0]], device=cuda)
    w = torch.tensor([[0.4, 0.3, 0.2, 0.1], [0.25, 0.25, 0.25, 0.25]], device=cuda)
    out = kernels.moe_decode(kind, x, ids, w, banks)
    ref = moe.baseline_decode(kind, x.float().cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy(), npb)
    assert gd.rel_l2(out.float(), ref) <= 1e-3


def grouped_oracle(kind, x, groups, bank, N):
    npb = gd.to_np_bank(bank)
    xn = x.float().cpu().numpy()
    out = np.zeros((x.shape[0], N), np.float32)
    for e, _, _, first, rows in groups.cpu().tolist():
        out[first:first + rows] = moe.baseline_rows(kind, xn[first:first + rows], npb, e * N, N)
    return out


@pytest.mark.parametrize("kind", gd.BASELINE_KINDS)
@pytest.mark.parametrize("N,K", [(1536, 2048), (2048, 768)])
def test_baseline_grouped_mma(cuda, kind, N, K):
    counts = [0, 1, 127, 128, 129, 300, 5, 0, 64, 256, 17, 2, 0, 90, 33, 3]
    bank = gd.rand_bank(kind, E, N, K, 60 + K, cuda)
    offsets = np.concatenate([[0], np.cumsum(counts)])
    gen = torch.Generator().manual_seed(61)
    x = torch.randn((int(offsets[-1]), K), generator=gen).to(cuda)
    groups = torch.tensor([(e, e, 0, int(offsets[e]), n) for e, n in enumerate(counts) if n],
                          dtype=torch.int32).to(cuda)
    got = kernels.grouped_mma(kind, x, groups, bank, None, N, kernels.grouped_tiles(counts))
    want = grouped_oracle(kind, x, groups, bank, N)
    assert gd.rel_l2(got, want) <= 1e-5


@pytest.mark.parametrize("kind", gd.BASELINE_KINDS)
def test_baseline_resident_prefill(cuda, kind):
    """A 2048-token prompt (skewed routing, 128 experts) through the fused prompt pass, rows checked on the oracle."""
    from drama3_b200 import offload
    Ex = 128
    gu, dn = gd.rand_bank(kind, Ex, 2 * I, H, 70, cuda), gd.rand_bank(kind, Ex, H, I, 71, cuda)
    skew = -1.1 * torch.log(torch.randperm(Ex, generator=torch.Generator().manual_seed(72)).float() + 1)
    x = gd.rand_rows(2048, H, 73, cuda)
    ids, w = gd.rand_routing(2048, Ex, 8, 74, cuda, skew=skew)
    out = offload.resident_prefill(x, ids, w.to(torch.bfloat16), (gu, dn), (2 * I, H), kind, (None, None), Ex)
    rows = torch.arange(0, 2048, 128)
    ref = moe.baseline_prefill(kind, x[rows].float().cpu().numpy(), ids[rows].cpu().numpy(),
                               w[rows].to(torch.bfloat16).float().cpu().numpy(),
                               (gd.to_np_bank(gu), gd.to_np_bank(dn)))
    assert out.dtype == torch.bfloat16 and gd.rel_l2(out[rows].float(), ref) <= 1e-3
