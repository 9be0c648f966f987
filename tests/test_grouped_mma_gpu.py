"""The tensor-core grouped GEMM (tcgen05) against the reference-API grouped kernels (themselves matched to the
reference's kernels) and the oracle: every format, both projections' shapes, ragged groups (empty, 1, 127, 128, 129,
several tiles), rows outside every group left untouched, an upper-bound tile count."""
import numpy as np
import pytest
import torch

import gpu_data as gd
from drama3_b200 import _lib, kernels
from oracle import moe

pytestmark = pytest.mark.gpu
E = 16
COUNTS = [0, 1, 127, 128, 129, 300, 5, 0, 64, 256, 17, 2, 0, 90, 33, 3]


def grouped_case(kind, N, K, seed, device):
    bank = gd.rand_bank(kind, E, N, K, seed, device)
    offsets = np.concatenate([[0], np.cumsum(COUNTS)])
    rows = int(offsets[-1]) + 7  # 7 rows past the last group stay untouched
    gen = torch.Generator().manual_seed(seed + 1)
    x = torch.randn((rows, K), generator=gen)
    x[3] *= 1e-3  # rows of very different magnitudes
    x[200] *= 50.0
    x = x.to(device)
    order = torch.randperm(E, generator=gen).tolist()  # groups listed out of expert order
    groups = torch.tensor([(e, e, 0, int(offsets[e]), COUNTS[e]) for e in order if COUNTS[e]], dtype=torch.int32)
    return bank, x, groups.to(device)


def reference_grouped(kind, x, groups, bank, cb, N):
    """The reference-API grouped kernel (slot = expert), over the same banks."""
    if kind == "fp8":
        return kernels.grouped_fp8(x, groups, bank, bank, N)
    if kind == "int8":
        return kernels.grouped_int8(x, groups, bank, bank, N)
    return kernels.grouped_codes(x, groups, bank, bank, cb, int(kind[1]), N)


@pytest.mark.parametrize("kind", gd.KINDS)
@pytest.mark.parametrize("N,K", [(1536, 2048), (2048, 768)])
def test_grouped_mma_matches_grouped_kernels(cuda, kind, N, K):
    bank, x, groups = grouped_case(kind, N, K, 11 + N + K, cuda)
    cb = gd.codebooks(kind, cuda)[0]
    tiles = kernels.grouped_tiles(COUNTS)
    got = kernels.grouped_mma(kind, x, groups, bank, cb, N, tiles)
    want = reference_grouped(kind, x, groups, bank, cb, N)
    live = int(sum(COUNTS))
    assert gd.rel_l2(got[:live], want[:live]) <= 1e-5
    # per row, not only overall
    err = (got[:live] - want[:live]).norm(dim=1) / want[:live].norm(dim=1).clamp_min(1e-30)
    assert float(err.max()) <= 1e-4


@pytest.mark.parametrize("kind", ["fp8", "w6"])
def test_grouped_mma_tile_bound_and_repeat(cuda, kind):
    """An upper-bound tile count runs the same tiles; repeated calls give identical rows (no state kept)."""
    N, K = 1536, 2048
    bank, x, groups = grouped_case(kind, N, K, 5, cuda)
    cb = gd.codebooks(kind, cuda)[0]
    exact = kernels.grouped_tiles(COUNTS)
    a = kernels.grouped_mma(kind, x, groups, bank, cb, N, exact)
    b = kernels.grouped_mma(kind, x, groups, bank, cb, N, exact + 5)
    c = kernels.grouped_mma(kind, x, groups, bank, cb, N, exact)
    live = int(sum(COUNTS))
    assert torch.isfinite(a[:live]).all()
    assert torch.equal(a[:live], b[:live]) and torch.equal(a[:live], c[:live])


@pytest.mark.parametrize("kind", gd.KINDS)
def test_grouped_mma_matches_oracle(cuda, kind):
    """A small case against the numpy restatement of the reference's grouped kernels."""
    N, K = 256, 512
    bank = gd.rand_bank(kind, 4, N, K, 21, cuda)
    gen = torch.Generator().manual_seed(22)
    x = torch.randn((200, K), generator=gen).to(cuda)
    groups = torch.tensor([(2, 2, 0, 0, 150), (0, 0, 0, 150, 1), (3, 3, 0, 151, 49)], dtype=torch.int32).to(cuda)
    cb = gd.codebooks(kind, cuda)[0]
    got = kernels.grouped_mma(kind, x, groups, bank, cb, N, kernels.grouped_tiles([150, 1, 49]))
    npb = gd.to_np_bank(bank)
    want = moe.grouped(kind, x.cpu().numpy(), groups.cpu().numpy(), npb, npb, N,
                       None if cb is None else cb.cpu().numpy())
    assert gd.rel_l2(got, want) <= 1e-5


def test_grouped_mma_rejects_bad_shapes(cuda):
    bank = gd.rand_bank("fp8", 2, 256, 512, 1, cuda)
    x = torch.zeros((4, 512), device=cuda)
    groups = torch.tensor([(0, 0, 0, 0, 4)], dtype=torch.int32, device=cuda)
    with pytest.raises(Exception):
        kernels.grouped_mma("fp8", x[:, :384].contiguous(), groups, bank, None, 256, 1)  # K % 256 != 0


@pytest.mark.parametrize("kind", ["fp8", "int8", "w4"])
def test_grouped_mma_fused_staging(cuda, kind):
    """Gather from bf16 rows by index, SwiGLU and ConvRot inside the staging give what the separate launches give."""
    N, K = 1536, 2048
    bank, x, groups = grouped_case(kind, N, K, 31, cuda)
    cb = gd.codebooks(kind, cuda)[0]
    tiles = kernels.grouped_tiles(COUNTS)
    live = int(sum(COUNTS))
    gen = torch.Generator().manual_seed(32)
    src = torch.randn((900, K), generator=gen).to(torch.bfloat16).to(cuda)
    index = torch.randint(0, 900, (x.shape[0],), generator=gen).to(cuda)
    got = kernels.grouped_mma(kind, src, groups, bank, cb, N, tiles, row_index=index)
    want = kernels.grouped_mma(kind, src[index].float(), groups, bank, cb, N, tiles)
    assert gd.rel_l2(got[:live], want[:live]) <= 1e-6
    always = torch.ones((1,), dtype=torch.int32, device=cuda)
    got = kernels.grouped_mma(kind, x, groups, bank, cb, N, tiles, rotate=True)
    want = kernels.grouped_mma(kind, kernels.rotate(x, always), groups, bank, cb, N, tiles)
    assert gd.rel_l2(got[:live], want[:live]) <= 1e-5
    # SwiGLU (+ rotation) of gate | up rows, for the down projection's K = 768
    bank2 = gd.rand_bank(kind, E, 2048, 768, 33, cuda)
    h = torch.randn((x.shape[0], 1536), generator=gen).to(cuda) * 3
    got = kernels.grouped_mma(kind, h, groups, bank2, cb, 2048, tiles, swiglu=True, rotate=kind != "fp8")
    if kind == "fp8":
        g, u = h.chunk(2, dim=-1)
        staged = g / (1 + torch.exp(-g)) * u
    else:
        staged = kernels.rotate(h, always, swiglu=True)
    want = kernels.grouped_mma(kind, staged.contiguous(), groups, bank2, cb, 2048, tiles)
    assert gd.rel_l2(got[:live], want[:live]) <= 1e-5


@pytest.mark.parametrize("wdtype", [torch.float32, torch.bfloat16])
def test_prefill_combine(cuda, wdtype):
    T, k, H = 300, 8, 2048
    gen = torch.Generator().manual_seed(40)
    sorted_out = torch.randn((T * k, H), generator=gen).to(cuda)
    order = torch.randperm(T * k, generator=gen).to(cuda)
    pos = torch.empty_like(order)
    pos[order] = torch.arange(T * k, device=cuda)
    w = torch.softmax(torch.randn((T, k), generator=gen), -1).to(wdtype).to(cuda)
    got = kernels.prefill_combine(sorted_out, pos.view(T, k), w)
    full = torch.empty_like(sorted_out)
    full[order] = sorted_out * w.reshape(-1)[order].unsqueeze(1).float()
    ref = full.view(T, k, H).sum(dim=1)
    assert got.dtype == torch.bfloat16 and gd.rel_l2(got.float(), ref.to(torch.bfloat16).float()) <= 1e-3
    got32 = kernels.prefill_combine(sorted_out, pos.view(T, k), w, dtype=torch.float32)
    assert gd.rel_l2(got32, ref) <= 1e-6


@pytest.mark.parametrize("kind", gd.KINDS)
def test_resident_prefill_fused_matches_oracle(cuda, kind):
    """A 2048-token prompt through one MoE layer of the benchmark's shape (128 experts), skewed routing, fused path."""
    from drama3_b200 import offload
    Ex, H, I = 128, 2048, 768
    gu = gd.rand_bank(kind, Ex, 2 * I, H, 50, cuda)
    dn = gd.rand_bank(kind, Ex, H, I, 51, cuda)
    cbs = gd.codebooks(kind, cuda)
    skew = -1.1 * torch.log(torch.randperm(Ex, generator=torch.Generator().manual_seed(52)).float() + 1)
    x = gd.rand_rows(2048, H, 53, cuda)
    ids, w = gd.rand_routing(2048, Ex, 8, 54, cuda, skew=skew)
    out = offload.resident_prefill(x, ids, w.to(torch.bfloat16), (gu, dn), (2 * I, H), kind, cbs, Ex)
    # the oracle on a row subset (the full prompt takes minutes in numpy): rows through their own experts
    rows = torch.arange(0, 2048, 64)
    npb = (gd.to_np_bank(gu), gd.to_np_bank(dn))
    cbn = tuple(None if c is None else c.cpu().numpy() for c in cbs)
    ref = moe.resident_prefill(kind, x[rows].float().cpu().numpy(), ids[rows].cpu().numpy(),
                               w[rows].to(torch.bfloat16).float().cpu().numpy(), npb, cbn)
    assert out.dtype == torch.bfloat16 and gd.rel_l2(out[rows].float(), ref) <= 1e-3


def test_grouped_mma_too_few_tiles_records_fault(cuda):
    """A caller that sizes fewer row tiles than its groups need gets the fault bit, not a crash or a hang."""
    from drama3_b200 import _lib
    N, K = 1536, 2048
    bank, x, groups = grouped_case("fp8", N, K, 7, cuda)
    _lib.take_fault()
    kernels.grouped_mma("fp8", x, groups, bank, None, N, 2)
    assert _lib.take_fault() & 8
    kernels.grouped_mma("fp8", x, groups, bank, None, N, kernels.grouped_tiles(COUNTS))
    assert _lib.take_fault() == 0


def test_grouped_mma_many_units_per_cta(cuda):
    """A prompt large enough that each CTA takes more units than its shared-memory unit table holds (128 experts x
    800 rows: 10752 units over at most 148 CTAs, 64 cached): the last experts' units come from the tile table, and
    their rows equal those of a call holding only those experts, bit for bit (tiles are computed independently)."""
    E, N, K, per = 128, 1536, 2048, 800
    kind = "w6a8"
    bank = gd.rand_bank(kind, E, N, K, 400, cuda)
    x = gd.rand_rows(E * per, K, 401, cuda)
    groups = torch.tensor([(e, e, 0, e * per, per) for e in range(E)], dtype=torch.int32, device=cuda)
    tiles = kernels.grouped_tiles([per] * E)
    assert tiles * (N // 128) > 64 * 148
    _lib.take_fault()
    big = kernels.grouped_mma(kind, x, groups, bank, None, N, tiles)
    last = torch.tensor([(e, e, 0, (e - E + 2) * per, per) for e in (E - 2, E - 1)], dtype=torch.int32, device=cuda)
    small = kernels.grouped_mma(kind, x[(E - 2) * per:].contiguous(), last, bank, None, N,
                                kernels.grouped_tiles([per, per]))
    torch.cuda.synchronize()
    assert _lib.take_fault() == 0
    assert torch.equal(big[(E - 2) * per:], small)
