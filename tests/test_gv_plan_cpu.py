"""The one-line streaming decode's work plan (csrc/decode_gv.cuh, moe_decode_gv_kernel), restated in integers and
checked on the CPU for every grid size the dispatch accepts (128..256 CTAs) and every count of valid pairs (1..8):
every phase-1 unit is owned by exactly one CTA, every output row by exactly one row block of each pair, a row block
fits the 8 MMA warps' 16-row tiles, the ring never reuses a stage that still holds down rows, and the counters it
uses stay inside the decode workspace's synchronization arrays."""
import pytest

GV_K, UNIT_CH, STAGES, P2_ROWS, WARPS = 2048, 4, 3, 64, 8
MIN_GRID, MAX_GRID = 128, 256          # d3::GV_MIN_GRID, d3::DEC_MAX_GRID
UNITS = {"fp8c": 4, "fp8": 4, "int8": 4, "w4a8": 8}  # units per ring stage


def plan(G, nv, I, units_per_stage):
    """Per CTA: (unit range, phase-2 pair, row range, ring items), as the kernel computes them."""
    upp = I // UNIT_CH
    T1 = nv * upp
    RB = G // nv
    RR = (GV_K + RB - 1) // RB
    NRB = (GV_K + RR - 1) // RR
    out = []
    for b in range(G):
        u_lo, u_hi = b * T1 // G, (b + 1) * T1 // G
        live = b < nv * RB and b % RB < NRB
        q2, rb = b // RB, b % RB
        r0 = rb * RR
        rows2 = min(GV_K, r0 + RR) - r0 if live else 0
        n1 = u_hi - u_lo
        n1s = (n1 + units_per_stage - 1) // units_per_stage
        items = n1s + (rows2 + P2_ROWS - 1) // P2_ROWS
        out.append(dict(u=(u_lo, u_hi), live=live, q2=q2, rb=rb, r0=r0, rows2=rows2, n1s=n1s, items=items,
                        nt2=(rows2 + 15) // 16, NRB=NRB, RB=RB))
    return out


@pytest.mark.parametrize("kind", sorted(UNITS))
@pytest.mark.parametrize("I", [512, 768])
def test_plan_covers_everything_once(kind, I):
    for G in range(MIN_GRID, MAX_GRID + 1):
        for nv in range(1, 9):
            p = plan(G, nv, I, UNITS[kind])
            # units: a partition of [0, nv * I / 4) in CTA order
            owned = [u for c in p for u in range(*c["u"])]
            assert owned == list(range(nv * I // UNIT_CH)), (G, nv)
            # rows: each pair's row blocks partition [0, 2048); each block has one CTA per pair
            for q in range(nv):
                rows = sorted(r for c in p if c["live"] and c["q2"] == q for r in range(c["r0"], c["r0"] + c["rows2"]))
                assert rows == list(range(GV_K)), (G, nv, q)
            blocks = {}
            for c in p:
                if c["live"]:
                    blocks.setdefault(c["rb"], []).append(c)
            for rb, members in blocks.items():
                assert sorted(m["q2"] for m in members) == list(range(nv))
                assert len({(m["r0"], m["rows2"]) for m in members}) == 1  # the same rows for every pair
            # the consumers of each pair: NRB row blocks (the depart counter's target)
            for q in range(nv):
                assert sum(1 for c in p if c["live"] and c["q2"] == q) == p[0]["NRB"]


@pytest.mark.parametrize("kind", sorted(UNITS))
@pytest.mark.parametrize("I", [512, 768])
def test_plan_fits_tiles_ring_and_counters(kind, I):
    for G in range(MIN_GRID, MAX_GRID + 1):
        for nv in range(1, 9):
            for c in plan(G, nv, I, UNITS[kind]):
                assert c["nt2"] <= WARPS                  # one 16-row down tile a warp
                assert c["rows2"] <= WARPS * 16
                # down-row items (indices n1s..items-1) never wait on a stage that holds another down-row item
                for i in range(c["n1s"], c["items"]):
                    if i >= STAGES:
                        assert i - STAGES < c["n1s"]
                # counters: a.depart[32 q + 16] for q < 8 and a.arrive[rb] for rb < G, both 256 words
                assert 32 * (nv - 1) + 16 < 256 and c["rb"] < 256
                # the ring holds the CTA's whole unit share at the start for the e4m3 formats at 8 pairs
            share = max(c["u"][1] - c["u"][0] for c in plan(G, nv, I, UNITS[kind]))
            assert share <= 2 * UNITS[kind] * STAGES  # at most two passes of the ring


def test_plan_matches_the_benchmark_grid():
    """148 CTAs, 8 pairs, I = 768: 10-11 units a CTA, 18 row blocks of at most 114 rows."""
    p = plan(148, 8, 768, 4)
    assert {c["u"][1] - c["u"][0] for c in p} == {10, 11}
    assert p[0]["RB"] == 18 and max(c["rows2"] for c in p) == 114
    assert sum(c["live"] for c in p) == 144
