"""Legality sweep of the M-keyed tile planner (htpg_plan_info).

Mirrors the structure of the reference's planner test
(tests/test-f16-gemm-plan.c:5-44): every plan over a grid of shapes must be
legal for the device — tiles cover the problem, shared memory fits, the grid
fits the SMs (an even number of CTAs for CTA-pair tiles), K splits only where
the reduction is exact (INT8) and never leave an empty split, and the FP16 path
keeps K whole inside a CTA so its accumulation order does not depend on the plan.
"""
import itertools

import pytest

import htpg

SMEM_LIMIT = 232448
MS = [1, 2, 4, 16, 17, 31, 32, 33, 77, 128, 129, 255, 256, 257, 1000, 4096, 4100, 16384, 65536]
NS = [32, 64, 128, 192, 640, 1536, 3072, 4096, 4608, 6144, 14336, 16384]
KS = [32, 64, 160, 768, 1152, 1536, 4096, 6144, 14336, 16384]


@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("sms", [148, 132, 16])
def test_plans_are_legal(kind, sms):
    checked = 0
    for m, n, k in itertools.product(MS, NS, KS):
        if kind == 0 and n % 64:
            continue
        p = htpg.plan_info(kind, m, n, k, sms)
        elems = 128 if kind == 0 else 64
        kb_total = -(-k // elems)
        assert p["kb_total"] == kb_total
        assert p["smem"] <= SMEM_LIMIT
        if p["swap"] == 2:
            # register-fed decode: 16-column groups x k-blocks cut into `units`
            # contiguous chunks, each spanning at most 32 groups
            assert kind == 0 and m <= 16 and p["bn"] == (8 if m <= 8 else 16)
            assert p["tiles_a"] * 16 >= n and p["tiles_b"] == 1 and p["splits"] == 1
            atoms = p["tiles_a"] * kb_total
            assert p["grid"] == min(p["units"], sms) and 1 <= p["units"] <= atoms
            assert -(-atoms // p["units"]) <= 30 * kb_total
            assert p["units"] * 2 * 16 * p["bn"] * 4 + p["tiles_a"] * 4 <= 2 * 1024 * 1024 + 4096
            checked += 1
            continue
        tiles = p["tiles_a"] * p["tiles_b"] * p["splits"]
        if p["tail_s"] > 1:
            # swapped pair plan with its sparse last round cut into K pieces
            pairs = sms // 2
            assert p["swap"] == 3 and p["full_units"] % pairs == 0 and p["full_units"] < tiles
            tail = tiles - p["full_units"]
            assert tail <= pairs // 2 and tail * p["tail_s"] <= pairs
            assert p["units"] == p["full_units"] + tail * p["tail_s"] and kb_total >= max(24, 4 * p["tail_s"])
            assert p["tail_s"] <= p["bn"] // 32
        else:
            assert p["units"] == tiles and p["full_units"] == p["units"]
        assert 1 <= p["grid"] <= sms and p["grid"] <= (2 * p["units"] if p["bn"] else p["units"])
        # K ranges: every split non-empty, together exactly [0, kb_total)
        assert p["splits"] * p["kb_per_split"] >= kb_total
        assert (p["splits"] - 1) * p["kb_per_split"] < kb_total
        if p["swap"] == 3:
            # CTA pair in the swapped orientation: 256-column weight tiles x bn rows
            assert kind == 0 and m > 128 and p["bn"] in (128, 256) and p["splits"] == 1
            assert p["tiles_a"] == -(-n // 256) and p["tiles_b"] == -(-m // p["bn"]) and p["grid"] % 2 == 0
        elif p["swap"]:
            assert kind == 0 and m <= 32 and p["bn"] in (16, 32)
            assert p["tiles_a"] * 128 >= n and p["tiles_b"] * p["bn"] >= m
        else:
            assert p["splits"] == 1                       # K whole in the normal orientation
            pair = p["tiles_a"] * 256 >= m and p["tiles_a"] == -(-m // 256) and m > 128 \
                and p["grid"] % 2 == 0 and p["bn"] in (128, 256)
            rows = 256 if pair else 128
            assert p["tiles_a"] * rows >= m and p["tiles_b"] * p["bn"] >= n
            assert p["bn"] in (32, 64, 128, 256)
        if kind == 1:
            assert p["splits"] == 1 and not p["swap"]
        checked += 1
    assert checked > 1500


def test_headline_shapes():
    # C4 and the C3 linears take CTA-pair 256-row tiles; C5 decode shapes the
    # register-fed decode kernel over all SMs (or, switched, the swapped K-split
    # tcgen05 plan); C1/C2 single-CTA tiles that still fill the SMs.
    c4 = htpg.plan_info(0, 16384, 6144, 1536)
    assert c4["swap"] == 3 and c4["bn"] == 256 and c4["tiles_a"] == 24 and c4["tiles_b"] == 64
    assert c4["grid"] == 148
    try:
        htpg.set_pair_direct(False)
        c4 = htpg.plan_info(0, 16384, 6144, 1536)
        assert c4["swap"] == 0 and c4["bn"] == 256 and c4["tiles_a"] == 64 and c4["grid"] == 148
    finally:
        htpg.set_pair_direct(True)
    for m in (1, 4, 16):
        up = htpg.plan_info(0, m, 14336, 4096)
        down = htpg.plan_info(0, m, 4096, 14336)
        # register-fed where the swapped plan would split K, and at M <= 8
        assert up["swap"] == (2 if m <= 8 else 1) and down["swap"] == 2 and down["grid"] == 148
    try:
        htpg.set_decode_kernel(1)
        for m in (1, 4, 16):
            up = htpg.plan_info(0, m, 14336, 4096)
            down = htpg.plan_info(0, m, 4096, 14336)
            assert up["swap"] == 1 and down["swap"] == 1 and down["splits"] > 1
            assert down["units"] <= 148 and up["units"] <= 148
    finally:
        htpg.set_decode_kernel(0)
    assert htpg.plan_info(0, 17, 4096, 14336)["swap"] == 1
    c1 = htpg.plan_info(0, 256, 4608, 1152)
    assert not c1["swap"] and c1["units"] >= 0.85 * 148
    c2 = htpg.plan_info(1, 77, 3072, 768)
    assert not c2["swap"] and c2["splits"] == 1


def _tail_split(tiles, kb_total, bn, pairs=74):
    """Restatement of the planner's tail split: (full_units, tail_s)."""
    tail = tiles % pairs
    if tail == 0 or kb_total < 24:
        return tiles, 1
    pieces = min(pairs // tail, kb_total // 4, bn // 32)
    if pieces < 2:
        return tiles, 1
    return tiles - tail, pieces


@pytest.mark.parametrize("m,n,k", [(4096, 1536, 1536), (4096, 1536, 6144), (4096, 6144, 1536), (4096, 4608, 1536),
                                   (16384, 6144, 1536), (1000, 1280, 1536), (4096, 1536, 3200), (4100, 1536, 4096),
                                   (4096, 1280, 6144)])
def test_tail_split(m, n, k):
    """Swapped pair plans cut a last round that would leave at least half of the
    74 SM pairs idle into K pieces of tiles with at least 24 k-blocks; the C3
    fc2 (96 tiles of 48 k-blocks: 74 whole, 22 tail tiles x 3 pieces) takes
    it, C4, the other C3 shapes (fuller last rounds or 12 k-blocks) keep
    whole tiles."""
    p = htpg.plan_info(0, m, n, k)
    assert p["swap"] == 3
    tiles = p["tiles_a"] * p["tiles_b"]
    full, s = _tail_split(tiles, p["kb_total"], p["bn"])
    assert (p["full_units"], p["tail_s"]) == (full, s)
    assert p["units"] == full + (tiles - full) * s
    if (m, n, k) == (4096, 1536, 6144):
        assert (full, s, p["units"]) == (74, 3, 140)
    if (m, n, k) in ((16384, 6144, 1536), (4096, 4608, 1536)):
        assert s == 1
    try:
        htpg.set_pair_tail_split(False)
        q = htpg.plan_info(0, m, n, k)
        assert q["tail_s"] == 1 and q["units"] == tiles and q["bn"] == p["bn"]
    finally:
        htpg.set_pair_tail_split(True)


def test_qk0_plan():
    """Fused opcode 2-4 kernel: 16/32 activation rows per tile, stream-K grid of
    at most one CTA per SM with at least four k-blocks each."""
    p = htpg.qk0_plan_info(2, 1, 14336, 4096)
    assert p["bn"] == 16 and p["tiles_a"] == 112 and p["kb_total"] == 64 and p["grid"] == 148
    p = htpg.qk0_plan_info(8, 32, 128, 64)
    assert p["bn"] == 32 and p["grid"] == 1 and p["smem"] <= 232448
    p = htpg.qk0_plan_info(20, 17, 384, 96)
    assert p["bn"] == 32 and p["tiles_b"] == 1 and p["kb_total"] == 2 and p["grid"] == 1


def _decode_slots(atoms, chunks, kb):
    """Restatement of decode.cu's chunk arithmetic: which (chunk, side) partial
    tiles each column group's finisher reads, and which ones chunks write."""
    start = [atoms * c // chunks for c in range(chunks + 1)]
    owner = lambda a: ((a + 1) * chunks - 1) // atoms
    written, read = {}, {}
    for c in range(chunks):
        a0, a1 = start[c], start[c + 1]
        assert a1 > a0
        cg0, cg1 = a0 // kb, (a1 - 1) // kb
        assert cg1 - cg0 + 1 <= 32
        for cg in range(cg0, cg1 + 1):
            if cg * kb < a0 or (cg + 1) * kb > a1:
                key = (c, 0 if cg == cg0 else 1)
                assert key not in written
                written[key] = cg
    for cg in range(-(-atoms // kb)):
        first, last = owner(cg * kb), owner((cg + 1) * kb - 1)
        assert start[first] <= cg * kb < start[first + 1]
        if first == last:
            continue
        for o in range(first, last + 1):
            key = (o, 0 if start[o] // kb == cg else 1)
            assert key not in read
            read[key] = cg
    return written, read


@pytest.mark.parametrize("m,n,k,sms", [(1, 14336, 4096, 148), (16, 4096, 14336, 148), (3, 64, 32, 148),
                                       (9, 64, 16384, 148), (16, 1536, 6144, 132), (1, 128, 16384, 16),
                                       (2, 192, 1152, 148), (7, 65536, 32, 148), (1, 6144, 160, 148)])
def test_decode_partial_tiles_are_consistent(m, n, k, sms):
    """Every partial tile a chunk publishes is read by exactly the finisher of
    its column group, and the arrival count equals the number of writers."""
    p = htpg.plan_info(0, m, n, k, sms)
    assert p["swap"] == 2
    kb = p["kb_total"]
    written, read = _decode_slots(p["tiles_a"] * kb, p["units"], kb)
    assert written == read


QK0_DECODE_NS = [32, 96, 160, 1536, 4096, 14336]
QK0_DECODE_KS = [32, 96, 2048, 4096, 14336, 65536]


@pytest.mark.parametrize("wtype", [2, 8, 20])
@pytest.mark.parametrize("sms", [148, 16])
def test_qk0_decode_plans_are_legal(wtype, sms):
    """Register-fed opcode 2-4 decode plans (m <= 32): the grid is the tile
    groups x k ranges, no range is empty, the activation slice holds the widest
    range, a CTA's shared memory fits (two CTAs per SM within 112 KB each; a
    one-per-SM plan asks for more than half the SM so its CTAs spread)."""
    rings = 16 * 4 * 8 * (272 if wtype == 8 else 144)
    for m, n, k in itertools.product([1, 4, 8, 9, 16, 17, 32], QK0_DECODE_NS, QK0_DECODE_KS):
        p = htpg.qk0_decode_plan_info(wtype, m, n, k, sms)
        nt = 1 if m <= 8 else 2 if m <= 16 else 4
        assert p["ntiles"] == n // 32 and p["ktiles"] == k // 32
        assert p["tiles"] in (16, 8, 4) and p["per_sm"] in (1, 2)
        assert 1 <= p["splits"] <= p["ktiles"]
        assert p["grid"] == -(-p["ntiles"] // p["tiles"]) * p["splits"]
        widest = -(-p["ktiles"] // p["splits"])
        assert p["slice"] == 8 * nt * (widest * 32 + 16) * 2 <= 64 * 1024
        assert p["smem"] == max(rings + p["slice"], 116 * 1024 if p["per_sm"] == 1 else 0)
        assert p["smem"] <= (112 * 1024 if p["per_sm"] == 2 else 227 * 1024)
        if wtype == 8:
            assert p["per_sm"] == 1   # Q8_0's rings leave no room for two CTAs


@pytest.mark.parametrize("m,k,n,want", [
    (1, 4096, 14336, {2: (1, 16), 8: (1, 16), 20: (1, 16)}),
    (16, 4096, 14336, {2: (1, 16), 8: (1, 16), 20: (1, 16)}),
    (4, 14336, 4096, {2: (1, 16), 8: (1, 16), 20: (1, 16)}),
    (16, 14336, 4096, {2: (1, 16), 8: (1, 16), 20: (1, 16)}),
    (32, 4096, 14336, {2: (1, 16), 8: (1, 16), 20: (1, 16)}),
    (32, 14336, 4096, {2: (1, 16), 8: (1, 16), 20: (1, 16)}),
])
def test_qk0_decode_plan_choices(m, k, n, want):
    """On the LLM projections the planner picks the launch shape measured
    fastest (back to back on a B200) or one within 4% of it; a forced shape
    overrides it until reset."""
    for wtype, (per_sm, tiles) in want.items():
        p = htpg.qk0_decode_plan_info(wtype, m, n, k)
        assert (p["per_sm"], p["tiles"]) == (per_sm, tiles), wtype
        assert p["grid"] <= per_sm * 148
    try:
        htpg.set_qdec_shape(1, 16)
        assert htpg.qk0_decode_plan_info(2, m, n, k)["tiles"] == 16
        htpg.set_qdec_shape(2, 4)
        with pytest.raises(RuntimeError):
            htpg.qk0_decode_plan_info(8, m, n, k)   # Q8_0: no room for two CTAs per SM
    finally:
        htpg.set_qdec_shape(0, 0)
    assert htpg.lib().htpg_set_qdec_shape(3, 4) == htpg.EARGS
    assert htpg.lib().htpg_set_qdec_shape(1, 2) == htpg.EARGS
