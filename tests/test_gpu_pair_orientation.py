"""The two orientations of the CTA-pair W8A8 GEMM give identical bits.

Normal orientation: activation rows are the pair's 256-row MMA operand and the
epilogue stages 32 x 32 tiles in shared memory for TMA stores.  Swapped
orientation (the default for row-major outputs): the weight columns are the
256-row operand, activation rows the MMA N, and the epilogue stores each
output row's 32 columns from registers as one 128-byte line.  The INT32 sums
are exact and both epilogues evaluate the same IEEE operations, so outputs
must agree bit for bit; the oracle checks sampled rows within the W8A8
tolerance (max-abs-rel 2e-3) and mode 0 / the raw INT32 mode exactly.

Shapes cover ragged M (a last activation tile with few rows), N that is not a
multiple of the 256-column weight tile, K that is not a multiple of the
128-byte k-block, both activation-tile widths (256 and 128 rows) and the
benchmark's C4 shape.
"""
import numpy as np
import pytest

import htpg
import oracle as O

pytestmark = pytest.mark.gpu

W8A8_TOL = 2e-3

SHAPES = [  # (m, k, n)
    (1000, 512, 1280),      # ragged M, 128-row activation tiles
    (2100, 800, 1344),      # K = 6.25 k-blocks, N = 5.25 weight tiles
    (4100, 256, 4608),      # 4 rows in the last activation tile
    (4096, 6144, 1536),     # C3 fc2 shape (48 k-blocks)
    (4096, 1536, 1536),     # C3 out-projection shape (96 tiles on 74 SM pairs)
    (257, 1152, 4608),
]


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _both(gpu, c, mode, bias, raw=False):
    import torch
    hw = htpg.w8a8_weights(_t(c.blob, gpu), c.k, c.n)
    x = _t(c.x, gpu)
    b = _t(bias, gpu) if bias is not None else None
    outs, plans = [], []
    try:
        for direct in (True, False):
            htpg.set_pair_direct(direct)
            plans.append(htpg.plan_info(0, c.m, c.n, c.k)["swap"])
            if raw:
                o = torch.full((c.m, c.n), -7, dtype=torch.int32, device=gpu)
                htpg.check(htpg.w8a8_run(hw, o, x, None, mode=4), "raw run")
            else:
                o = torch.full((c.m, c.n), float("nan"), device=gpu)
                htpg.check(htpg.w8a8_run(hw, o, x, b, mode=mode), "run")
            htpg.check(htpg.check_device(), "device watchdog")
            outs.append(o.cpu().numpy())
    finally:
        htpg.set_pair_direct(True)
    assert plans == [3, 0], plans          # swapped pair, then the normal pair orientation
    return outs


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_raw_int32_identical_and_exact(gpu, m, k, n):
    c = O.make_w8a8(21, f"po{m}", m, k, n, 0.01, False, 0, inverse_range=(0.5, 2.0) if m % 2 else None)
    a, b = _both(gpu, c, 4, None, raw=True)
    np.testing.assert_array_equal(a, b)
    rows = np.unique(np.concatenate([np.arange(0, m, 97), np.arange(max(0, m - 5), m)])).astype(np.int32)
    _, _, _, acc = O.w8a8_linear(c.x[rows], c.blob, k, n, want_intermediates=True)
    np.testing.assert_array_equal(a[rows], acc)


@pytest.mark.parametrize("m,k,n", SHAPES[:3] + SHAPES[5:])
@pytest.mark.parametrize("mode,with_bias", [(0, False), (0, True), (1, True), (2, False), (2, True)])
def test_outputs_identical(gpu, m, k, n, mode, with_bias):
    c = O.make_w8a8(22, f"po{m}", m, k, n, 0.005, with_bias, mode)
    bias = c.bias if with_bias else None
    a, b = _both(gpu, c, mode, bias)
    assert not np.isnan(a).any()
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    rows = np.unique(np.concatenate([np.arange(3, m, 61), [m - 1]])).astype(np.int32)
    ref = O.w8a8_linear(c.x, c.blob, k, n, bias=bias, mode=mode, rows=rows)
    if mode == 0:
        np.testing.assert_array_equal(a[rows].view(np.uint32), ref.view(np.uint32))
    else:
        assert O.max_abs_rel(a[rows], ref) <= W8A8_TOL


def test_c4_identical(gpu):
    c = O.config_c4()
    a, b = _both(gpu, c, 1, c.bias)
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))


def test_ldo_padded_output(gpu, lib):
    """A row pitch larger than N (ldo = n + 40 floats): only the first n
    columns of each row are written by either orientation."""
    import torch
    m, k, n = 1500, 768, 1536
    c = O.make_w8a8(23, "ldo", m, k, n, 0.01, True, 1)
    hw = htpg.w8a8_weights(_t(c.blob, gpu), k, n)
    x, bias = _t(c.x, gpu), _t(c.bias, gpu)
    ldo = n + 40
    res = []
    try:
        for direct in (True, False):
            htpg.set_pair_direct(direct)
            o = torch.full((m, ldo), 123.0, device=gpu)
            htpg.check(htpg.w8a8_run(hw, o, x, bias, mode=1, ldo=ldo), "run")
            htpg.check(htpg.check_device(), "watchdog")
            res.append(o.cpu().numpy())
    finally:
        htpg.set_pair_direct(True)
    np.testing.assert_array_equal(res[0].view(np.uint32), res[1].view(np.uint32))
    assert (res[0][:, n:] == 123.0).all()


@pytest.mark.parametrize("m,k,n", [(4096, 3200, 1536), (4100, 4096, 1536), (4096, 6144, 1536), (4096, 6144, 1280)])
@pytest.mark.parametrize("mode,with_bias", [(4, False), (1, True), (2, False), (0, True)])
def test_tail_split_identical(gpu, m, k, n, mode, with_bias):
    """A last round of tiles cut into K pieces (the pieces exchange their INT32
    sums, each finishing the 32-row chunks it owns) gives the bits of whole
    tiles: ragged K pieces (25 k-blocks in 3), two pieces with a ragged last
    activation tile, the C3 fc2 shape (48 k-blocks in 3) and eight pieces of
    six k-blocks (one chunk per piece)."""
    import torch
    c = O.make_w8a8(25, f"ts{m}", m, k, n, 0.01, with_bias, mode if mode != 4 else 0)
    hw = htpg.w8a8_weights(_t(c.blob, gpu), k, n)
    x = _t(c.x, gpu)
    b = _t(c.bias, gpu) if with_bias else None
    outs = []
    try:
        for split in (True, False):
            htpg.set_pair_tail_split(split)
            plan = htpg.plan_info(0, m, n, k)
            assert plan["swap"] == 3 and (plan["tail_s"] > 1) == split
            if mode == 4:
                o = torch.full((m, n), -7, dtype=torch.int32, device=gpu)
            else:
                o = torch.full((m, n), float("nan"), device=gpu)
            htpg.check(htpg.w8a8_run(hw, o, x, b, mode=mode), "run")
            htpg.check(htpg.check_device(), "device watchdog")
            outs.append(o.cpu().numpy())
    finally:
        htpg.set_pair_tail_split(True)
    a, w = outs
    np.testing.assert_array_equal(a.view(np.uint32), w.view(np.uint32))
    rows = np.unique(np.concatenate([np.arange(0, m, 211), np.arange(max(0, m - 8), m)])).astype(np.int32)
    if mode == 4:
        _, _, _, acc = O.w8a8_linear(c.x[rows], c.blob, k, n, want_intermediates=True)
        np.testing.assert_array_equal(a[rows], acc)
    else:
        assert not np.isnan(a).any()
        ref = O.w8a8_linear(c.x, c.blob, k, n, bias=c.bias if with_bias else None, mode=mode, rows=rows)
        if mode == 0:
            np.testing.assert_array_equal(a[rows].view(np.uint32), ref.view(np.uint32))
        else:
            assert O.max_abs_rel(a[rows], ref) <= W8A8_TOL
