"""The CTA-pair W8A8 kernel that keeps the weight columns in tensor memory.

For CTA-pair plans with K <= 1536 the weight tile is the MMA's A operand in
tensor memory and only activation tiles stream through shared memory.  Its
INT32 accumulators and mode-0 outputs must be bit-exact against the oracle
(linear_w8a8.c:130-192) and every mode must equal the streaming CTA-pair
kernel bit for bit (same per-element epilogue).
"""
import numpy as np
import pytest

import htpg
import oracle as O

W8A8_TOL = 2e-3

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _run(lib, gpu, c, mode, bias=None, raw=False, tw=True):
    import torch
    blob, x = _t(c.blob, gpu), _t(c.x, gpu)
    out = torch.full((c.m, c.n), float("nan"), dtype=torch.float32, device=gpu)
    if raw:
        out = torch.empty(c.m, c.n, dtype=torch.int32, device=gpu)
        mode = 4
    b = _t(bias, gpu) if bias is not None else None
    htpg.set_tmem_weights(tw)
    try:
        rc = lib.htpg_w8a8_linear(htpg.ptr(out), htpg.ptr(x), htpg.ptr(blob), htpg.ptr(b), c.m, c.k, c.n,
                                  c.n, mode, htpg.stream_ptr())
        htpg.check(rc, "htpg_w8a8_linear")
        htpg.check(htpg.check_device(), "device watchdog")
    finally:
        htpg.set_tmem_weights(False)
        lib.htpg_weight_cache_drop(htpg.ptr(blob))
    return out.cpu().numpy()


# pair plans with K <= 1536: ragged M (last 64-token sub-tile partial), N not a
# multiple of 256 (last weight tile partial), K not a multiple of 128, a pair
# whose range spans several weight tiles
SHAPES = [(1000, 512, 1280), (2048, 768, 2304), (4100, 256, 4608), (2304, 1184, 3072), (1500, 1536, 1216),
          (4096, 1536, 1536)]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_plan_is_pair_k_le_1536(m, k, n):
    p = htpg.plan_info(0, m, n, k)
    assert p["swap"] == 0 and p["tiles_a"] == (m + 255) // 256 and p["kb_total"] <= 12


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_tw_int32_bitexact(gpu, lib, m, k, n):
    c = O.make_w8a8(11, f"tw{m}", m, k, n, 0.01, False, 0, inverse_range=(0.5, 2.0) if m % 2 else None)
    _, _, _, acc = O.w8a8_linear(c.x, c.blob, k, n, want_intermediates=True)
    np.testing.assert_array_equal(_run(lib, gpu, c, 0, raw=True), acc)


@pytest.mark.parametrize("m,k,n", SHAPES[:5])
def test_tw_output_bitexact_mode0(gpu, lib, m, k, n):
    c = O.make_w8a8(12, f"tw{m}", m, k, n, 0.01, False, 0)
    ref = O.w8a8_linear(c.x, c.blob, k, n)
    got = _run(lib, gpu, c, 0)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("with_bias", [False, True])
def test_tw_matches_streaming_pair_kernel(gpu, lib, mode, with_bias):
    m, k, n = 2100, 1536, 2304
    c = O.make_w8a8(13, "twm", m, k, n, 0.005, with_bias, mode)
    bias = c.bias if with_bias else None
    a = _run(lib, gpu, c, mode, bias=bias, tw=True)
    b = _run(lib, gpu, c, mode, bias=bias, tw=False)
    assert not np.isnan(a).any()
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))
    rows = np.arange(1, m, 41, dtype=np.int32)
    ref = O.w8a8_linear(c.x, c.blob, k, n, bias=bias, mode=mode, rows=rows)
    assert O.max_abs_rel(a[rows], ref) <= W8A8_TOL


def test_tw_c4_matches_streaming_pair_kernel(gpu, lib):
    """C4 (M=16384, K=1536, N=6144, bias + GELU): identical bits, sampled rows
    against the oracle."""
    import torch
    m, k, n = 16384, 1536, 6144
    c = O.make_w8a8(3, "c4tw", m, k, n, 0.005, True, 1)
    hw = htpg.w8a8_weights(_t(c.blob, gpu), k, n)
    x, b = _t(c.x, gpu), _t(c.bias, gpu)
    outs = []
    try:
        for tw in (True, False):
            htpg.set_tmem_weights(tw)
            o = torch.full((m, n), float("nan"), dtype=torch.float32, device=gpu)
            htpg.check(htpg.w8a8_run(hw, o, x, b, mode=1), "w8a8_run")
            htpg.check(htpg.check_device(), "device watchdog")
            outs.append(o)
    finally:
        htpg.set_tmem_weights(False)
    assert torch.equal(outs[0].view(torch.int32), outs[1].view(torch.int32))
    rows = np.arange(5, m, 509, dtype=np.int32)
    ref = O.w8a8_linear(c.x, c.blob, k, n, bias=c.bias, mode=1, rows=rows)
    assert O.max_abs_rel(outs[0].cpu().numpy()[rows], ref) <= W8A8_TOL
