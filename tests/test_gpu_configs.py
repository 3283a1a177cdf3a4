"""Parity at the exact benchmark configurations, every row checked.

The five configurations of the benchmark (C1 single W8A8 linear, C2 CLIP fc1
through the FP16 GEMM + QuickGELU, C3 the four DiT linears at M=4096 -- exact
(4096, k, n) entries of the reference's plan table,
linear_w8a8_allocation_table.h:26-29 --, C4 the M=16384 fc1 + GELU and C5 the
six decode linears) run through the C ABI on their seeded inputs and are
compared with the OpenMP build of the oracle on all rows.  They put the
kernels the benchmark times under test at the benchmark's own shapes: the
CTA-pair GEMM with 256-column tiles at K=1536 and K=6144, the swapped and
register-fed decode kernels at K=4096 and K=14336.

Bars: INT32 accumulators (HTPG_MODE_RAW) bit-exact; mode-0 outputs (with or
without bias) bit-exact; GELU / QuickGELU outputs within max-abs-rel 2e-3
(W8A8) and 1e-2 (FP16 weights; within 1e-5 of the FP32-accumulating oracle).
"""
import os

import numpy as np
import pytest

import htpg
import oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

W8A8_TOL = 2e-3
F16_TOL = 1e-2


@pytest.fixture(scope="module", autouse=True)
def _oracle_threads():
    O.lib("omp").orc_set_threads(max(1, os.cpu_count() or 1))


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _run(gpu, c, mode, raw=False):
    """Opcode-15 arithmetic on prepared weights: returns the output (or the raw
    INT32 accumulators) as a numpy array."""
    import torch
    w = htpg.w8a8_weights(_t(c.blob, gpu), c.k, c.n)
    x = _t(c.x, gpu)
    b = _t(c.bias, gpu) if c.bias is not None else None
    if raw:
        out = torch.empty(c.m, c.n, dtype=torch.int32, device=gpu)
        htpg.check(htpg.w8a8_run(w, out, x, None, mode=4), "raw run")
    else:
        out = torch.full((c.m, c.n), float("nan"), device=gpu)
        htpg.check(htpg.w8a8_run(w, out, x, b, mode=mode), "run")
    htpg.check(htpg.check_device(), "device watchdog")
    return out.cpu().numpy()


def _check_w8a8(gpu, c):
    ref, _, _, acc = O.w8a8_linear(c.x, c.blob, c.k, c.n, bias=c.bias, mode=c.mode, kind="omp",
                                   want_intermediates=True)
    np.testing.assert_array_equal(_run(gpu, c, c.mode, raw=True), acc)
    got = _run(gpu, c, c.mode)
    assert not np.isnan(got).any()
    if c.mode == 0:
        np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
    else:
        assert O.max_abs_rel(got, ref) <= W8A8_TOL


def test_c1(gpu):
    _check_w8a8(gpu, O.config_c1())


def test_c1_with_inverse(gpu):
    _check_w8a8(gpu, O.config_c1(inverse=True))


def test_c2(gpu, lib):
    import torch
    c = O.config_c2()
    out = torch.full((c.m, c.n), float("nan"), device=gpu)
    wd, xd, bd = _t(c.wperm.view(np.int16), gpu), _t(c.x, gpu), _t(c.bias, gpu)
    htpg.check(lib.htpg_f16_linear(htpg.ptr(out), htpg.ptr(xd), htpg.ptr(wd), htpg.ptr(bd), c.m, c.k, c.n,
                                   c.n, c.mode, htpg.stream_ptr()), "htpg_f16_linear")
    htpg.check(htpg.check_device(), "device watchdog")
    lib.htpg_weight_cache_drop(htpg.ptr(wd))
    got = out.cpu().numpy()
    for round_acc in (False, True):
        ref = O.f16_linear(c.x, c.wperm, c.k, c.n, bias=c.bias, mode=c.mode, round_acc_f16=round_acc, kind="omp")
        assert O.max_abs_rel(got, ref) <= (1e-5 if not round_acc else F16_TOL)


@pytest.mark.parametrize("layer", [0, 1, 2, 3], ids=[name for name, *_ in O.C3_LAYERS])
def test_c3_dit_linears(gpu, layer):
    c = O.config_c3()[layer]
    plan = htpg.plan_info(0, c.m, c.n, c.k)
    assert plan["swap"] in (0, 3) and c.m == 4096     # CTA-pair tiles, either orientation
    _check_w8a8(gpu, c)


def test_c4_every_row(gpu):
    c = O.config_c4()
    plan = htpg.plan_info(0, c.m, c.n, c.k)
    assert plan["swap"] == 3 and plan["bn"] == 256    # 256 x 256 CTA-pair tiles, swapped orientation
    _check_w8a8(gpu, c)


@pytest.mark.parametrize("i", range(6), ids=["up_m1", "up_m4", "up_m16", "down_m1", "down_m4", "down_m16"])
def test_c5_decode(gpu, i):
    _check_w8a8(gpu, O.config_c5()[i])
