"""htpg_w8a8_run_static: the W8A8 run whose scratch is a fixed static device
array, called through the C ABI.  Each case runs twice in a row on the
allocation-free entry point and is compared with htpg_w8a8_run (the workspace
path) within the W8A8 output tolerance; the shapes cover the swapped split-K,
single-CTA, CTA-pair and channel-major plans, interleaved so that every call
starts from the array contents another shape left.  Free device memory must
not move while the static calls run on a stream the workspace path never saw.
Collected last so it also runs after every other GPU test in one process.
"""

import numpy as np
import pytest
import torch

import htpg
import oracle as O

pytestmark = pytest.mark.gpu

W8A8_TOL = 2e-3  # max-abs-rel bound of the W8A8 FP32 outputs

# (m, k, n, mode, bias, channels, inverse)
CASES = [
    (16, 4096, 1024, 0, False, 0, True),      # swapped orientation, exact INT32 split-K
    (300, 512, 640, 1, True, 0, False),       # 128-row tiles, bias + GELU
    (1000, 512, 1280, 2, True, 0, True),      # CTA-pair tiles, bias + QuickGELU
    (64, 256, 512, 3, True, 448, False),      # channel-major output, 448 channels
    (8192, 1536, 1024, 1, True, 0, False),    # 12.6 MB of activation codes
    (4, 14336, 512, 0, True, 0, False),       # deep K split across many CTAs
]


def _case(i, m, k, n, mode, bias, channels, inverse):
    c = O.make_w8a8(7, f"static{i}", m, k, n, 0.01, bias, mode,
                    inverse_range=(0.5, 2.0) if inverse else None)
    dev = torch.device("cuda:0")
    t = {
        "x": torch.from_numpy(c.x).to(dev),
        "blob": torch.from_numpy(c.blob).to(dev),
        "bias": torch.from_numpy(c.bias).to(dev) if bias else None,
    }
    t["w"] = htpg.w8a8_weights(t["blob"], k, n)
    shape = (channels, m) if mode == 3 else (m, n)
    t["ref"] = torch.full(shape, float("nan"), device=dev)
    t["out"] = [torch.full(shape, float("nan"), device=dev) for _ in range(2)]
    return t


def _static(t, out, mode, channels, stream):
    L = htpg.lib()
    return L.htpg_w8a8_run_static(t["w"].handle, htpg.ptr(out), 0, htpg.ptr(t["x"]), htpg.ptr(t["bias"]),
                                  t["x"].shape[0], channels, mode, htpg.stream_ptr(stream))


def _max_abs_rel(a, b):
    a = a.double()
    b = b.double()
    return float(((a - b).abs() / b.abs().clamp_min(1.0)).max())


def test_static_scratch_matches_workspace_path(gpu):
    cases = [_case(i, *c) for i, c in enumerate(CASES)]
    for t, (m, k, n, mode, bias, ch, inv) in zip(cases, CASES):
        htpg.check(htpg.w8a8_run(t["w"], t["ref"], t["x"], t["bias"], channels=ch, mode=mode), "htpg_w8a8_run")
    torch.cuda.synchronize()

    side = torch.cuda.Stream()
    # first call on this device: the one-time set-up of the static array
    htpg.check(_static(cases[1], cases[1]["out"][0], CASES[1][3], CASES[1][5], side), "set-up call")
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    order = [0, 4, 1, 3, 2, 5, 0]   # every call starts from another shape's leftovers
    for i in order:
        t, (m, k, n, mode, bias, ch, inv) = cases[i], CASES[i]
        for rep in range(2):        # two calls in a row
            htpg.check(_static(t, t["out"][rep], mode, ch, side), f"static case {i} call {rep}")
    side.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert abs(free0 - free1) < (4 << 20), (free0, free1)
    htpg.check(htpg.check_device(), "watchdog")

    for i, t in enumerate(cases):
        assert torch.isfinite(t["ref"]).all()
        for rep in range(2):
            assert torch.isfinite(t["out"][rep]).all(), (i, rep)
            err = _max_abs_rel(t["out"][rep], t["ref"])
            assert err <= W8A8_TOL, (CASES[i], rep, err)


def test_static_scratch_refuses_oversize(gpu):
    dev = torch.device("cuda:0")
    m, k, n = 16384, 2048, 256      # 33.5 MB of codes: more than the 32 MiB array
    x = torch.zeros(m, k, device=dev)
    w_int = np.ones((n, k), np.int8)
    blob = torch.from_numpy(O.w8a8_pack(w_int, np.full(n, 1e-3, np.float32), None)).to(dev)
    w = htpg.w8a8_weights(blob, k, n)
    out = torch.full((m, n), 7.0, device=dev)
    rc = htpg.lib().htpg_w8a8_run_static(w.handle, htpg.ptr(out), 0, htpg.ptr(x), None, m, 0, 0,
                                         htpg.stream_ptr(None))
    assert rc == htpg.ESCRATCH
    assert b"static scratch" in htpg.lib().htpg_last_cuda_error()
    assert htpg.lib().htpg_strerror(rc) == b"request does not fit the static scratch array"
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())  # nothing launched
    # the largest documented shape, M=16384 at K=1536, fits
    x2 = x[:, :1536].contiguous()
    blob2 = torch.from_numpy(O.w8a8_pack(w_int[:, :1536].copy(), np.full(n, 1e-3, np.float32), None)).to(dev)
    w2 = htpg.w8a8_weights(blob2, 1536, n)
    htpg.check(htpg.lib().htpg_w8a8_run_static(w2.handle, htpg.ptr(out), 0, htpg.ptr(x2), None, m, 0, 0,
                                               htpg.stream_ptr(None)), "M=16384 K=1536")
    torch.cuda.synchronize()
    assert bool((out == 0.0).all())
    assert htpg.lib().htpg_w8a8_run_static(None, htpg.ptr(out), 0, htpg.ptr(x2), None, m, 0, 0, None) \
        == htpg.EARGS
