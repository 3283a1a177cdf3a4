"""htpg_w8a8_run_static: the W8A8 run whose scratch is a fixed static device
array, called through the C ABI.  Each case runs twice in a row on the
allocation-free entry point and is compared with htpg_w8a8_run (the workspace
path), which runs the same kernels on the same inputs: the outputs must be
bit-identical (the W8A8 output tolerance, max-abs-rel 2e-3, is checked
against the oracle on sampled rows as well).  The shapes cover the swapped
split-K, register-fed decode, single-CTA, CTA-pair and channel-major plans,
interleaved so that every call starts from the array contents another shape
left.  While the static calls run on a stream the workspace path never saw,
nothing may be allocated: free device memory, torch's allocator counters and
the library's own stream workspaces must all stay as they were after a
warm-up pass.  Collected last so it also runs after every other GPU test in
one process.
"""
import ctypes

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
    (4, 14336, 512, 0, True, 0, False),       # register-fed decode, deep K split across many CTAs
    (24, 6144, 1536, 0, False, 0, False),     # swapped orientation, M between 16 and 32
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
    t["shape"] = shape
    return t


def _static(t, out, mode, channels, stream):
    L = htpg.lib()
    return L.htpg_w8a8_run_static(t["w"].handle, htpg.ptr(out), 0, htpg.ptr(t["x"]), htpg.ptr(t["bias"]),
                                  t["x"].shape[0], channels, mode, htpg.stream_ptr(stream))


def _workspace_bytes():
    ws, qws = ctypes.c_size_t(), ctypes.c_size_t()
    htpg.check(htpg.lib().htpg_debug_workspaces(ctypes.byref(ws), ctypes.byref(qws)), "htpg_debug_workspaces")
    return ws.value, qws.value


def _alloc_state():
    st = torch.cuda.memory_stats()
    return (st.get("allocation.all.allocated", 0), st.get("segment.all.allocated", 0),
            torch.cuda.memory_reserved(), _workspace_bytes())


def test_static_scratch_matches_workspace_path(gpu):
    cases = [_case(i, *c) for i, c in enumerate(CASES)]
    for t, (m, k, n, mode, bias, ch, inv) in zip(cases, CASES):
        htpg.check(htpg.w8a8_run(t["w"], t["ref"], t["x"], t["bias"], channels=ch, mode=mode), "htpg_w8a8_run")
    torch.cuda.synchronize()

    side = torch.cuda.Stream()
    order = [0, 4, 1, 3, 2, 5, 6, 0]   # every call starts from another shape's leftovers
    dev = torch.device("cuda:0")
    # every output buffer exists before the measured region (two calls in a row per entry)
    outs = [[torch.full(cases[i]["shape"], float("nan"), device=dev) for _ in range(2)] for i in order]
    warm = [torch.empty(t["shape"], device=dev) for t in cases]
    torch.cuda.synchronize()
    # warm-up pass: the first call on this device does the array's set-up, and
    # every plan's kernel gets its attributes (and, with lazy module loading,
    # its module) on its first use
    for i, t in enumerate(cases):
        htpg.check(_static(t, warm[i], CASES[i][3], CASES[i][5], side), f"warm-up case {i}")
    side.synchronize()
    free0, state0 = torch.cuda.mem_get_info()[0], _alloc_state()
    for j, i in enumerate(order):
        t, (m, k, n, mode, bias, ch, inv) = cases[i], CASES[i]
        for rep in range(2):        # two calls in a row
            htpg.check(_static(t, outs[j][rep], mode, ch, side), f"static case {i} call {rep}")
    side.synchronize()
    free1, state1 = torch.cuda.mem_get_info()[0], _alloc_state()
    assert abs(free0 - free1) <= (1 << 20), (free0, free1)
    assert state0 == state1, (state0, state1)
    htpg.check(htpg.check_device(), "watchdog")

    for j, i in enumerate(order):
        for rep in range(2):
            assert torch.equal(outs[j][rep].view(torch.int32), cases[i]["ref"].view(torch.int32)), (CASES[i], rep)
    for i, t in enumerate(cases):
        m, k, n, mode, bias, ch, inv = CASES[i]
        assert torch.isfinite(t["ref"]).all()
        c = O.make_w8a8(7, f"static{i}", m, k, n, 0.01, bias, mode,
                        inverse_range=(0.5, 2.0) if inv else None)
        rows = np.arange(0, m, max(1, m // 7), dtype=np.int32)
        ref = O.w8a8_linear(c.x, c.blob, k, n, bias=c.bias, channels=ch or n, mode=mode, rows=rows)
        got = t["ref"].cpu().numpy()
        got = got[:, rows] if mode == 3 else got[rows]
        assert O.max_abs_rel(got, ref) <= W8A8_TOL, CASES[i]


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
