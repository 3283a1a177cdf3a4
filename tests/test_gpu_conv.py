"""Opcode 17 (packed-FP16 NCHW convolution) on the GPU against the oracle.

The device runs im2col (FP16, round to nearest) and the FP16 GEMM with FP32
accumulation and the channel-major epilogue; the oracle restates the
reference's gather and GEMM (mat_mul.c:2189-2343).  Tolerances: within 1e-5
max-abs-rel of the FP32-accumulating oracle (same products, different summation
order) and within the 1e-2 FP16 bar of the FP16-rounded-accumulator variant.
"""
import ctypes
import struct

import numpy as np
import pytest
import torch

import htpg
import oracle as O

pytestmark = pytest.mark.gpu

GEOMS = [
    dict(iw=9, ih=7, ic=3, oc=5),
    dict(iw=6, ih=5, ic=4, oc=40, upscale=2),
    dict(iw=11, ih=9, ic=2, oc=8, sx=2, sy=2, px=0, py=0),
    dict(iw=10, ih=8, ic=3, oc=7, dx=2, dy=2, px=2, py=2),
    dict(iw=5, ih=4, ic=33, oc=9, kw=1, kh=1, px=0, py=0, batch=2),
    dict(iw=32, ih=32, ic=64, oc=64, batch=2),                 # VAE-like 3x3
    dict(iw=16, ih=16, ic=32, oc=96, upscale=2),               # upsample block
    dict(iw=40, ih=24, ic=16, oc=128, kw=5, kh=5, px=2, py=2),
]


def _rel(a, b):
    return float(np.max(np.abs(a.astype(np.float64) - b)) / max(np.max(np.abs(b)), 1e-30))


def _struct(prm):
    return (ctypes.c_uint8 * 124).from_buffer_copy(htpg.conv_params_bytes(prm))


@pytest.mark.parametrize("geom", GEOMS)
def test_conv_matches_oracle(gpu, lib, geom):
    prm = O.conv_params(**geom)
    x, _, wperm, bias = O.conv_case(31 + geom["ic"], prm)
    ref32 = O.conv2d(x, wperm, bias, prm, kind="omp")
    ref16 = O.conv2d(x, wperm, bias, prm, round_acc_f16=True, kind="omp")
    xd = torch.from_numpy(x).to(gpu)
    wd = torch.from_numpy(wperm.view(np.int16)).to(gpu)
    bd = torch.from_numpy(bias).to(gpu)
    out = torch.full(ref32.shape, float("nan"), device=gpu)
    p = _struct(prm)
    try:
        rc = lib.hmx_conv2d_nchw_f16(htpg.ptr(out), htpg.ptr(xd), htpg.ptr(wd), htpg.ptr(bd), p)
    finally:
        # the one-call entry points cache the repacked weight by address; the
        # allocator may hand this address to the next test's weight
        lib.htpg_weight_cache_drop(htpg.ptr(wd))
    assert rc == 0, (rc, lib.htpg_last_cuda_error())
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert _rel(got, ref32) <= 1e-5
    assert _rel(got, ref16) <= 1e-2
    gather_us, weight_us, hmx_us, store_us = struct.unpack_from("<4i", bytes(p), 108)
    assert hmx_us > 0 and store_us == 0


def test_conv_chunked_rows(gpu, lib):
    """Output rows split over several GEMM launches (small staging budget)."""
    prm = O.conv_params(iw=24, ih=20, ic=8, oc=24, batch=2)
    x, _, wperm, bias = O.conv_case(5, prm)
    ref = O.conv2d(x, wperm, bias, prm, kind="omp")
    w = htpg.f16_weights(torch.from_numpy(wperm.view(np.int16)).to(gpu), prm["kp"], prm["np"])
    xd, bd = torch.from_numpy(x).to(gpu), torch.from_numpy(bias).to(gpu)
    out = torch.full(ref.shape, float("nan"), device=gpu)
    try:
        htpg.check(lib.htpg_conv_set_chunk_bytes(128 * prm["kp"] * 2), "chunk")   # 128 rows per launch
        htpg.check(lib.htpg_conv2d_run(w.handle, htpg.ptr(out), htpg.ptr(xd), htpg.ptr(bd), _struct(prm),
                                       htpg.stream_ptr()), "htpg_conv2d_run")
        torch.cuda.synchronize()
    finally:
        lib.htpg_conv_set_chunk_bytes(256 << 20)
    assert _rel(out.cpu().numpy(), ref) <= 1e-5


def test_conv_through_executor(gpu, lib):
    prm = O.conv_params(iw=12, ih=10, ic=6, oc=20, upscale=2)
    x, _, wperm, bias = O.conv_case(9, prm)
    ref = O.conv2d(x, wperm, bias, prm, kind="omp")
    fds, ptrs = {}, {}

    def alloc(name, arr):
        fd, p = ctypes.c_int(), ctypes.c_void_p()
        htpg.check(lib.htpg_buffer_alloc(arr.nbytes, htpg.BUF_HOST, ctypes.byref(fd), ctypes.byref(p)), name)
        ctypes.memmove(p.value, arr.ctypes.data, arr.nbytes)
        fds[name], ptrs[name] = fd.value, p.value

    try:
        alloc("out", np.zeros(ref.size, np.float32))
        alloc("x", np.ascontiguousarray(x))
        alloc("w", wperm)
        alloc("b", bias)
        payload = htpg.conv_params_bytes(prm, (fds["out"], 0), (fds["x"], 0), (fds["w"], 0), (fds["b"], 0))
        req = np.frombuffer(struct.pack("<I", 17) + payload, np.uint8).copy()
        assert lib.execute_op_simple(req.ctypes.data, req.nbytes) == 0
        got = np.empty(ref.size, np.float32)
        ctypes.memmove(got.ctypes.data, ptrs["out"], got.nbytes)
        assert _rel(got.reshape(ref.shape), ref) <= 1e-5
        elapsed = struct.unpack_from("<i", req.tobytes(), 4 + 104)[0]
        assert elapsed > 0
    finally:
        for fd in fds.values():
            lib.htpg_buffer_release(fd)
