"""Opcode 19 (FP32 model auxiliaries) on the GPU against the oracle, every
mode, through the device ABI and the executor.  The norms reduce in a
different order (FP32 partial sums per thread, FP64 block sums): outputs agree
within 2e-5 of the tensor's absolute maximum; the activations use the
reference's stable sigmoid and agree to a few ulp."""
import ctypes
import struct

import numpy as np
import pytest
import torch

import htpg
import oracle as O
from test_oracle_kat import aux_cases

pytestmark = pytest.mark.gpu


def _run(lib, gpu, prm, x, w, b, eps=1e-6):
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(gpu)
    xd, wd, bd = t(x), t(w), t(b)
    out = torch.full((prm["count"],), float("nan"), device=gpu)
    p = (ctypes.c_uint8 * 76).from_buffer_copy(htpg.aux_params_bytes(prm, eps))
    rc = lib.hvx_model_aux_f32(htpg.ptr(out), htpg.ptr(xd), htpg.ptr(wd), htpg.ptr(bd), p)
    assert rc == 0, rc
    return out.cpu().numpy()


@pytest.mark.parametrize("case", aux_cases(), ids=lambda c: c[0])
def test_model_aux_matches_oracle(gpu, lib, case):
    name, prm, x, w, b, _ = case
    got = _run(lib, gpu, prm, x, w, b)
    ref = O.model_aux(x, w, b, prm)
    assert np.isfinite(got).all()
    assert np.max(np.abs(got - ref)) <= 2e-5 * max(1.0, np.max(np.abs(ref))), name


def test_model_aux_dit_shapes(gpu, lib):
    """DiT-sized rows: LayerNorm + modulation over 4096 tokens x 1536, GroupNorm
    over a 512-channel 64x64 image, SwiGLU over 4096 x 6144."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 4096, 1536)).astype(np.float32)
    w, b = rng.standard_normal((2, 1536)).astype(np.float32), rng.standard_normal((2, 1536)).astype(np.float32)
    prm = dict(mode=9, count=x.size, width=1536, channels=1, spatial=4096, groups=1, batch=2, other_count=3072,
               activation=0)
    got, ref = _run(lib, gpu, prm, x, w, b), O.model_aux(x, w, b, prm, kind="omp")
    assert np.max(np.abs(got - ref)) <= 2e-5 * np.max(np.abs(ref))
    x = rng.standard_normal((1, 512, 64, 64)).astype(np.float32)
    w, b = rng.standard_normal(512).astype(np.float32), rng.standard_normal(512).astype(np.float32)
    prm = dict(mode=2, count=x.size, width=1, channels=512, spatial=4096, groups=32, batch=1, other_count=512,
               activation=1)
    got, ref = _run(lib, gpu, prm, x, w, b), O.model_aux(x, w, b, prm, kind="omp")
    assert np.max(np.abs(got - ref)) <= 2e-5 * np.max(np.abs(ref))
    x = rng.standard_normal((4096, 12288)).astype(np.float32)
    prm = dict(mode=12, count=4096 * 6144, width=6144, channels=12288, spatial=4096, groups=1, batch=1,
               other_count=0, activation=0)
    got, ref = _run(lib, gpu, prm, x, None, None), O.model_aux(x, None, None, prm, kind="omp")
    assert np.max(np.abs(got - ref)) <= 2e-5 * np.max(np.abs(ref))


def test_model_aux_through_executor(gpu, lib):
    name, prm, x, w, b, _ = [c for c in aux_cases() if c[0] == "modulate0"][0]
    ref = O.model_aux(x, w, b, prm)
    fds, ptrs = {}, {}

    def alloc(key, arr):
        arr = np.ascontiguousarray(arr, np.float32)
        fd, p = ctypes.c_int(), ctypes.c_void_p()
        htpg.check(lib.htpg_buffer_alloc(arr.nbytes, htpg.BUF_HOST, ctypes.byref(fd), ctypes.byref(p)), key)
        ctypes.memmove(p.value, arr.ctypes.data, arr.nbytes)
        fds[key], ptrs[key] = fd.value, p.value

    try:
        alloc("out", np.zeros(prm["count"]))
        alloc("x", x)
        alloc("w", w)
        alloc("b", b)
        payload = htpg.aux_params_bytes(prm, 1e-6, (fds["out"], 0), (fds["x"], 0), (fds["w"], 0), (fds["b"], 0))
        req = np.frombuffer(struct.pack("<I", 19) + payload, np.uint8).copy()
        assert lib.execute_op_simple(req.ctypes.data, req.nbytes) == 0
        got = np.empty(prm["count"], np.float32)
        ctypes.memmove(got.ctypes.data, ptrs["out"], got.nbytes)
        assert np.max(np.abs(got - ref)) <= 2e-5 * max(1.0, np.max(np.abs(ref)))
    finally:
        for fd in fds.values():
            lib.htpg_buffer_release(fd)
