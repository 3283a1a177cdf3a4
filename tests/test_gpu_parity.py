"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Bars: INT8 activation codes, row scales and INT32
accumulators bit-exact; W8A8 FP32 outputs within max-abs-rel 2e-3 (achieved
bit-exact without an activation); FP16-weight GEMM outputs within
max-abs-rel 1e-2 of the oracle with FP32 accumulation.
"""
import numpy as np
import pytest

import htpg
import oracle as O

W8A8_TOL = 2e-3
F16_TOL = 1e-2

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _quant_case(m, k, seed, kind="normal"):
    x = O.normal(m * k, 1.0, 0.01, 20.0, seed).reshape(m, k)
    if kind == "edges" and m >= 4:
        x[0, :] = 0.0                       # all-zero row: scale clamps to 1e-12
        x[1, :] = 1e-30                     # subnormal-scale row
        x[2, ::7] = 1.0e38                  # huge outliers (finite after x*inverse)
        x[3, :] = np.float32(-0.0)
    return x


@pytest.mark.parametrize("m,k", [(1, 32), (3, 64), (77, 768), (256, 1152), (1000, 1536),
                                 (2048, 1536), (16, 14336), (5, 4096), (9, 6144), (4096, 768),
                                 (1200, 2048), (1500, 160), (1300, 3072)])
@pytest.mark.parametrize("inverse", [False, True])
def test_quantize_rows_bitexact(gpu, lib, m, k, inverse):
    import torch
    x = _quant_case(m, k, 1000 + m + k, "edges")
    inv = O.uniform(k, 0.5, 2.0, 77) if inverse else None
    codes_ref, scales_ref = O.quantize_rows(x, inv)
    codes = torch.empty(m, k, dtype=torch.int8, device=gpu)
    scales = torch.empty(m, dtype=torch.float32, device=gpu)
    xd = _t(x, gpu)                       # keep device copies alive until the kernel ran
    invd = _t(inv, gpu) if inverse else None
    htpg.check(lib.htpg_quantize_rows(htpg.ptr(codes), htpg.ptr(scales), htpg.ptr(xd), htpg.ptr(invd),
                                      m, k, htpg.stream_ptr()), "quantize")
    torch.cuda.synchronize()
    got_codes = codes.cpu().numpy().astype(np.int16) + 128
    np.testing.assert_array_equal(got_codes, codes_ref.astype(np.int16))
    np.testing.assert_array_equal(scales.cpu().numpy().view(np.uint32), scales_ref.view(np.uint32))


W8A8_SHAPES = [  # (m, k, n): swapped (m<=32) incl. split-K, and normal tiles with ragged edges
    (1, 128, 64), (4, 256, 128), (16, 512, 192), (32, 1152, 256), (33, 256, 192),
    (77, 768, 640), (128, 128, 128), (200, 1152, 640), (256, 1152, 4608), (300, 2048, 1024),
    (4, 14336, 4096), (16, 4096, 1024),
    # CTA-pair (256-row) tiles: ragged M, BN = 128 and 256
    (1000, 512, 1280), (2048, 768, 2304), (4100, 256, 4608),
]


def _w8a8_case(m, k, n, seed=0, outliers=0.01, inverse=False, bias=False, mode=0):
    c = O.make_w8a8(seed, f"t{m}x{k}x{n}", m, k, n, outliers, bias, mode,
                    inverse_range=(0.5, 2.0) if inverse else None)
    return c


def _run_w8a8(lib, gpu, c, mode, bias=None, channels=None, raw=False):
    import torch
    channels = c.n if channels is None else channels
    blob = _t(c.blob, gpu)
    x = _t(c.x, gpu)
    if raw:
        out = torch.empty(c.m, c.n, dtype=torch.int32, device=gpu)
        mode = htpg_mode_raw = 4
    elif mode == 3:
        out = torch.full((channels, c.m), float("nan"), dtype=torch.float32, device=gpu)
    else:
        out = torch.full((c.m, c.n), float("nan"), dtype=torch.float32, device=gpu)
    b = _t(bias, gpu) if bias is not None else None
    rc = lib.htpg_w8a8_linear(htpg.ptr(out), htpg.ptr(x), htpg.ptr(blob), htpg.ptr(b), c.m, c.k, c.n,
                              channels, mode, htpg.stream_ptr())
    htpg.check(rc, "htpg_w8a8_linear")
    htpg.check(htpg.check_device(), "device watchdog")
    lib.htpg_weight_cache_drop(htpg.ptr(blob))
    return out.cpu().numpy()


@pytest.mark.parametrize("m,k,n", W8A8_SHAPES)
def test_w8a8_int32_accumulators_bitexact(gpu, lib, m, k, n):
    c = _w8a8_case(m, k, n, seed=m)
    _, codes, scales, acc = O.w8a8_linear(c.x, c.blob, k, n, want_intermediates=True)
    got = _run_w8a8(lib, gpu, c, 0, raw=True)
    np.testing.assert_array_equal(got, acc)


@pytest.mark.parametrize("m,k,n", W8A8_SHAPES)
def test_w8a8_output_bitexact_mode0(gpu, lib, m, k, n):
    c = _w8a8_case(m, k, n, seed=m + 1, inverse=(m % 2 == 1))
    ref = O.w8a8_linear(c.x, c.blob, k, n)
    got = _run_w8a8(lib, gpu, c, 0)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("m,k,n", [(4, 256, 192), (77, 768, 640), (300, 512, 256), (16, 4096, 1024),
                                   (1100, 512, 1280)])
@pytest.mark.parametrize("mode", [0, 1, 2, 3])
@pytest.mark.parametrize("with_bias", [False, True])
def test_w8a8_epilogue_modes(gpu, lib, m, k, n, mode, with_bias):
    c = _w8a8_case(m, k, n, seed=7 * m + mode, outliers=0.005)
    bias = O.normal(n, 0.01, 0, 1, 99 + n) if with_bias else None
    channels = n - 64 + 5 if mode == 3 else n   # cropped channel-major store
    ref = O.w8a8_linear(c.x, c.blob, k, n, bias=bias, channels=channels, mode=mode)
    got = _run_w8a8(lib, gpu, c, mode, bias=bias, channels=channels)
    assert not np.isnan(got).any()
    err = O.max_abs_rel(got, ref)
    assert err <= W8A8_TOL, err
    if mode in (0, 3):
        np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def _f16_case(m, k, n, seed):
    x = O.normal(m * k, 1.0, 0, 1, seed).reshape(m, k)
    w = O.f16_normal(k * n, 0.02, seed + 1).reshape(k, n)
    return x, w, O.f16_pack_permuted(w)


def _run_f16(lib, gpu, x, wperm, m, k, n, bias=None, channels=None, mode=0, raw=False):
    import torch
    channels = n if channels is None else channels
    if mode == 3:
        out = torch.full((channels, m), float("nan"), dtype=torch.float32, device=gpu)
    else:
        out = torch.full((m, n), float("nan"), dtype=torch.float32, device=gpu)
    wdev = _t(wperm.view(np.int16), gpu)
    b = _t(bias, gpu) if bias is not None else None
    xd = _t(x, gpu)
    rc = lib.htpg_f16_linear(htpg.ptr(out), htpg.ptr(xd), htpg.ptr(wdev), htpg.ptr(b), m, k, n,
                             channels, 4 if raw else mode, htpg.stream_ptr())
    htpg.check(rc, "htpg_f16_linear")
    htpg.check(htpg.check_device(), "device watchdog")
    lib.htpg_weight_cache_drop(htpg.ptr(wdev))
    return out.cpu().numpy()


@pytest.mark.parametrize("m,k,n", [(1, 32, 32), (77, 768, 3072), (128, 256, 96), (300, 1024, 512),
                                   (512, 512, 1024), (1024, 512, 1536), (2000, 256, 2048)])
def test_f16_accumulator_close_to_fp64(gpu, lib, m, k, n):
    x, w, wperm = _f16_case(m, k, n, 5 + m)
    got = _run_f16(lib, gpu, x, wperm, m, k, n, raw=True)
    x16 = x.astype(np.float16).astype(np.float64)
    w64 = w.view(np.float16).astype(np.float64)
    ref = x16 @ w64
    # FP32 accumulation of exact FP16 products over K terms
    assert O.max_abs_rel(got, ref) <= 1e-5


@pytest.mark.parametrize("m,k,n", [(77, 768, 3072), (5, 64, 96), (256, 512, 256), (1030, 256, 1536)])
@pytest.mark.parametrize("mode", [0, 1, 2, 3])
@pytest.mark.parametrize("with_bias", [False, True])
def test_f16_epilogue_modes(gpu, lib, m, k, n, mode, with_bias):
    x, w, wperm = _f16_case(m, k, n, 17 + mode)
    bias = O.normal(n, 0.01, 0, 1, 3 + n) if with_bias else None
    channels = n - 32 + 7 if mode == 3 else n
    got = _run_f16(lib, gpu, x, wperm, m, k, n, bias=bias, channels=channels, mode=mode)
    assert not np.isnan(got).any()
    for round_acc in (False, True):   # FP32 accumulator, and the HMX FP16-rounded one
        ref = O.f16_linear(x, wperm, k, n, bias=bias, channels=channels, mode=mode,
                           round_acc_f16=round_acc)
        assert O.max_abs_rel(got, ref) <= F16_TOL
    ref = O.f16_linear(x, wperm, k, n, bias=bias, channels=channels, mode=mode)
    assert O.max_abs_rel(got, ref) <= 1e-5


def test_watchdog_clear(gpu, lib):
    assert htpg.check_device() == 0


@pytest.mark.parametrize("m,mode,with_bias", [(1500, 0, False), (1500, 1, True), (300, 0, False)])
def test_w8a8_executor_host_buffers(gpu, lib, m, mode, with_bias):
    """Opcode 15 through the executor with host (pinned) buffers: from 1024 rows
    the rows go through in chunks whose copies in, GEMMs and copies out overlap
    on three streams (the last chunk ragged); below, one staged run."""
    import ctypes
    import struct
    k, n = 256, 192
    c = O.make_w8a8(7, "exec", m, k, n, 0.01, with_bias, mode)
    ref = O.w8a8_linear(c.x, c.blob, k, n, bias=c.bias if with_bias else None, mode=mode)
    fds, ptrs = {}, {}

    def alloc(name, arr):
        fd, p = ctypes.c_int(), ctypes.c_void_p()
        htpg.check(lib.htpg_buffer_alloc(arr.nbytes, htpg.BUF_HOST, ctypes.byref(fd), ctypes.byref(p)), name)
        ctypes.memmove(p.value, arr.ctypes.data, arr.nbytes)
        fds[name], ptrs[name] = fd.value, p.value

    try:
        alloc("out", np.full(m * n, np.nan, np.float32))
        alloc("x", np.ascontiguousarray(c.x))
        alloc("cst", c.blob)
        payload = struct.pack("<iiiiiiiiii", fds["out"], 0, fds["x"], 0, fds["cst"], 0, m, k, n, 0)
        if with_bias:
            alloc("bias", np.ascontiguousarray(c.bias))
            payload += struct.pack("<iiii", fds["bias"], 0, n, mode)
        req = np.frombuffer(struct.pack("<I", 15) + payload, np.uint8).copy()
        assert lib.execute_op_simple(req.ctypes.data, req.nbytes) == 0
        got = np.empty(m * n, np.float32)
        ctypes.memmove(got.ctypes.data, ptrs["out"], got.nbytes)
        got = got.reshape(m, n)
        if mode == 0:
            np.testing.assert_array_equal(got, ref)
        else:
            assert O.max_abs_rel(got, ref) <= W8A8_TOL
    finally:
        for fd in fds.values():
            lib.htpg_buffer_release(fd)


# Register-fed decode kernel (M <= 16): ragged K (k-blocks with 32/64/96 valid
# bytes), odd M (1..16 with 8 or 16 rows held), column groups that straddle
# work chunks (small and large K relative to N), and N from 64 to 16384.
DECODE_SHAPES = [(1, 32, 64), (2, 96, 64), (8, 160, 128), (9, 14336, 4096), (13, 14336, 4096),
                 (16, 16384, 1536), (5, 1024, 16384), (3, 224, 4608), (11, 6144, 192), (4, 4096, 14336)]


@pytest.mark.parametrize("m,k,n", DECODE_SHAPES)
def test_decode_int32_and_output_bitexact(gpu, lib, m, k, n):
    plan = htpg.plan_info(0, m, n, k)
    assert plan["swap"] == 2                       # the register-fed decode kernel
    # (shapes with M > 8 here all take a K-split swapped plan otherwise)
    c = _w8a8_case(m, k, n, seed=3 * m + k, inverse=(m % 2 == 0))
    _, codes, scales, acc = O.w8a8_linear(c.x, c.blob, k, n, want_intermediates=True)
    np.testing.assert_array_equal(_run_w8a8(lib, gpu, c, 0, raw=True), acc)
    ref = O.w8a8_linear(c.x, c.blob, k, n)
    got = _run_w8a8(lib, gpu, c, 0)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("m,k,n", [(1, 4096, 14336), (16, 14336, 4096), (7, 1152, 4608)])
@pytest.mark.parametrize("mode,with_bias", [(0, False), (1, True), (2, False), (3, True)])
def test_decode_kernels_give_identical_bits(gpu, lib, m, k, n, mode, with_bias):
    """The register-fed decode kernel and the swapped tcgen05 kernel share the
    epilogue and sum INT32 exactly: their outputs agree bit for bit."""
    c = _w8a8_case(m, k, n, seed=m + mode, outliers=0.005)
    bias = O.normal(n, 0.01, 0, 1, 5 + n) if with_bias else None
    channels = n - 64 + 5 if mode == 3 else n
    outs = []
    try:
        for which in (0, 1):
            htpg.set_decode_kernel(which)
            outs.append(_run_w8a8(lib, gpu, c, mode, bias=bias, channels=channels))
    finally:
        htpg.set_decode_kernel(0)
    assert not np.isnan(outs[0]).any()
    np.testing.assert_array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))
    ref = O.w8a8_linear(c.x, c.blob, k, n, bias=bias, channels=channels, mode=mode)
    assert O.max_abs_rel(outs[0], ref) <= W8A8_TOL
