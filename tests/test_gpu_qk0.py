"""Opcodes 2-4 (ggml-block weights: Q4_0, Q8_0, IQ4_NL) on the GPU.

The dequantised FP16 weight is bit-exact against the oracle's restatement of
the reference's super-block decode (mat_mul.c:389-525).  The GEMM output is
checked against the oracle's FP32-accumulating GEMM of the same FP16 operands
(1e-5 max-abs-rel: same products, different summation order) and against the
variant that reads the accumulator through FP16 as the reference's HMX readout
does (the 1e-2 FP16 bar).  M <= 32 runs on both small-M kernels: the
register-fed decode kernel and the fused tcgen05 kernel (stream-K over the
CTAs; the shapes below give tiles finished by one CTA, by several CTAs and
CTAs that span tiles), the default being the faster one; larger M
dequantises once and runs the FP16 GEMM.
"""
import ctypes
import struct

import numpy as np
import pytest
import torch

import htpg
import oracle as O

pytestmark = pytest.mark.gpu

TYPES = [O.GGML_Q4_0, O.GGML_Q8_0, O.GGML_IQ4_NL]

CASES = [
    # (m, k, n)
    (1, 64, 128),
    (5, 96, 160),        # K % 64 = 32, N % 128 = 32
    (16, 4096, 128),     # one tile shared by many CTAs
    (17, 512, 384),      # 32-row activation tiles, ragged M
    (32, 1024, 4096),
    (3, 14336, 4096),    # LLM down projection shape
    (8, 4096, 14336),    # LLM up projection shape
    (4, 64, 4096),       # one k-block per tile: every iteration is its own accumulator piece
    (2, 128, 2048),      # two k-blocks per tile: commit groups split at piece starts
    (33, 128, 256),      # large-M path from here on
    (77, 768, 3072),
    (256, 512, 1024),
]


def _rel(a, b):
    return float(np.max(np.abs(a.astype(np.float64) - b)) / max(np.max(np.abs(b)), 1e-30))


def _case(wtype, m, k, n, seed):
    src = O.qk0_random(wtype, k, n, seed=seed)
    x = O.normal(m * k, 1.0, outlier_p=0.01, outlier_scale=20.0, seed=seed + 1).reshape(m, k)
    return src, x


@pytest.mark.parametrize("wtype", TYPES)
@pytest.mark.parametrize("m,k,n", CASES)
def test_qk0_linear_matches_oracle(gpu, lib, wtype, m, k, n):
    src, x = _case(wtype, m, k, n, seed=m * 7 + k + n + wtype)
    ref32 = O.qk0_linear(x, src, wtype, k, n, kind="omp")
    ref16 = O.qk0_linear(x, src, wtype, k, n, round_acc_f16=True, kind="omp")
    wd = torch.from_numpy(src).to(gpu)
    xd = torch.from_numpy(x).to(gpu)
    outs = []
    try:
        for which in ((0, 1, 2) if m <= 32 else (0,)):   # default, tcgen05, register-fed for m <= 32
            htpg.set_qk0_decode(which)
            out = torch.full((m, n), float("nan"), device=gpu)
            htpg.check(htpg.qk0_linear(out, xd, wd, wtype, m, k, n), "htpg_qk0_linear")
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy())
    finally:
        htpg.set_qk0_decode(0)
        # the one-call entry point caches the prepared weight by address; the
        # allocator may hand this address to the next test's weight
        lib.htpg_weight_cache_drop(htpg.ptr(wd))
    assert htpg.check_device() == 0
    for got in outs:
        assert np.isfinite(got).all()
        assert _rel(got, ref32) <= 1e-5
        assert _rel(got, ref16) <= 1e-2


DECODE_CASES = [  # (m, k, n) for the register-fed decode kernel (m <= 16)
    (1, 32, 64),         # one k-tile, two column tiles
    (5, 96, 160),        # odd number of k-tiles (record padding), N % 128 = 32
    (8, 4096, 14336),    # LLM up projection
    (12, 2048, 1536),    # two 8-token MMA tiles, ragged M
    (16, 14336, 4096),   # LLM down projection, 16 tokens (Q8_0)
    (2, 8192, 96),       # few column tiles: many k ranges per tile
    (4, 14336, 4096),    # LLM down projection, 4 tokens
    (24, 4096, 2048),    # four 8-token MMA tiles, ragged M
    (32, 14336, 4096),   # LLM down projection, 32 tokens
]


@pytest.mark.parametrize("wtype", TYPES)
@pytest.mark.parametrize("m,k,n", DECODE_CASES)
def test_qk0_decode_kernels_agree(gpu, lib, wtype, m, k, n):
    """The register-fed decode kernel and the tcgen05 kernel decode the same
    FP16 weights and activations and accumulate in FP32 in different orders:
    both within 1e-5 of the FP32-accumulating oracle and of each other (every
    type, up to 32 rows, whichever kernel the library would pick)."""
    src, x = _case(wtype, m, k, n, seed=m * 11 + k + n + wtype)
    ref32 = O.qk0_linear(x, src, wtype, k, n, kind="omp")
    wd, xd = torch.from_numpy(src).to(gpu), torch.from_numpy(x).to(gpu)
    w = htpg.qk0_weights(wd, wtype, k, n)
    outs = []
    try:
        for which in (2, 1):       # register-fed for every m <= 32, then tcgen05
            htpg.set_qk0_decode(which)
            out = torch.full((m, n), float("nan"), device=gpu)
            htpg.check(htpg.qk0_run(w, out, xd, m), "htpg_qk0_run")
            assert htpg.check_device() == 0
            outs.append(out.cpu().numpy())
    finally:
        htpg.set_qk0_decode(0)
    for got in outs:
        assert np.isfinite(got).all()
        assert _rel(got, ref32) <= 1e-5
    assert _rel(outs[0], outs[1].astype(np.float64)) <= 1e-5


SHAPE_CASES = [  # (m, k, n) run under every launch shape of the register-fed kernel
    (5, 96, 160),        # three k-tiles: more warps than k-tiles in narrow shapes
    (12, 2048, 1536),    # two 8-token MMA tiles, ragged M
    (16, 14336, 4096),   # LLM down projection: the slice bounds the k ranges
    (1, 4096, 1024),
    (29, 2048, 1024),    # four 8-token MMA tiles, ragged M
]


@pytest.mark.parametrize("wtype", TYPES)
@pytest.mark.parametrize("m,k,n", SHAPE_CASES)
def test_qk0_decode_every_launch_shape(gpu, lib, wtype, m, k, n):
    """Every launch shape of the register-fed kernel (one or two CTAs per SM x
    16, 8 or 4 weight tiles per CTA) that fits the problem gives results
    within 1e-5 of the oracle, bit-identical on a rerun; a shape that does not
    fit (Q8_0's rings leave no room for two CTAs per SM) is refused with
    HTPG_ENOPLAN, by the plan query and by the run."""
    src, x = _case(wtype, m, k, n, seed=m * 13 + k + n + wtype)
    ref32 = O.qk0_linear(x, src, wtype, k, n, kind="omp")
    wd, xd = torch.from_numpy(src).to(gpu), torch.from_numpy(x).to(gpu)
    w = htpg.qk0_weights(wd, wtype, k, n)
    ran = 0
    try:
        htpg.set_qk0_decode(2)
        for per_sm in (1, 2):
            for tiles in (16, 8, 4):
                htpg.set_qdec_shape(per_sm, tiles)
                out = torch.full((m, n), float("nan"), device=gpu)
                plan = (ctypes.c_int64 * 8)()
                rc = lib.htpg_qk0_decode_plan_info(wtype, m, n, k, 148, plan)
                if rc == htpg.ENOPLAN:
                    assert wtype == O.GGML_Q8_0 and per_sm == 2
                    assert htpg.qk0_run(w, out, xd, m) == htpg.ENOPLAN
                    continue
                htpg.check(rc, "htpg_qk0_decode_plan_info")
                assert (plan[0], plan[1]) == (per_sm, tiles)
                htpg.check(htpg.qk0_run(w, out, xd, m), "htpg_qk0_run")
                again = torch.full((m, n), float("nan"), device=gpu)
                htpg.check(htpg.qk0_run(w, again, xd, m), "htpg_qk0_run")
                assert htpg.check_device() == 0
                got = out.cpu().numpy()
                assert np.isfinite(got).all(), (per_sm, tiles)
                assert _rel(got, ref32) <= 1e-5, (per_sm, tiles)
                assert np.array_equal(got, again.cpu().numpy()), (per_sm, tiles)
                ran += 1
    finally:
        htpg.set_qdec_shape(0, 0)
        htpg.set_qk0_decode(0)
    assert ran == (3 if wtype == O.GGML_Q8_0 else 6)


@pytest.mark.parametrize("wtype", TYPES)
def test_qk0_repeated_runs_are_identical(gpu, lib, wtype):
    """Both small-M kernels sum their partial tiles (k ranges of the
    register-fed kernel, stream-K pieces of the tcgen05 kernel) in a fixed
    order: bit-identical reruns."""
    m, k, n = 16, 8192, 256
    src, x = _case(wtype, m, k, n, seed=5)
    wd, xd = torch.from_numpy(src).to(gpu), torch.from_numpy(x).to(gpu)
    w = htpg.qk0_weights(wd, wtype, k, n)
    ref = O.qk0_linear(x, src, wtype, k, n, kind="omp")
    try:
        for which in (0, 1):
            htpg.set_qk0_decode(which)
            outs = []
            for _ in range(3):
                out = torch.empty((m, n), device=gpu)
                htpg.check(htpg.qk0_run(w, out, xd, m), "htpg_qk0_run")
                outs.append(out.cpu().numpy())
            assert all(np.array_equal(outs[0], o) for o in outs[1:])
            assert _rel(outs[0], ref) <= 1e-5
    finally:
        htpg.set_qk0_decode(0)


@pytest.mark.parametrize("wtype", TYPES)
@pytest.mark.parametrize("k,n", [(64, 32), (96, 160), (4096, 512)])
def test_qk0_dequantize_bit_exact(gpu, lib, wtype, k, n):
    bb = O.qk0_block_bytes(wtype)
    rng = np.random.default_rng(k + n + wtype)
    src = rng.integers(0, 256, k * n // 256 * bb, dtype=np.uint8)
    blocks = src.reshape(-1, bb)
    scales = rng.normal(0, 0.02, (blocks.shape[0], 8)).astype(np.float16).view(np.uint16)
    special = np.array([0x0001, 0x03FF, 0x0400, 0x7BFF, 0x8001, 0x0000, 0xFBFF], np.uint16)
    scales[::5] = rng.choice(special, (scales[::5].shape[0], 8))   # subnormals, overflow to inf, zero
    blocks[:, :16] = scales.view(np.uint8).reshape(-1, 16)
    want = O.qk0_dequant(src, wtype, k, n)
    wd = torch.from_numpy(src).to(gpu)
    out = torch.zeros((n, k), dtype=torch.int16, device=gpu)
    htpg.check(lib.htpg_qk0_dequantize(htpg.ptr(out), htpg.ptr(wd), k, n, wtype, htpg.stream_ptr()),
               "htpg_qk0_dequantize")
    got = out.cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(got, want)


def test_qk0_reference_entry_point_codes(gpu, lib):
    m, k, n = 4, 64, 64
    src, x = _case(O.GGML_Q8_0, m, k, n, seed=1)
    wd, xd = torch.from_numpy(src).to(gpu), torch.from_numpy(x).to(gpu)
    out = torch.zeros((m, n), device=gpu)
    f = lib.hmx_mat_mul_permuted_qk_0_d16a32
    try:
        assert f(htpg.ptr(out), htpg.ptr(xd), htpg.ptr(wd), m, k, n, O.GGML_Q8_0) == 0
    finally:
        lib.htpg_weight_cache_drop(htpg.ptr(wd))
    assert _rel(out.cpu().numpy(), O.qk0_linear(x, src, O.GGML_Q8_0, k, n)) <= 1e-5
    assert f(None, htpg.ptr(xd), htpg.ptr(wd), m, k, n, 8) == -1
    assert f(htpg.ptr(out), htpg.ptr(xd), htpg.ptr(wd), 0, k, n, 8) == -1
    assert f(htpg.ptr(out), htpg.ptr(xd), htpg.ptr(wd), m, 48, n, 8) == -1
    assert f(htpg.ptr(out), htpg.ptr(xd), htpg.ptr(wd), m, k, 16, 8) == -1
    assert f(htpg.ptr(out), htpg.ptr(xd), htpg.ptr(wd), m, k, n, 3) == -1        # Q4_1: not served
    assert f(htpg.ptr(out) + 4, htpg.ptr(xd), htpg.ptr(wd), m, k, n - 32, 8) == -1   # alignment


@pytest.mark.parametrize("op,wtype", [(2, O.GGML_Q4_0), (3, O.GGML_Q8_0), (4, O.GGML_IQ4_NL)])
def test_qk0_through_executor(gpu, lib, op, wtype):
    m, k, n = 9, 256, 192
    src, x = _case(wtype, m, k, n, seed=op)
    ref = O.qk0_linear(x, src, wtype, k, n, kind="omp")
    fds, ptrs = {}, {}

    def alloc(name, arr):
        fd, p = ctypes.c_int(), ctypes.c_void_p()
        htpg.check(lib.htpg_buffer_alloc(arr.nbytes, htpg.BUF_HOST, ctypes.byref(fd), ctypes.byref(p)), name)
        ctypes.memmove(p.value, arr.ctypes.data, arr.nbytes)
        fds[name], ptrs[name] = fd.value, p.value

    try:
        alloc("out", np.zeros(m * n, np.float32))
        alloc("x", np.ascontiguousarray(x))
        alloc("w", src)
        payload = struct.pack("<iiiiiiiii", fds["out"], 0, fds["x"], 0, fds["w"], 0, m, k, n) + b"\0" * 56
        payload += struct.pack("<i", 0)                                   # elapsed_us (96-byte form)
        req = np.frombuffer(struct.pack("<I", op) + payload, np.uint8).copy()
        assert lib.execute_op_simple(req.ctypes.data, req.nbytes) == 0
        got = np.empty(m * n, np.float32)
        ctypes.memmove(got.ctypes.data, ptrs["out"], got.nbytes)
        assert _rel(got.reshape(m, n), ref) <= 1e-5
        assert struct.unpack_from("<i", req.tobytes(), 4 + 92)[0] > 0
    finally:
        for fd in fds.values():
            lib.htpg_buffer_release(fd)



def test_qk0_prepared_weight_outlives_the_stream(gpu, lib):
    """The stage records are a copy: the caller's stream can be freed or
    overwritten after htpg_qk0_weights_create; both the fused (M <= 32) and the
    large-M path read only the records."""
    k, n = 320, 224                      # K % 64 = 32 and N % 128 = 96: padded records
    src, x = _case(O.GGML_IQ4_NL, 40, k, n, seed=77)
    wd = torch.from_numpy(src).to(gpu)
    w = htpg.qk0_weights(wd, O.GGML_IQ4_NL, k, n)
    wd.fill_(0xFF)                       # garbage where the stream was
    torch.cuda.synchronize()
    for m in (7, 40):
        xd = torch.from_numpy(np.ascontiguousarray(x[:m])).to(gpu)
        out = torch.full((m, n), float("nan"), device=gpu)
        htpg.check(htpg.qk0_run(w, out, xd, m), "htpg_qk0_run")
        assert _rel(out.cpu().numpy(), O.qk0_linear(x[:m], src, O.GGML_IQ4_NL, k, n)) <= 1e-5
