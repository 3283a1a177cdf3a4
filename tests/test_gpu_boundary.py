"""The reference-facing entry points on their success paths, on the GPU,
against the oracle.

Each test posts what a caller of the reference posts and checks both the
answer fields and the numbers:

* opcode 16 (F16EpilogueParams, 56 bytes; reference op_executor.cc:446-471)
  through execute_op_simple with host and device buffers, and through a live
  message channel (commu.c:99-269) together with opcodes 15 and 1;
* opcode 1 (MatMulParams, 92 bytes and the 96-byte form with elapsed_us;
  op_executor.cc:473-540), with HTPG_OP_TRACE set so the debug hashes
  (FNV-1a of the activation and output bytes, op_executor.cc:46-56) are filled;
* the direct IDL calls htp_ops_mat_mul_permuted_w16a32 and _trace
  (commu.c:637-808) on an initialised backend, and their session wrappers;
* htp_ops_test_ops (commu.c:813-827);
* the 104-byte profiled opcode-15 request in modes 1-3 (op_reg.h:87-149,
  linear_w8a8.c:328-508) and the kernel-level hmx_mat_mul_native_w8a8_profiled;
* the watchdog path: after a launch gives up, htpg_check_device restores the
  zeroed scratch that the split-K and stream-K kernels rely on.

Bars: W8A8 mode-0 outputs bit-exact; F16 outputs within max-abs-rel 1e-2 of
the oracle with FP32 and with FP16-rounded accumulation, and within 1e-5 of the
FP32-accumulating oracle.
"""
import ctypes
import struct
import time

import numpy as np
import pytest

import htpg
import oracle as O

pytestmark = pytest.mark.gpu

W8A8_TOL = 2e-3
F16_TOL = 1e-2
AEE_SUCCESS = 0


def fnv1a(data: bytes) -> int:
    h = 14695981039346656037
    for b in data:
        h ^= b
        h = (h * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


class Bufs:
    """RPCMEM stand-ins: pinned host buffers made by the library (page aligned),
    or torch device tensors registered under caller-chosen fds."""

    def __init__(self, L, base_fd=7000):
        self.L, self.next_fd = L, base_fd
        self.fd, self.ptr, self.kind, self.keep, self.nbytes = {}, {}, {}, {}, {}

    def add(self, name, arr, kind=htpg.BUF_HOST):
        arr = np.ascontiguousarray(arr)
        if kind == htpg.BUF_HOST:
            fd, p = ctypes.c_int(), ctypes.c_void_p()
            htpg.check(self.L.htpg_buffer_alloc(arr.nbytes, htpg.BUF_HOST, ctypes.byref(fd), ctypes.byref(p)), name)
            ctypes.memmove(p.value, arr.ctypes.data, arr.nbytes)
            self.fd[name], self.ptr[name] = fd.value, p.value
        else:
            import torch
            t = torch.from_numpy(arr.view(np.uint8).copy()).to("cuda:0")
            fd = self.next_fd
            self.next_fd += 1
            htpg.check(self.L.htpg_buffer_register(fd, t.data_ptr(), arr.nbytes, htpg.BUF_DEVICE), name)
            self.fd[name], self.ptr[name], self.keep[name] = fd, t.data_ptr(), t
        self.kind[name], self.nbytes[name] = kind, arr.nbytes
        return self.fd[name]

    def read(self, name, dtype=np.float32):
        if self.kind[name] == htpg.BUF_HOST:
            out = np.empty(self.nbytes[name], np.uint8)
            ctypes.memmove(out.ctypes.data, self.ptr[name], out.nbytes)
        else:
            import torch
            torch.cuda.synchronize()
            out = self.keep[name].cpu().numpy()
        return out.view(dtype)

    def release(self):
        for fd in self.fd.values():
            self.L.htpg_buffer_release(fd)


@pytest.fixture()
def bufs(gpu, lib):
    b = Bufs(lib)
    yield b
    b.release()


def execute(L, op, payload: bytes):
    req = np.frombuffer(struct.pack("<I", op) + payload, np.uint8).copy()
    rc = L.execute_op_simple(req.ctypes.data, req.nbytes)
    return rc, req[4:].tobytes()


def f16_payload(fo, fa, fw, fb, m, k, n, channels, mode, elapsed=-1):
    return struct.pack("<8i6i", fo, 0, fa, 0, fw, 0, fb, 0, m, k, n, channels, mode, elapsed)


def matmul_payload(fo, fa, fw, m, k, n, with_elapsed, elapsed=-1):
    p = struct.pack("<6i3i", fo, 0, fa, 0, fw, 0, m, k, n) + b"\xee" * (92 - 36)
    return p + (struct.pack("<i", elapsed) if with_elapsed else b"")


def matmul_debug(payload: bytes):
    """MatMulParams debug fields (include/op_reg.h): vtcm_base, vtcm_size,
    vtcm_ctx, hmx_ctx, worker_pool, hmx_lock_result, act_hash, out_hash,
    out_hash_after_invalidate."""
    return struct.unpack_from("<QIiiQiQQQ", payload, 36)


def _f16_case(m, k, n, seed, bias, mode):
    x = O.normal(m * k, 1.0, 0, 1, seed).reshape(m, k)
    w = O.f16_normal(k * n, 0.02, seed + 1).reshape(k, n)
    b = O.normal(n, 0.01, 0, 1, seed + 2) if bias else None
    return x, O.f16_pack_permuted(w), b


def _check_f16(got, x, wperm, k, n, bias, channels, mode):
    assert not np.isnan(got).any()
    for round_acc in (False, True):   # FP32 accumulator and the HMX FP16-rounded one
        ref = O.f16_linear(x, wperm, k, n, bias=bias, channels=channels, mode=mode, round_acc_f16=round_acc)
        assert O.max_abs_rel(got, ref) <= F16_TOL
        if not round_acc:
            assert O.max_abs_rel(got, ref) <= 1e-5


# ------------------------------------------------------------------ opcode 16
@pytest.mark.parametrize("m,k,n", [(77, 768, 3072), (130, 256, 160)])
@pytest.mark.parametrize("mode", [0, 1, 2, 3])
@pytest.mark.parametrize("with_bias", [False, True])
def test_opcode16_execute_host_buffers(lib, bufs, m, k, n, mode, with_bias):
    x, wperm, b = _f16_case(m, k, n, 40 + mode + 4 * m, with_bias, mode)
    channels = n - 32 + 3 if mode == 3 else n
    fo = bufs.add("out", np.full(m * channels, np.nan, np.float32))
    fa, fw = bufs.add("x", x), bufs.add("w", wperm)
    fb = bufs.add("bias", b[:channels].copy()) if with_bias else -1
    rc, payload = execute(lib, 16, f16_payload(fo, fa, fw, fb, m, k, n, channels, mode))
    assert rc == 0
    elapsed = struct.unpack_from("<i", payload, 52)[0]
    assert 0 <= elapsed < 10_000_000
    got = bufs.read("out").reshape((channels, m) if mode == 3 else (m, n))
    _check_f16(got, x, wperm, k, n, b, channels, mode)


@pytest.mark.parametrize("mode,with_bias", [(2, True), (3, False)])
def test_opcode16_execute_device_buffers(lib, bufs, mode, with_bias):
    """C2 (CLIP fc1, M=77, K=768, N=3072) with every operand in HBM."""
    c = O.config_c2()
    m, k, n = c.m, c.k, c.n
    channels = 3000 if mode == 3 else n
    fo = bufs.add("out", np.full(m * channels, np.nan, np.float32), htpg.BUF_DEVICE)
    fa, fw = bufs.add("x", c.x, htpg.BUF_DEVICE), bufs.add("w", c.wperm, htpg.BUF_DEVICE)
    fb = bufs.add("bias", c.bias[:channels].copy(), htpg.BUF_DEVICE) if with_bias else -1
    rc, _ = execute(lib, 16, f16_payload(fo, fa, fw, fb, m, k, n, channels, mode))
    assert rc == 0
    got = bufs.read("out").reshape((channels, m) if mode == 3 else (m, n))
    _check_f16(got, c.x, c.wperm, k, n, c.bias if with_bias else None, channels, mode)


def test_opcode16_weight_rewrite_is_picked_up(lib, bufs):
    """A weight buffer rewritten in place and announced through a put
    (htpg_buffer_touch) is repacked again, not served from the cache."""
    m, k, n = 40, 128, 96
    x, w1, _ = _f16_case(m, k, n, 71, False, 0)
    _, w2, _ = _f16_case(m, k, n, 72, False, 0)
    fo, fa, fw = bufs.add("out", np.zeros(m * n, np.float32)), bufs.add("x", x), bufs.add("w", w1)
    assert execute(lib, 16, f16_payload(fo, fa, fw, -1, m, k, n, n, 0))[0] == 0
    _check_f16(bufs.read("out").reshape(m, n), x, w1, k, n, None, n, 0)
    ctypes.memmove(bufs.ptr["w"], w2.ctypes.data, w2.nbytes)
    assert lib.htpg_buffer_touch(fw) == 0
    assert execute(lib, 16, f16_payload(fo, fa, fw, -1, m, k, n, n, 0))[0] == 0
    _check_f16(bufs.read("out").reshape(m, n), x, w2, k, n, None, n, 0)


# ------------------------------------------------------------------ channel
class Channel:
    """The caller's side of the shared-memory message channel: MessageHeader
    {state v[0..7], checksum, n_reqs, req_offsets[n+1]}, then per request a
    RequestHeader {state, type} and its data (include/message.h)."""

    def __init__(self, buf):
        self.buf = buf

    def post(self, requests, timeout=60.0):
        b = self.buf
        b[:] = 0
        n = len(requests)
        hdr = 16 + 4 * (n + 1)
        offs, body = [hdr], b""
        for typ, data in requests:
            r = struct.pack("<ii", 0x5A5A5A5A, typ) + data
            body += r
            offs.append(offs[-1] + len(r))
        b[8:16] = np.frombuffer(struct.pack("<Ii", 0, n), np.uint8)
        b[16:16 + 4 * (n + 1)] = np.frombuffer(struct.pack("<" + "i" * (n + 1), *offs), np.uint8)
        b[hdr:hdr + len(body)] = np.frombuffer(body, np.uint8)
        b[0] = 1
        t0 = time.time()
        while b[1] != 1:
            assert time.time() - t0 < timeout, "receiver did not answer"
            time.sleep(0.0005)
        states = [struct.unpack_from("<i", b, offs[i])[0] for i in range(n)]
        datas = [b[offs[i] + 8:offs[i + 1]].tobytes() for i in range(n)]
        return states, datas


def test_live_channel_runs_opcodes_16_15_and_1(lib, bufs):
    """One message with three compute requests on an initialised backend: C2
    through opcode 16, a W8A8 linear with bias + GELU through the 56-byte
    opcode-15 form, and opcode 1 with elapsed_us."""
    c2 = O.config_c2()
    w8 = O.make_w8a8(2, "chan", 300, 512, 640, 0.005, True, 1)
    x1, w1, _ = _f16_case(64, 256, 192, 91, False, 0)
    f = dict(
        o16=bufs.add("o16", np.full(c2.m * c2.n, np.nan, np.float32)), x16=bufs.add("x16", c2.x),
        w16=bufs.add("w16", c2.wperm), b16=bufs.add("b16", c2.bias),
        o15=bufs.add("o15", np.full(w8.m * w8.n, np.nan, np.float32)), x15=bufs.add("x15", w8.x),
        c15=bufs.add("c15", w8.blob), b15=bufs.add("b15", w8.bias),
        o1=bufs.add("o1", np.full(64 * 192, np.nan, np.float32)), x1=bufs.add("x1", x1), w1=bufs.add("w1", w1))
    chan = np.zeros(8192, np.uint8)
    h = ctypes.c_uint64()
    assert lib.htp_ops_open(None, ctypes.byref(h)) == 0
    assert lib.htpg_buffer_register(7999, chan.ctypes.data, chan.nbytes, htpg.BUF_HOST) == 0
    try:
        assert lib.htp_ops_init_backend(h) == 0
        assert lib.htp_ops_create_channel(h, 7999, chan.nbytes) == 0
        p16 = struct.pack("<I", 16) + f16_payload(f["o16"], f["x16"], f["w16"], f["b16"], c2.m, c2.k, c2.n, c2.n, 2)
        p15 = struct.pack("<I", 15) + struct.pack("<10i", f["o15"], 0, f["x15"], 0, f["c15"], 0, w8.m, w8.k, w8.n,
                                                  -1) + struct.pack("<4i", f["b15"], 0, w8.n, 1)
        p1 = struct.pack("<I", 1) + matmul_payload(f["o1"], f["x1"], f["w1"], 64, 256, 192, True)
        states, datas = Channel(chan).post([(2, p16), (2, p15), (2, p1)])
        assert states == [0, 0, 0]
        assert struct.unpack_from("<i", datas[0], 4 + 52)[0] >= 0       # opcode 16 elapsed_us
        assert struct.unpack_from("<i", datas[1], 4 + 36)[0] >= 0       # opcode 15 elapsed_us
        assert struct.unpack_from("<i", datas[2], 4 + 92)[0] >= 0       # opcode 1 elapsed_us
        assert lib.htp_ops_destroy_channel(h) == 0
    finally:
        lib.htp_ops_close(h)
        lib.htpg_buffer_release(7999)
    _check_f16(bufs.read("o16").reshape(c2.m, c2.n), c2.x, c2.wperm, c2.k, c2.n, c2.bias, c2.n, 2)
    ref15 = O.w8a8_linear(w8.x, w8.blob, w8.k, w8.n, bias=w8.bias, mode=1)
    assert O.max_abs_rel(bufs.read("o15").reshape(w8.m, w8.n), ref15) <= W8A8_TOL
    _check_f16(bufs.read("o1").reshape(64, 192), x1, w1, 256, 192, None, 192, 0)


# ------------------------------------------------------------------ opcode 1
@pytest.mark.parametrize("with_elapsed", [False, True])
@pytest.mark.parametrize("trace", [False, True])
def test_opcode1_execute(lib, bufs, monkeypatch, with_elapsed, trace):
    m, k, n = 77, 768, 512
    x, wperm, _ = _f16_case(m, k, n, 101, False, 0)
    if trace:
        monkeypatch.setenv("HTPG_OP_TRACE", "1")
    else:
        monkeypatch.delenv("HTPG_OP_TRACE", raising=False)
    fo, fa, fw = bufs.add("out", np.full(m * n, np.nan, np.float32)), bufs.add("x", x), bufs.add("w", wperm)
    rc, payload = execute(lib, 1, matmul_payload(fo, fa, fw, m, k, n, with_elapsed))
    assert rc == 0
    got = bufs.read("out").reshape(m, n)
    _check_f16(got, x, wperm, k, n, None, n, 0)
    dbg = matmul_debug(payload)
    if trace:
        assert dbg[:6] == (0, 0, 0, 0, 0, 0)          # no VTCM, HMX context or worker pool here
        assert dbg[6] == fnv1a(x.tobytes())
        assert dbg[7] == fnv1a(got.tobytes())
        assert dbg[8] == dbg[7]
    else:
        assert payload[36:92] == b"\xee" * 56         # untouched when tracing is off
    if with_elapsed:
        assert 0 <= struct.unpack_from("<i", payload, 92)[0] < 10_000_000


def test_opcode1_device_buffers_misaligned_is_minus_three(lib, bufs):
    m, k, n = 8, 64, 64
    x, wperm, _ = _f16_case(m, k, n, 5, False, 0)
    fo = bufs.add("out", np.zeros(m * n + 32, np.float32), htpg.BUF_DEVICE)
    fa, fw = bufs.add("x", x, htpg.BUF_DEVICE), bufs.add("w", wperm, htpg.BUF_DEVICE)
    p = struct.pack("<6i3i", fo, 64, fa, 0, fw, 0, m, k, n) + b"\0" * 56
    assert execute(lib, 1, p)[0] == -3
    p = struct.pack("<6i3i", fo, 128, fa, 0, fw, 0, m, k, n) + b"\0" * 56
    assert execute(lib, 1, p)[0] == 0
    got = bufs.read("out")[32:32 + m * n].reshape(m, n)
    _check_f16(got, x, wperm, k, n, None, n, 0)


# ------------------------------------------------------------------ IDL calls
@pytest.fixture()
def backend(lib):
    h = ctypes.c_uint64()
    assert lib.htp_ops_open(None, ctypes.byref(h)) == 0
    assert lib.htp_ops_init_backend(h) == 0
    yield h
    assert lib.htp_ops_close(h) == 0


@pytest.mark.parametrize("kind", [htpg.BUF_HOST, htpg.BUF_DEVICE])
def test_direct_w16a32_and_trace(lib, bufs, backend, kind):
    m, k, n = 100, 512, 320
    x, wperm, _ = _f16_case(m, k, n, 111, False, 0)
    fo = bufs.add("out", np.full(m * n, np.nan, np.float32), kind)
    fa, fw = bufs.add("x", x, kind), bufs.add("w", wperm, kind)
    assert lib.htp_ops_mat_mul_permuted_w16a32(backend, fo, 0, fa, 0, fw, 0, m, k, n) == 0
    got = bufs.read("out").reshape(m, n)
    _check_f16(got, x, wperm, k, n, None, n, 0)
    ha, ho, ho2 = ctypes.c_uint64(1), ctypes.c_uint64(1), ctypes.c_uint64(1)
    assert lib.htp_ops_mat_mul_permuted_w16a32_trace(backend, fo, 0, fa, 0, fw, 0, m, k, n, ctypes.byref(ha),
                                                     ctypes.byref(ho), ctypes.byref(ho2)) == 0
    got2 = bufs.read("out").reshape(m, n)
    np.testing.assert_array_equal(got2.view(np.uint32), got.view(np.uint32))   # same kernels, same bits
    assert ha.value == fnv1a(x.tobytes())
    assert ho.value == fnv1a(got2.tobytes()) == ho2.value


def test_session_wrappers_run_w16a32(lib, bufs):
    """The sd.cpp-facing session layer (src/host/session.c, op_export.c):
    open a session, initialise its backend, run opcode 1 through the
    htp_ops_rpc_* wrappers on the session and on the global handle."""
    m, k, n = 33, 256, 128
    x, wperm, _ = _f16_case(m, k, n, 121, False, 0)
    fo, fa, fw = bufs.add("out", np.full(m * n, np.nan, np.float32)), bufs.add("x", x), bufs.add("w", wperm)
    s = ctypes.c_void_p()
    assert lib.htp_ops_session_open(ctypes.byref(s), 3, b"parity", 0) == 0
    try:
        assert lib.htp_ops_session_init_backend(s) == 0
        assert lib.htp_ops_session_is_initialized(s) == 1
        assert lib.htp_ops_rpc_mat_mul_permuted_w16a32_session(s, fo, 0, fa, 0, fw, 0, m, k, n) == 0
        _check_f16(bufs.read("out").reshape(m, n), x, wperm, k, n, None, n, 0)
        ha, ho, ho2 = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        assert lib.htp_ops_rpc_mat_mul_permuted_w16a32_trace_session(
            s, fo, 0, fa, 0, fw, 0, m, k, n, ctypes.byref(ha), ctypes.byref(ho), ctypes.byref(ho2)) == 0
        assert ha.value == fnv1a(x.tobytes())
        assert lib.htp_ops_set_active_session(s) == 0
        ctypes.memset(bufs.ptr["out"], 0xff, m * n * 4)
        assert lib.htp_ops_rpc_mat_mul_permuted_w16a32(fo, 0, fa, 0, fw, 0, m, k, n) == 0
        _check_f16(bufs.read("out").reshape(m, n), x, wperm, k, n, None, n, 0)
    finally:
        lib.htp_ops_session_close(s)


def test_test_ops_succeeds(lib, backend):
    scope = ctypes.c_int32(-7)
    assert lib.htp_ops_test_ops(backend, ctypes.byref(scope)) == AEE_SUCCESS
    assert scope.value == 0


# ------------------------------------------------------------------ 104-byte opcode 15
PROFILE_FMT = "<II7Q"   # mode, reserved, setup, activation, weight, hmx, output, mac, readout ticks


@pytest.mark.parametrize("mode", [1, 2, 3])
@pytest.mark.parametrize("m,k,n", [(256, 1152, 4608), (20, 2048, 1024), (4, 4096, 512)])
def test_opcode15_profiled_trailer(lib, bufs, mode, m, k, n):
    c = O.make_w8a8(0, f"prof{m}", m, k, n, 0.01, False, 0)
    fo = bufs.add("out", np.full(m * n, np.nan, np.float32))
    fa, fc = bufs.add("x", c.x), bufs.add("cst", c.blob)
    trailer = struct.pack(PROFILE_FMT, mode, 0xdead, *([12345] * 7))
    rc, payload = execute(lib, 15, struct.pack("<10i", fo, 0, fa, 0, fc, 0, m, k, n, -1) + trailer)
    assert rc == 0
    ref = O.w8a8_linear(c.x, c.blob, k, n)
    got = bufs.read("out").reshape(m, n)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert 0 <= struct.unpack_from("<i", payload, 36)[0] < 10_000_000      # elapsed_us
    f = struct.unpack_from(PROFILE_FMT, payload, 40)
    pmode, reserved, setup, act, weight, hmx, output, mac, readout = f
    assert pmode == mode
    assert act > 0 and hmx > 0                     # 19.2 MHz ticks of the two phases
    assert weight == 0 and output == 0             # both inside the GEMM launch
    assert setup < 19200 * 10_000
    plan = htpg.plan_info(0, m, n, k)
    if mode == 1:
        assert reserved == 0 and mac == 0 and readout == 0
    elif mode == 2:
        assert reserved == 0 and mac == hmx and readout == 0
    else:
        assert reserved & 0x80000000 == 0          # no allocation table: never a "table hit"
        # low half: 64-row activation tiles per output tile; high half: 64-column weight groups
        rows64, cols64 = reserved & 0xffff, reserved >> 16
        if plan["swap"] in (1, 2):                 # small-M swapped tiles / register-fed decode
            assert (rows64, cols64) == (1, 2)
        elif plan["swap"] == 3:                    # CTA pair, swapped: 256 weight columns x bn rows
            assert (rows64, cols64) == (plan["bn"] // 64, 4)
        else:                                      # 128-row tiles or 256-row CTA-pair tiles
            assert rows64 in (2, 4) and cols64 == max(1, plan["bn"] // 64)
        assert mac == plan["units"]
        assert readout >= k * n                    # every weight byte loaded at least once


def test_kernel_level_profiled_matches_executor(gpu, lib):
    import torch
    m, k, n = 256, 1152, 4608
    c = O.config_c1()
    dev = gpu
    blob, x = torch.from_numpy(c.blob).to(dev), torch.from_numpy(c.x).to(dev)
    out = torch.full((m, n), float("nan"), device=dev)
    prof = (ctypes.c_uint8 * 64).from_buffer_copy(struct.pack(PROFILE_FMT, 3, 0, *([7] * 7)))
    assert lib.hmx_mat_mul_native_w8a8_profiled(htpg.ptr(out), htpg.ptr(x), htpg.ptr(blob), m, k, n, prof) == 0
    ref = O.w8a8_linear(c.x, c.blob, k, n)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    f = struct.unpack(PROFILE_FMT, bytes(prof))
    assert f[0] == 3 and f[3] > 0 and f[5] > 0 and f[7] == htpg.plan_info(0, m, n, k)["units"]
    lib.htpg_weight_cache_drop(htpg.ptr(blob))
    # without a trailer: same bits
    out2 = torch.full((m, n), float("nan"), device=dev)
    assert lib.hmx_mat_mul_native_w8a8(htpg.ptr(out2), htpg.ptr(x), htpg.ptr(blob), m, k, n) == 0
    assert torch.equal(out.view(torch.int32), out2.view(torch.int32))
    lib.htpg_weight_cache_drop(htpg.ptr(blob))


# ------------------------------------------------------------------ watchdog recovery
def test_watchdog_restores_split_k_and_stream_k_scratch(gpu, lib):
    """An aborted launch can leave split-K partial sums and arrival counters
    non-zero.  With both kinds of scratch poisoned and the watchdog word set,
    htpg_check_device answers HTPG_EWATCHDOG once, and the next split-K W8A8
    run and stream-K opcode 2-4 run are exact again."""
    import torch
    dev = gpu
    cw = O.make_w8a8(5, "wd", 24, 6144, 1024, 0.0, False, 0)      # swapped plan, exact INT32 split-K
    plan = htpg.plan_info(0, cw.m, cw.n, cw.k)
    assert plan["swap"] == 1 and plan["splits"] > 1
    blob, xw = torch.from_numpy(cw.blob).to(dev), torch.from_numpy(cw.x).to(dev)
    hw = htpg.w8a8_weights(blob, cw.k, cw.n)
    src = O.qk0_random(O.GGML_Q4_0, 4096, 1024, seed=3)
    xq = O.normal(5 * 4096, 1.0, 0, 1, 4).reshape(5, 4096)
    hq = htpg.qk0_weights(torch.from_numpy(src).to(dev), O.GGML_Q4_0, 4096, 1024)
    xqd = torch.from_numpy(xq).to(dev)
    ref_w = O.w8a8_linear(cw.x, cw.blob, cw.k, cw.n)
    ref_q = O.qk0_linear(xq, src, O.GGML_Q4_0, 4096, 1024)

    def run_both():
        ow = torch.full((cw.m, cw.n), float("nan"), device=dev)
        oq = torch.full((5, 1024), float("nan"), device=dev)
        htpg.check(htpg.w8a8_run(hw, ow, xw), "w8a8")
        htpg.check(htpg.qk0_run(hq, oq, xqd, 5), "qk0")
        return ow, oq

    ow, oq = run_both()                     # both workspaces exist now
    assert htpg.check_device() == 0
    ws = (ctypes.c_size_t(), ctypes.c_size_t())
    htpg.check(lib.htpg_debug_workspaces(ctypes.byref(ws[0]), ctypes.byref(ws[1])), "workspaces")
    assert ws[0].value > 0 and ws[1].value > 0
    htpg.check(lib.htpg_debug_simulate_abort(0x5A), "simulate abort")
    flags = ctypes.c_uint32()
    assert lib.htpg_check_device(None, ctypes.byref(flags)) == htpg.EWATCHDOG
    assert flags.value != 0
    assert htpg.check_device() == 0         # cleared
    ow, oq = run_both()
    assert htpg.check_device() == 0
    np.testing.assert_array_equal(ow.cpu().numpy().view(np.uint32), ref_w.view(np.uint32))
    assert O.max_abs_rel(oq.cpu().numpy(), ref_q) <= 1e-5
