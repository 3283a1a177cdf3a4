"""Host runtime of libhtp_ops_b200.so on the CPU (no device calls reached).

Mirrors the reference dispatcher's contract (src/dsp/op_executor.cc:274-540):
payload sizes, shape limits, {fd, offset} resolution and header checks return
the reference's codes before any device work; the shared-memory message
channel (src/dsp/commu.c:99-269) runs its v[0]/v[1] handshake; sessions,
leases and capability markers behave like src/host/session.c and op_export.c.
"""
import ctypes
import struct
import time

import numpy as np
import pytest

import htpg
import oracle as O

AEE_EBADSTATE, AEE_EBADPARM, AEE_EUNSUPPORTED, AEE_EALREADY = 13, 14, 20, 26


@pytest.fixture(scope="module")
def L():
    return htpg.lib()


class Buffers:
    """Caller-owned host buffers registered under caller-chosen fds."""

    def __init__(self, L, base_fd):
        self.L, self.next_fd, self.keep = L, base_fd, []

    def add(self, arr, kind=htpg.BUF_HOST):
        fd = self.next_fd
        self.next_fd += 1
        self.keep.append(arr)
        assert self.L.htpg_buffer_register(fd, arr.ctypes.data, arr.nbytes, kind) == 0
        return fd

    def release(self):
        for fd in range(self.next_fd - len(self.keep), self.next_fd):
            self.L.htpg_buffer_release(fd)


def request(op, payload: bytes):
    buf = np.frombuffer(struct.pack("<I", op) + payload, np.uint8).copy()
    return buf


def run(L, op, payload):
    buf = request(op, payload)
    rc = L.execute_op_simple(buf.ctypes.data, buf.nbytes)
    return rc, buf


def w8a8_payload(out, act, cst, m, k, n, extra=b""):
    return struct.pack("<iiiiiiiiii", out[0], out[1], act[0], act[1], cst[0], cst[1], m, k, n, 0) + extra


# ------------------------------------------------------------------ library
def test_library_exports_every_declared_symbol(L):
    names = htpg.declared_symbols()
    assert len(names) > 70
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_capability_markers(L):
    assert L.htp_ops_f16_epilogue_version() == 1
    assert L.htp_ops_w8a8_epilogue_version() == 1
    assert L.htp_ops_native_model_version() == 0
    assert L.htp_ops_dit_aux_version() == 0
    assert L.htp_ops_dit_concat_version() == 0
    assert L.htpg_version() == 1
    assert L.htpg_strerror(-3) == b"constants header or alignment mismatch"


# ------------------------------------------------------------------ opcode 15
@pytest.fixture()
def w8a8_bufs(L):
    m, k, n = 8, 64, 128
    c = O.make_w8a8(0, "t", m, k, n, 0.0, True, 0)
    b = Buffers(L, 1000)
    fds = dict(out=b.add(np.zeros(m * n, np.float32)), act=b.add(c.x.copy()),
               cst=b.add(c.blob.copy()), bias=b.add(c.bias.copy()))
    yield b, fds, (m, k, n), c
    b.release()


@pytest.mark.parametrize("size", [0, 36, 39, 41, 47, 55, 57, 100, 105])
def test_w8a8_payload_size(L, size):
    rc, _ = run(L, 15, b"\0" * size)
    assert rc == -1


@pytest.mark.parametrize("m,k,n", [(0, 64, 64), (65537, 64, 64), (1, 16, 64), (1, 48, 64), (1, 16416, 64),
                                   (1, 64, 32), (1, 64, 100), (1, 64, 16448)])
def test_w8a8_shape_limits(L, m, k, n):
    rc, _ = run(L, 15, w8a8_payload((1, 0), (2, 0), (3, 0), m, k, n))
    assert rc == -1


def test_w8a8_unmapped_buffers(L, w8a8_bufs):
    b, f, (m, k, n), _ = w8a8_bufs
    assert run(L, 15, w8a8_payload((999, 0), (f["act"], 0), (f["cst"], 0), m, k, n))[0] == -2
    # buffer too small for the request (offset pushes past the end)
    assert run(L, 15, w8a8_payload((f["out"], 4), (f["act"], 0), (f["cst"], 0), m, k, n))[0] == -2
    assert run(L, 15, w8a8_payload((f["out"], 0), (f["act"], 0), (f["cst"], 0), m, k, n + 64))[0] == -2


@pytest.mark.parametrize("field,delta", [(0, 1), (1, 1), (2, 32), (3, 64), (4, 4), (5, 4), (6, 4), (7, 4), (8, 1)])
def test_w8a8_header_mismatch(L, w8a8_bufs, field, delta):
    b, f, (m, k, n), c = w8a8_bufs
    blob = b.keep[2]
    hdr = blob[:40].view(np.uint32)
    saved = hdr[field]
    hdr[field] = saved + delta
    try:
        rc, _ = run(L, 15, w8a8_payload((f["out"], 0), (f["act"], 0), (f["cst"], 0), m, k, n))
    finally:
        hdr[field] = saved
    assert rc == -3


def test_w8a8_profile_mode_checked_after_header(L, w8a8_bufs):
    b, f, (m, k, n), _ = w8a8_bufs
    prof = struct.pack("<II", 7, 0) + b"\0" * 56
    rc, _ = run(L, 15, w8a8_payload((f["out"], 0), (f["act"], 0), (f["cst"], 0), m, k, n, prof))
    assert rc == -1


def test_w8a8_cpu_control_must_be_mapped(L, w8a8_bufs):
    b, f, (m, k, n), _ = w8a8_bufs
    rc, _ = run(L, 15, w8a8_payload((f["out"], 0), (f["act"], 0), (f["cst"], 0), m, k, n,
                                    struct.pack("<ii", 4242, 0)))
    assert rc == -2


@pytest.mark.parametrize("channels,mode", [(128, 4), (128, -1), (129, 3), (0, 3), (100, 0), (100, 1)])
def test_w8a8_epilogue_extension_validation(L, w8a8_bufs, channels, mode):
    b, f, (m, k, n), _ = w8a8_bufs
    ext = struct.pack("<iiii", f["bias"], 0, channels, mode)
    rc, _ = run(L, 15, w8a8_payload((f["out"], 0), (f["act"], 0), (f["cst"], 0), m, k, n, ext))
    assert rc == -1


def test_w8a8_epilogue_bias_too_small(L, w8a8_bufs):
    b, f, (m, k, n), _ = w8a8_bufs
    small = b.add(np.zeros(8, np.float32))
    ext = struct.pack("<iiii", small, 0, n, 1)
    rc, _ = run(L, 15, w8a8_payload((f["out"], 0), (f["act"], 0), (f["cst"], 0), m, k, n, ext))
    assert rc == -2


# ------------------------------------------------------------------ opcode 16
def f16_payload(out, act, wt, bias, m, k, n, channels, mode):
    return struct.pack("<" + "i" * 14, out[0], out[1], act[0], act[1], wt[0], wt[1], bias[0], bias[1],
                       m, k, n, channels, mode, 0)


@pytest.mark.parametrize("size", [0, 52, 55, 57, 60])
def test_f16_payload_exact_size(L, size):
    assert run(L, 16, b"\0" * size)[0] == -1


@pytest.mark.parametrize("m,k,n,ch,mode", [(0, 32, 32, 32, 0), (1, 48, 32, 32, 0), (1, 32, 48, 48, 0),
                                           (1, 32, 64, 32, 0), (1, 32, 64, 65, 3), (1, 32, 64, 0, 3),
                                           (1, 32, 64, 64, 4), (1, 32, 64, 64, -1)])
def test_f16_shape_and_mode(L, m, k, n, ch, mode):
    assert run(L, 16, f16_payload((1, 0), (2, 0), (3, 0), (-1, 0), m, k, n, ch, mode))[0] == -1


def test_f16_unmapped_is_minus_one(L):
    # the reference returns -1 (not -2) for unresolved opcode-16 buffers
    assert run(L, 16, f16_payload((77, 0), (78, 0), (79, 0), (-1, 0), 4, 32, 64, 64, 0))[0] == -1


# ------------------------------------------------------------------ opcode 1
def test_w16a32_payload_and_mapping(L):
    assert run(L, 1, b"\0" * 91)[0] == -1
    p = struct.pack("<iiiiiiiii", 50, 0, 51, 0, 52, 0, 4, 32, 64) + b"\0" * 56
    assert len(p) == 92
    assert run(L, 1, p)[0] == -2
    b = Buffers(L, 2000)
    out = np.zeros(4 * 64 + 64, np.float32)
    act = np.zeros(4 * 32 + 64, np.float32)
    wt = np.zeros(32 * 64 + 64, np.uint16)
    fo, fa, fw = b.add(out), b.add(act), b.add(wt)
    misaligned = 4 if out.ctypes.data % 128 == 0 else 0
    p = struct.pack("<iiiiiiiii", fo, misaligned or 4, fa, 0, fw, 0, 4, 32, 64) + b"\0" * 56
    assert run(L, 1, p)[0] == -3
    b.release()


# ------------------------------------------------------------------ opcodes 2-4
def _mm(fo, fa, fw, m, k, n, out_off=0):
    return struct.pack("<iiiiiiiii", fo, out_off, fa, 0, fw, 0, m, k, n) + b"\0" * 56


@pytest.mark.parametrize("op,block", [(2, 144), (3, 272), (4, 144)])
def test_qk0_payload_and_mapping(L, op, block):
    """op_executor.cc:771-790 sizes the operands from m, k, n and the block
    size of the opcode's type; mat_mul.c:1604-1613 answers -1 for the rest."""
    assert run(L, op, b"\0" * 91)[0] == -1                        # shorter than MatMulParams
    assert run(L, op, _mm(50, 51, 52, 0, 32, 64))[0] == -1         # zero size
    assert run(L, op, _mm(50, 51, 52, 4, 32, 64))[0] == -2         # unmapped buffers
    b = Buffers(L, 2100 + 10 * op)
    m, k, n = 4, 64, 64
    out = np.zeros(m * n + 64, np.float32)
    act = np.zeros(m * k + 64, np.float32)
    wt = np.zeros(k * n // 256 * block, np.uint8)
    fo, fa, fw = b.add(out), b.add(act), b.add(wt)
    assert run(L, op, _mm(fo, fa, fw, m, k, n + 32))[0] == -2      # weight shorter than k*n/256 blocks
    assert run(L, op, _mm(fo, fa, fw, m, 48, 32))[0] == -1         # k % 32
    assert run(L, op, _mm(fo, fa, fw, m, 32, 16))[0] == -1         # n % 32
    off = (128 - out.ctypes.data % 128) % 128 + 4                   # output not 128-byte aligned
    assert run(L, op, _mm(fo, fa, fw, m, k, n - 32, out_off=off))[0] == -1
    b.release()


def test_unknown_and_foreign_opcodes(L):
    assert run(L, 200, b"\0" * 16)[0] == 0                  # ignored like the reference
    assert run(L, 0, b"\0" * 24)[0] == AEE_EUNSUPPORTED       # rms_norm: not on this path
    assert run(L, 18, b"\0" * 80)[0] == AEE_EUNSUPPORTED      # attention


# ------------------------------------------------------------------ registry
def test_buffer_registry(L):
    a = np.zeros(256, np.uint8)
    assert L.htpg_buffer_register(3000, a.ctypes.data, a.nbytes, htpg.BUF_HOST) == 0
    kind = ctypes.c_int(-1)
    p = L.htpg_buffer_resolve(3000, 16, 240, ctypes.byref(kind))
    assert p == a.ctypes.data + 16 and kind.value == htpg.BUF_HOST
    assert not L.htpg_buffer_resolve(3000, 16, 241, None)
    assert not L.htpg_buffer_resolve(3000, -1, 1, None)
    assert L.htpg_buffer_touch(3000) == 0
    assert L.htpg_buffer_release(3000) == 0
    assert L.htpg_buffer_release(3000) == htpg.EUNMAPPED
    assert L.htpg_buffer_touch(3000) == htpg.EUNMAPPED
    assert L.htpg_buffer_register(-1, a.ctypes.data, 8, 1) == htpg.EARGS
    assert L.htpg_buffer_register(3001, a.ctypes.data, 8, 7) == htpg.EARGS


# ------------------------------------------------------------------ channel
class Channel:
    def __init__(self, L, fd, buf):
        self.L, self.fd, self.buf = L, fd, buf

    def post(self, requests, timeout=10.0):
        """requests: list of (type, data bytes) -> list of states."""
        b = self.buf
        b[:] = 0
        n = len(requests)
        hdr = 16 + 4 * (n + 1)
        offs = [hdr]
        body = b""
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
        return [struct.unpack_from("<i", b, offs[i])[0] for i in range(n)]


@pytest.fixture()
def channel(L):
    h = ctypes.c_uint64()
    assert L.htp_ops_open(None, ctypes.byref(h)) == 0
    buf = np.zeros(4096, np.uint8)
    assert L.htpg_buffer_register(4000, buf.ctypes.data, buf.nbytes, htpg.BUF_HOST) == 0
    assert L.htp_ops_create_channel(h, 4000, 4096) == AEE_EBADSTATE   # backend not initialised
    assert L.htp_ops_init_mapping_backend(h) == 0
    assert L.htp_ops_create_channel(h, 4000, 4096) == 0
    assert L.htp_ops_create_channel(h, 4000, 4096) == AEE_EALREADY
    yield h, Channel(L, 4000, buf)
    assert L.htp_ops_destroy_channel(h) == 0
    assert L.htp_ops_close(h) == 0
    L.htpg_buffer_release(4000)


def test_channel_handshake_and_states(L, channel):
    h, ch = channel
    keep = np.zeros(64, np.uint8)
    assert L.htpg_buffer_register(4001, keep.ctypes.data, 64, htpg.BUF_HOST) == 0
    legacy_map = struct.pack("<iii", 0, 1, 4001)                       # one get
    v2_bad_token = struct.pack("<IHHQii", 0x32504D52, 2, 24, 99, 0, 0)
    v2_get = struct.pack("<IHHQii", 0x32504D52, 2, 24, 0, 0, 1) + struct.pack("<iIQQQ", 4001, 0, 0, 64, 0)
    v2_get_missing = struct.pack("<IHHQii", 0x32504D52, 2, 24, 0, 0, 1) + struct.pack("<iIQQQ", 4999, 0, 0, 8, 0)
    states = ch.post([(2, struct.pack("<I", 15) + b"\0" * 40),       # compute on a mapping-only backend
                      (1, legacy_map), (1, v2_bad_token), (1, v2_get), (1, v2_get_missing),
                      (0, b"")])                                      # no-op: state untouched
    assert states == [AEE_EBADSTATE, 0, -1, 0, -1, 0x5A5A5A5A]
    L.htpg_buffer_release(4001)


def test_channel_rejects_bad_layout_but_answers(L, channel):
    h, ch = channel
    b = ch.buf
    b[:] = 0
    b[8:16] = np.frombuffer(struct.pack("<Ii", 0, 100000), np.uint8)    # n_reqs beyond capacity
    b[0] = 1
    t0 = time.time()
    while b[1] != 1:
        assert time.time() - t0 < 10
        time.sleep(0.0005)


def test_backend_lifecycle_codes(L):
    h = ctypes.c_uint64()
    assert L.htp_ops_open(None, ctypes.byref(h)) == 0
    assert L.htp_ops_rms_norm_f32(h, 0, 0, 0, 0, 1, 1) == AEE_EBADSTATE
    scope = ctypes.c_int32()
    assert L.htp_ops_test_ops(h, ctypes.byref(scope)) == AEE_EBADSTATE
    assert L.htp_ops_init_backend_fraction(h, 0, 1) == AEE_EBADPARM
    assert L.htp_ops_init_backend_fraction(h, 3, 2) == AEE_EBADPARM
    assert L.htp_ops_init_mapping_backend(h) == 0
    assert L.htp_ops_rms_norm_f32(h, 0, 0, 0, 0, 1, 1) == AEE_EUNSUPPORTED
    assert L.htp_ops_release_backend(h) == 0
    assert L.htp_ops_rms_norm_f32(h, 0, 0, 0, 0, 1, 1) == AEE_EBADSTATE
    assert L.htp_ops_close(h) == 0
    assert L.htp_ops_close(h) == AEE_EBADSTATE   # stale handle


# ------------------------------------------------------------------ sessions
def test_sessions_and_active_handle(L, monkeypatch):
    assert L.open_dsp_session(3, 0) == 0
    dflt = L.htp_ops_default_session()
    assert dflt and L.get_global_handle() == L.htp_ops_session_handle(dflt)
    monkeypatch.setenv("SD_HTP_MULTI_SESSION", "1")
    s = ctypes.c_void_p()
    assert L.htp_ops_session_open(ctypes.byref(s), 3, None, 1) == 0
    assert L.htp_ops_session_is_reserved(s) == 1
    assert L.htp_ops_session_domain(s) == 3
    assert L.htp_ops_session_init_backend(s) == 0           # mapping-only lease in multi-session mode
    assert L.htp_ops_session_is_initialized(s) == 1
    assert L.htp_ops_set_active_session(s) == 0
    assert L.get_global_handle() == L.htp_ops_session_handle(s)
    assert L.htp_ops_set_default_session() == 0
    assert L.get_global_handle() == L.htp_ops_session_handle(dflt)
    s2 = ctypes.c_void_p()
    assert L.htp_ops_session_open(ctypes.byref(s2), 3, None, 1) == 0
    assert L.htp_ops_session_id(s2) != L.htp_ops_session_id(s)
    L.htp_ops_session_close(s2)
    L.htp_ops_session_close(s)
    assert L.htp_ops_session_handle(None) == 2 ** 64 - 1
    L.close_dsp_session()
    assert not L.htp_ops_default_session()


def _conv_prm(**kw):
    return O.conv_params(**kw)


@pytest.mark.parametrize("change", [dict(kp=32), dict(np_=32), dict(upscale=3), dict(ow_off=1), dict(size=-4)])
def test_conv_payload_validation(L, change):
    """Opcode 17 acceptance rules (op_executor.cc:405-418): -1 for a bad size,
    kp < ic*kh*kw, np < oc, upscale not 1/2, or an output size that does not
    follow from the geometry."""
    prm = _conv_prm(iw=8, ih=8, ic=8, oc=40)
    if "kp" in change:
        prm["kp"] = change["kp"]          # 8*3*3 = 72 > 32
    if "np_" in change:
        prm["np"] = change["np_"]         # oc 40 > 32
    if "upscale" in change:
        prm["upscale"] = change["upscale"]
    if "ow_off" in change:
        prm["ow"] += 1
    payload = htpg.conv_params_bytes(prm)
    if "size" in change:
        payload = payload[:change["size"]]
    rc, _ = run(L, 17, payload)
    assert rc == -1


def test_conv_unmapped_buffers(L):
    prm = _conv_prm(iw=8, ih=8, ic=8, oc=40)
    rc, _ = run(L, 17, htpg.conv_params_bytes(prm, output=(4242, 0), activation=(4243, 0), weight=(4244, 0)))
    assert rc == -1


def _aux(**kw):
    prm = dict(mode=0, count=64, width=16, channels=1, spatial=4, groups=1, batch=1, other_count=16, activation=0)
    prm.update(kw)
    return prm


@pytest.mark.parametrize("prm,wfd,bfd", [
    (_aux(mode=14), -1, -1), (_aux(count=0), -1, -1), (_aux(mode=8, count=63), -1, -1),
    (_aux(mode=2, groups=3, channels=4), -1, -1), (_aux(mode=12, channels=20), -1, -1),
    (_aux(mode=12, channels=40), 5, -1), (_aux(mode=9), -1, -1), (_aux(mode=10, other_count=17), 5, 6),
    (_aux(mode=11, width=15), 5, -1), (_aux(mode=3, other_count=0), 5, -1), (_aux(mode=3, other_count=7), 5, -1),
    (_aux(mode=0, other_count=15), 5, -1)])
def test_model_aux_validation(L, prm, wfd, bfd):
    """Opcode 19 acceptance rules (op_executor.cc:371-395): -1 before any buffer."""
    rc, _ = run(L, 19, htpg.aux_params_bytes(prm, output=(4242, 0), input_=(4243, 0), weight=(wfd, 0),
                                             bias=(bfd, 0)))
    assert rc == -1


def test_model_aux_payload_size(L):
    rc, _ = run(L, 19, htpg.aux_params_bytes(_aux())[:-4])
    assert rc == -1
