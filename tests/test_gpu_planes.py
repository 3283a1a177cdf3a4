"""CPU-epilogue form of opcode 15 on the GPU: hmx_mat_mul_native_w8a8_cpu
writes the raw byte planes of the unsigned-code INT32 accumulators into the
output tensor in the reference's export layout and fills the control block.
Compared byte for byte with the oracle (linear_w8a8.c:205-227, 512-526)."""
import ctypes
import struct

import numpy as np
import pytest
import torch

import htpg
import oracle as O

pytestmark = pytest.mark.gpu

CONTROL_BYTES = 17536   # include/op_reg.h W8A8CpuControl
SCALES_OFF, BATCHES_OFF = 128, 16512

SHAPES = [(1, 256, 128), (16, 4096, 1024), (70, 512, 640), (300, 256, 256), (1000, 512, 1280),
          (4096, 128, 64)]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_planes_and_control_match_oracle(gpu, lib, m, k, n):
    c = O.make_w8a8(11, "cpu-epilogue", m, k, n, 0.01, False, 0,
                    inverse_range=(0.5, 2.0) if m % 2 else None)
    planes, scales, _ = O.w8a8_planes(c.x, c.blob, k, n, kind="omp")
    x = torch.from_numpy(c.x).to(gpu)
    blob = torch.from_numpy(c.blob).to(gpu)
    out = torch.full((m, n), float("nan"), device=gpu)
    control = (ctypes.c_uint8 * CONTROL_BYTES)()
    struct.pack_into("<II", control, 0, 0, 0)
    rc = lib.hmx_mat_mul_native_w8a8_cpu(htpg.ptr(out), htpg.ptr(x), htpg.ptr(blob), m, k, n, control)
    lib.htpg_weight_cache_drop(htpg.ptr(blob))   # cached by address (see the header)
    assert rc == 0, (rc, lib.htpg_last_cuda_error())
    got = out.cpu().numpy().view(np.uint8).reshape(m, n * 4)
    assert np.array_equal(got, planes)
    cb = bytes(control)
    produced, flags, vtcm, act_rows, wcols, wloads = struct.unpack_from("<6I", cb, 0)
    assert produced == 1 and act_rows == m and wcols == n // 64 and wloads == 1
    assert struct.unpack_from("<Q", cb, 24)[0] == k * n
    assert np.array_equal(np.frombuffer(cb, np.float32, m, SCALES_OFF), scales)
    assert struct.unpack_from("<4i", cb, BATCHES_OFF) == (0, m, 0, n // 64)
    assert htpg.check_device() == 0


def test_control_checks(gpu, lib):
    x = torch.zeros(8, 64, device=gpu)
    out = torch.zeros(8, 64, device=gpu)
    blob = torch.from_numpy(O.make_w8a8(11, "c", 8, 64, 64, 0.0, False, 0).blob).to(gpu)
    assert lib.hmx_mat_mul_native_w8a8_cpu(htpg.ptr(out), htpg.ptr(x), htpg.ptr(blob), 8, 64, 64, None) == -12
    control = (ctypes.c_uint8 * CONTROL_BYTES)()
    assert lib.hmx_mat_mul_native_w8a8_cpu(htpg.ptr(out), htpg.ptr(x), htpg.ptr(blob), 4097, 64, 64,
                                           control) == -10


@pytest.mark.parametrize("ctl_kind", [htpg.BUF_HOST, htpg.BUF_DEVICE])
def test_cpu_payload_through_executor(gpu, lib, ctl_kind):
    """Opcode 15 with the 48-byte payload {NativeW8A8Params; control}: host
    buffers for the tensors, the control block in host or device memory."""
    m, k, n = 200, 256, 384
    c = O.make_w8a8(12, "exec-planes", m, k, n, 0.01, False, 0)
    planes, scales, _ = O.w8a8_planes(c.x, c.blob, k, n, kind="omp")
    fds, ptrs = {}, {}

    def alloc(name, nbytes, kind=htpg.BUF_HOST):
        fd, p = ctypes.c_int(), ctypes.c_void_p()
        htpg.check(lib.htpg_buffer_alloc(nbytes, kind, ctypes.byref(fd), ctypes.byref(p)), name)
        fds[name], ptrs[name] = fd.value, p.value

    alloc("out", m * n * 4)
    alloc("act", m * k * 4)
    alloc("cst", c.blob.nbytes)
    alloc("ctl", CONTROL_BYTES, ctl_kind)
    try:
        ctypes.memmove(ptrs["act"], c.x.ctypes.data, m * k * 4)
        ctypes.memmove(ptrs["cst"], c.blob.ctypes.data, c.blob.nbytes)
        payload = struct.pack("<10i", fds["out"], 0, fds["act"], 0, fds["cst"], 0, m, k, n, 0) + \
            struct.pack("<ii", fds["ctl"], 0)
        req = np.frombuffer(struct.pack("<I", 15) + payload, np.uint8).copy()
        rc = lib.execute_op_simple(req.ctypes.data, req.nbytes)
        assert rc == 0, rc
        got = np.empty(m * n * 4, np.uint8)
        ctypes.memmove(got.ctypes.data, ptrs["out"], got.nbytes)
        assert np.array_equal(got.reshape(m, n * 4), planes)
        cb = np.empty(CONTROL_BYTES, np.uint8)
        if ctl_kind == htpg.BUF_HOST:
            ctypes.memmove(cb.ctypes.data, ptrs["ctl"], CONTROL_BYTES)
        else:
            from cuda.bindings import runtime as rt
            err, = rt.cudaMemcpy(cb.ctypes.data, ptrs["ctl"], CONTROL_BYTES, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
            assert err == rt.cudaError_t.cudaSuccess
        assert struct.unpack_from("<I", cb, 0)[0] == 1
        assert np.array_equal(cb[SCALES_OFF:SCALES_OFF + 4 * m].view(np.float32), scales)
        assert struct.unpack_from("<4i", cb, BATCHES_OFF) == (0, m, 0, n // 64)
    finally:
        for fd in fds.values():
            lib.htpg_buffer_release(fd)
