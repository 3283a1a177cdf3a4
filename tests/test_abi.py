"""Wire ABI of this library against the reference's headers compiled here.

oracle/_ref/libref_abi.so is the shim oracle/ref_abi_shim.c built from the
reference's include/message.h and include/op_reg.h; oracle/_build/
libour_abi.so is the same shim built from this repository's include/.  Every
struct size, field offset, opcode value and the message validator must agree.
"""
import ctypes
import os
import subprocess

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_SO = os.path.join(REPO, "oracle", "_ref", "libref_abi.so")
OUR_SO = os.path.join(REPO, "oracle", "_build", "libour_abi.so")
REF_PLAN = os.path.join(REPO, "oracle", "_ref", "test-f16-gemm-plan")


class Fact(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("value", ctypes.c_long)]


def _load(path):
    L = ctypes.CDLL(path)
    L.ref_facts.restype = ctypes.POINTER(Fact)
    L.ref_validate_layout.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]
    return L


def _facts(L):
    out, p, i = {}, L.ref_facts(), 0
    while p[i].name:
        out[p[i].name.decode()] = p[i].value
        i += 1
    return out


@pytest.fixture(scope="module")
def shims():
    if not os.path.exists(OUR_SO):
        subprocess.run(["make", "-s", "-C", os.path.join(REPO, "oracle"), "abi"], check=True)
    if not os.path.exists(REF_SO):
        pytest.skip("reference shim not built (the reference tree is not on this machine)")
    return _load(REF_SO), _load(OUR_SO)


def test_layout_facts_identical(shims):
    ref, ours = shims
    fr, fo = _facts(ref), _facts(ours)
    assert len(fr) > 50 and fr.keys() == fo.keys()
    diff = {k: (fr[k], fo[k]) for k in fr if fr[k] != fo[k]}
    assert not diff, diff


def test_known_payload_sizes(shims):
    _, ours = shims
    f = _facts(ours)
    assert f["sizeof.NativeW8A8Params"] == 40
    assert f["sizeof.NativeW8A8ProfileParams"] == 104
    assert f["sizeof.NativeW8A8CpuParams"] == 48
    assert f["sizeof.F16EpilogueParams"] == 56
    assert f["sizeof.MatMulParams"] == 92
    assert f["sizeof.W8A8Header"] == 128
    assert f["enum.HTP_OPS_MAT_MUL_NATIVE_W8A8"] == 15
    assert f["enum.HTP_OPS_MAT_MUL_F16_EPILOGUE"] == 16
    assert f["enum.HTP_OPS_MAT_MUL_PERMUTED_W16A32"] == 1


def _validate(L, buf, cap):
    total = ctypes.c_size_t(0)
    ok = L.ref_validate_layout(buf.ctypes.data, cap, ctypes.byref(total))
    return ok, total.value if ok else None


def test_message_validator_agrees_on_fuzzed_headers(shims):
    ref, ours = shims
    rng = np.random.default_rng(1234)
    agree = accepted = 0
    for trial in range(3000):
        cap = int(rng.integers(8, 512))
        buf = np.zeros((max(cap, 64) + 64 + 3) // 4 * 4, np.uint8)
        n = int(rng.integers(-2, 8))
        hdr = buf.view(np.int32)
        hdr[3] = n
        # offsets: mostly plausible increasing values, sometimes garbage
        base = 16 + 4 * (max(n, 0) + 1)
        offs = [base + int(rng.integers(-8, 16))]
        for _ in range(max(n, 0)):
            offs.append(offs[-1] + int(rng.integers(-4, 40)))
        for i, o in enumerate(offs[:(len(buf) - 16) // 4]):
            hdr[4 + i] = o if rng.random() > 0.05 else int(rng.integers(-100, 10000))
        r1 = _validate(ref, buf, cap)
        r2 = _validate(ours, buf, cap)
        assert r1 == r2, (trial, n, cap, offs)
        agree += 1
        accepted += r1[0]
    assert agree == 3000 and accepted > 100


def test_reference_planner_test_passes_here():
    # tests/test-f16-gemm-plan.c of the reference, built unmodified into oracle/_ref
    if not os.path.exists(REF_PLAN):
        pytest.skip("reference planner test not built on this machine")
    out = subprocess.run([REF_PLAN], capture_output=True, text=True, check=True).stdout
    assert "3348 legal plans" in out
