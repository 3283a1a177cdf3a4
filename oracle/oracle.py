"""ctypes front-end of the CPU oracle (oracle/htp_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, never by the library.  See htp_oracle.h for what
the oracle restates (reference linear_w8a8.c / mat_mul.c arithmetic) and how
it is pinned.

Synthetic inputs follow the measurement plan of the five benchmark configurations:
splitmix64 with seed 0x5EED0000 + config_index (0-based), one derived stream
per tensor, Box-Muller normals on FP64 rounded to FP32.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

_libs: dict[str, ctypes.CDLL] = {}


def build(native: bool = False) -> None:
    """Compile the oracle (portable builds; `native` adds the host-tuned OpenMP build)."""
    targets = ["all"] + (["native"] if native else [])
    subprocess.run(["make", "-s", "-C", HERE] + targets, check=True)


def lib(kind: str = "st") -> ctypes.CDLL:
    """kind: 'st' single-thread, 'omp' portable OpenMP, 'native' host-tuned OpenMP."""
    if kind in _libs:
        return _libs[kind]
    path = {
        "st": os.path.join(HERE, "libhtp_oracle.so"),
        "omp": os.path.join(HERE, "libhtp_oracle_omp.so"),
        "native": os.path.join(HERE, "_build", "libhtp_oracle_native.so"),
    }[kind]
    if not os.path.exists(path):
        build(native=(kind == "native"))
    L = ctypes.CDLL(path)
    P, I, S, D, U64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_double, ctypes.c_uint64
    L.orc_fill_normal.argtypes = [P, S, D, D, D, U64]
    L.orc_fill_uniform.argtypes = [P, S, D, D, U64]
    L.orc_fill_int8.argtypes = [P, S, U64]
    L.orc_fill_f16_normal.argtypes = [P, S, D, U64]
    L.orc_f32_to_f16.argtypes = [ctypes.c_float]
    L.orc_f32_to_f16.restype = ctypes.c_uint16
    L.orc_deep_offset.argtypes = [I, I, I]
    L.orc_deep_offset.restype = S
    L.orc_f16_perm_offset.argtypes = [I, I, I]
    L.orc_f16_perm_offset.restype = S
    L.orc_cm_offset.argtypes = [I, I, I]
    L.orc_cm_offset.restype = S
    L.orc_w8a8_blob_bytes.argtypes = [I, I]
    L.orc_w8a8_blob_bytes.restype = S
    L.orc_w8a8_pack.argtypes = [P, P, P, P, I, I, U64]
    L.orc_w8a8_unpack_weight.argtypes = [P, P, I, I]
    L.orc_f16_pack_permuted.argtypes = [P, P, I, I]
    L.orc_quantize_rows.argtypes = [P, P, P, P, I, I]
    L.orc_w8a8_accumulate.argtypes = [P, P, P, I, I, I]
    L.orc_w8a8_linear_rows.argtypes = [P, P, P, P, I, I, I, I, I, P, I, P, P, P]
    L.orc_w8a8_planes.argtypes = [P, P, I, I]
    L.orc_conv2d_nchw_f16.argtypes = [P, P, P, P, P, I]
    L.orc_conv_im2col.argtypes = [P, P, P, I]
    L.orc_model_aux.argtypes = [P, P, P, P, P, ctypes.c_float]
    L.orc_activation.argtypes = [ctypes.c_float, I]
    L.orc_activation.restype = ctypes.c_float
    L.orc_epilogue_activation.argtypes = [ctypes.c_float, I]
    L.orc_epilogue_activation.restype = ctypes.c_float
    L.orc_f16_linear_rows.argtypes = [P, P, P, P, I, I, I, I, I, I, P, I]
    L.orc_qk0_block_bytes.argtypes = [I]
    L.orc_qk0_block_bytes.restype = S
    L.orc_qk0_element.argtypes = [P, I, I]
    L.orc_qk0_element.restype = ctypes.c_uint16
    L.orc_qk0_dequant.argtypes = [P, P, I, I, I]
    L.orc_qk0_quantize.argtypes = [P, P, I, I, I]
    L.orc_qk0_linear_rows.argtypes = [P, P, P, I, I, I, I, I, P, I]
    L.orc_threads.restype = I
    L.orc_set_threads.argtypes = [I]
    _libs[kind] = L
    return L


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ---------------------------------------------------------------- generators
def normal(count, sigma=1.0, outlier_p=0.0, outlier_scale=1.0, seed=0):
    out = np.empty(count, np.float32)
    lib().orc_fill_normal(_p(out), count, sigma, outlier_p, outlier_scale, seed)
    return out


def uniform(count, lo, hi, seed):
    out = np.empty(count, np.float32)
    lib().orc_fill_uniform(_p(out), count, lo, hi, seed)
    return out


def int8_uniform(count, seed):
    out = np.empty(count, np.int8)
    lib().orc_fill_int8(_p(out), count, seed)
    return out


def f16_normal(count, sigma, seed):
    out = np.empty(count, np.uint16)
    lib().orc_fill_f16_normal(_p(out), count, sigma, seed)
    return out


def tensor_seed(config_index: int, tensor: int, layer: int = 0) -> int:
    """Seed of one tensor: 0x5EED0000 + config_index, then a per-tensor stream."""
    return ((0x5EED0000 + config_index) << 16) | (layer << 8) | tensor


# ---------------------------------------------------------------- layouts
def w8a8_pack(w_nk: np.ndarray, sw: np.ndarray, inverse: np.ndarray | None = None, signature: int = 0):
    n, k = w_nk.shape
    blob = np.zeros(lib().orc_w8a8_blob_bytes(k, n), np.uint8)
    w_nk = np.ascontiguousarray(w_nk, np.int8)
    sw = np.ascontiguousarray(sw, np.float32)
    inv = None if inverse is None else np.ascontiguousarray(inverse, np.float32)
    lib().orc_w8a8_pack(_p(blob), _p(w_nk), _p(sw), _p(inv), k, n, signature)
    return blob


def w8a8_unpack(blob: np.ndarray, k: int, n: int) -> np.ndarray:
    w = np.empty((n, k), np.int8)
    lib().orc_w8a8_unpack_weight(_p(w), _p(blob), k, n)
    return w


def blob_inverse(blob: np.ndarray, k: int, n: int) -> np.ndarray:
    """inverse[k] of a constants blob (W8A8Header.inverse_offset = 128 + k*n + 8n)."""
    off = 128 + k * n + 8 * n
    return blob[off:off + 4 * k].view(np.float32).copy()


def f16_pack_permuted(w_kn_bits: np.ndarray) -> np.ndarray:
    k, n = w_kn_bits.shape
    out = np.empty(k * n, np.uint16)
    src = np.ascontiguousarray(w_kn_bits, np.uint16)
    lib().orc_f16_pack_permuted(_p(out), _p(src), k, n)
    return out


# ---------------------------------------------------------------- arithmetic
def quantize_rows(x: np.ndarray, inverse: np.ndarray | None = None, kind="st"):
    m, k = x.shape
    codes = np.empty((m, k), np.uint8)
    scales = np.empty(m, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    inv = None if inverse is None else np.ascontiguousarray(inverse, np.float32)
    lib(kind).orc_quantize_rows(_p(codes), _p(scales), _p(x), _p(inv), m, k)
    return codes, scales


def w8a8_accumulate(codes: np.ndarray, w_nk: np.ndarray, kind="st"):
    m, k = codes.shape
    n = w_nk.shape[0]
    acc = np.empty((m, n), np.int32)
    lib(kind).orc_w8a8_accumulate(_p(acc), _p(np.ascontiguousarray(codes)),
                                  _p(np.ascontiguousarray(w_nk, np.int8)), m, k, n)
    return acc


def w8a8_planes(x, blob, k, n, kind="st"):
    """Oracle opcode-15 CPU-epilogue output: (plane bytes [m][n*4] uint8, row
    scales, unsigned-code INT32 accumulators)."""
    m = x.shape[0]
    inverse = blob_inverse(blob, k, n)
    codes, scales = quantize_rows(x, None if np.all(inverse == 1.0) else inverse, kind)
    w_nk = w8a8_unpack(blob, k, n)
    acc = w8a8_accumulate(codes, w_nk, kind)
    out = np.zeros((m, n * 4), np.uint8)
    lib(kind).orc_w8a8_planes(_p(out), _p(acc), m, n)
    return out, scales, acc


def w8a8_linear(x, blob, k, n, bias=None, channels=None, mode=0, rows=None, kind="st",
                want_intermediates=False):
    """Oracle opcode-15 output for `rows` (all rows if None).

    Returns out ([nrows][n], or [channels][nrows] in mode 3) and, with
    want_intermediates, (codes u8, row scales, signed INT32 accumulators)."""
    m = x.shape[0]
    x = np.ascontiguousarray(x, np.float32)
    channels = n if channels is None else channels
    rows_arr = None if rows is None else np.ascontiguousarray(rows, np.int32)
    nrows = m if rows is None else len(rows_arr)
    out = np.zeros((channels, nrows) if mode == 3 else (nrows, n), np.float32)
    codes = scales = acc = None
    if want_intermediates:
        codes = np.empty((nrows, k), np.uint8)
        scales = np.empty(nrows, np.float32)
        acc = np.empty((nrows, n), np.int32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib(kind).orc_w8a8_linear_rows(_p(out), _p(x), _p(blob), _p(b), m, k, n, channels, mode,
                                   _p(rows_arr), nrows, _p(codes), _p(scales), _p(acc))
    if want_intermediates:
        return out, codes, scales, acc
    return out


def f16_linear(x, wperm, k, n, bias=None, channels=None, mode=0, round_acc_f16=False, rows=None,
               kind="st"):
    m = x.shape[0]
    x = np.ascontiguousarray(x, np.float32)
    channels = n if channels is None else channels
    rows_arr = None if rows is None else np.ascontiguousarray(rows, np.int32)
    nrows = m if rows is None else len(rows_arr)
    out = np.zeros((channels, nrows) if mode == 3 else (nrows, n), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    lib(kind).orc_f16_linear_rows(_p(out), _p(x), _p(np.ascontiguousarray(wperm, np.uint16)), _p(b),
                                  m, k, n, channels, mode, int(round_acc_f16), _p(rows_arr), nrows)
    return out


# ggml types of opcodes 2-4 (quants.h:36-74; op_executor.cc:75-88)
GGML_Q4_0, GGML_Q8_0, GGML_IQ4_NL = 2, 8, 20
QK0_TYPES = {2: GGML_Q4_0, 3: GGML_Q8_0, 4: GGML_IQ4_NL}  # opcode -> weight type


def qk0_block_bytes(wtype: int) -> int:
    return int(lib().orc_qk0_block_bytes(wtype))


def qk0_weight_bytes(wtype: int, k: int, n: int) -> int:
    return k * n // 256 * qk0_block_bytes(wtype)


def qk0_quantize(w_kn: np.ndarray, wtype: int) -> np.ndarray:
    """FP32 [k][n] -> super-block stream (uint8) of the given ggml type."""
    k, n = w_kn.shape
    out = np.zeros(qk0_weight_bytes(wtype, k, n), np.uint8)
    lib().orc_qk0_quantize(_p(out), _p(np.ascontiguousarray(w_kn, np.float32)), wtype, k, n)
    return out


def qk0_random(wtype: int, k: int, n: int, seed: int, sigma: float = 0.02) -> np.ndarray:
    """Seeded super-block stream: an N(0, sigma) weight quantised to the type."""
    return qk0_quantize(normal(k * n, sigma, seed=seed).reshape(k, n), wtype)


def qk0_dequant(src: np.ndarray, wtype: int, k: int, n: int) -> np.ndarray:
    """Super-block stream -> FP16 bits, row-major [n][k]."""
    out = np.zeros((n, k), np.uint16)
    lib().orc_qk0_dequant(_p(out), _p(np.ascontiguousarray(src, np.uint8)), wtype, k, n)
    return out


def qk0_linear(x, src, wtype, k, n, round_acc_f16=False, rows=None, kind="st"):
    m = x.shape[0]
    x = np.ascontiguousarray(x, np.float32)
    rows_arr = None if rows is None else np.ascontiguousarray(rows, np.int32)
    nrows = m if rows is None else len(rows_arr)
    out = np.zeros((nrows, n), np.float32)
    lib(kind).orc_qk0_linear_rows(_p(out), _p(x), _p(np.ascontiguousarray(src, np.uint8)), wtype, m, k, n,
                                  int(round_acc_f16), _p(rows_arr), nrows)
    return out


def epilogue(v: float, mode: int) -> float:
    return lib().orc_epilogue_activation(v, mode)


def max_abs_rel(got: np.ndarray, ref: np.ndarray) -> float:
    """max_i |g_i - o_i| / max(max_j |o_j|, 1e-30) — the tolerance metric of the parity bars."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    denom = max(float(np.max(np.abs(ref))) if ref.size else 0.0, 1e-30)
    return float(np.max(np.abs(got - ref))) / denom if ref.size else 0.0


# ---------------------------------------------------------------- configs
@dataclass
class W8A8Case:
    """One opcode-15 linear: inputs in the reference's formats."""
    name: str
    m: int
    k: int
    n: int
    x: np.ndarray            # [m][k] FP32
    w: np.ndarray            # [n][k] INT8
    sw: np.ndarray           # [n] FP32
    inverse: np.ndarray | None
    bias: np.ndarray | None  # [n] FP32
    mode: int = 0
    channels: int = 0
    blob: np.ndarray = field(default=None, repr=False)

    def __post_init__(self):
        if not self.channels:
            self.channels = self.n
        if self.blob is None:
            self.blob = w8a8_pack(self.w, self.sw, self.inverse, signature=0x5EEDF16 + self.n)

    def ops(self) -> float:
        return 2.0 * self.m * self.n * self.k

    def bytes(self) -> float:
        """Algorithmic HBM bytes: 4MK + KN + 4N + 4MN (+4N bias)."""
        out = 4.0 * self.m * (self.channels if self.mode == 3 else self.n)
        return 4.0 * self.m * self.k + self.k * self.n + 4.0 * self.n + out + \
            (4.0 * self.n if self.bias is not None else 0.0)


@dataclass
class F16Case:
    name: str
    m: int
    k: int
    n: int
    x: np.ndarray            # [m][k] FP32
    w_kn: np.ndarray         # [k][n] FP16 bits
    bias: np.ndarray | None
    mode: int = 0
    channels: int = 0
    wperm: np.ndarray = field(default=None, repr=False)

    def __post_init__(self):
        if not self.channels:
            self.channels = self.n
        if self.wperm is None:
            self.wperm = f16_pack_permuted(self.w_kn)

    def ops(self) -> float:
        return 2.0 * self.m * self.n * self.k

    def bytes(self) -> float:
        """Algorithmic HBM bytes: 4MK + 2KN + 4N (bias) + 4M*channels."""
        return 4.0 * self.m * self.k + 2.0 * self.k * self.n + \
            (4.0 * self.n if self.bias is not None else 0.0) + 4.0 * self.m * self.channels


def make_w8a8(cfg: int, name: str, m: int, k: int, n: int, outlier_p: float, bias: bool, mode: int,
              layer: int = 0, inverse_range: tuple | None = None, m_gen: int | None = None) -> W8A8Case:
    x = normal(m * k, 1.0, outlier_p, 20.0, tensor_seed(cfg, 1, layer)).reshape(m, k)
    w = int8_uniform(n * k, tensor_seed(cfg, 2, layer)).reshape(n, k)
    sw = uniform(n, 1e-3, 1e-2, tensor_seed(cfg, 3, layer))
    b = normal(n, 0.01, 0, 1, tensor_seed(cfg, 4, layer)) if bias else None
    inv = None
    if inverse_range is not None:
        inv = uniform(k, inverse_range[0], inverse_range[1], tensor_seed(cfg, 5, layer))
    return W8A8Case(name, m, k, n, x, w, sw, inv, b, mode)


def config_c1(inverse=False) -> W8A8Case:
    """C1: single W8A8 linear M=256, K=1152, N=4608; 1% x20 outliers."""
    return make_w8a8(0, "C1", 256, 1152, 4608, 0.01, False, 0,
                     inverse_range=(0.5, 2.0) if inverse else None)


def config_c2() -> F16Case:
    """C2: CLIP fc1, opcode 16 mode 2 (bias + QuickGELU), M=77, K=768, N=3072."""
    m, k, n = 77, 768, 3072
    x = normal(m * k, 1.0, 0, 1, tensor_seed(1, 1)).reshape(m, k)
    w = f16_normal(k * n, 0.02, tensor_seed(1, 2)).reshape(k, n)
    b = normal(n, 0.01, 0, 1, tensor_seed(1, 4))
    return F16Case("C2", m, k, n, x, w, b, mode=2)


C3_LAYERS = [  # (name, K, N, bias, mode)
    ("qkv", 1536, 4608, False, 0),
    ("out", 1536, 1536, False, 0),
    ("fc1", 1536, 6144, True, 1),
    ("fc2", 6144, 1536, True, 0),
]


def config_c3(m: int = 4096) -> list[W8A8Case]:
    """C3: DiT block linear stack, M=4096 tokens, hidden 1536; 0.5% x20 outliers."""
    return [make_w8a8(2, name, m, k, n, 0.005, bias, mode, layer=i)
            for i, (name, k, n, bias, mode) in enumerate(C3_LAYERS)]


def config_c4(m: int = 16384) -> W8A8Case:
    """C4: M=16384, K=1536, N=6144 fc1 + bias + GELU; C3's value distributions."""
    return make_w8a8(3, "C4", m, 1536, 6144, 0.005, True, 1)


def config_c5() -> list[W8A8Case]:
    """C5: decode shapes M in {1,4,16}; up K=4096,N=14336; down K=14336,N=4096."""
    cases = []
    for i, (name, k, n) in enumerate([("up", 4096, 14336), ("down", 14336, 4096)]):
        for m in (1, 4, 16):
            c = make_w8a8(4, f"{name}_m{m}", m, k, n, 0.0, False, 0, layer=i)
            cases.append(c)
    return cases


# ---------------------------------------------------------------- opcode 17
CONV_FIELDS = ("iw", "ih", "ic", "oc", "batch", "ow", "oh", "kw", "kh", "sx", "sy", "px", "py", "dx", "dy",
               "kp", "np", "upscale")


def conv_params(iw, ih, ic, oc, batch=1, kw=3, kh=3, sx=1, sy=1, px=1, py=1, dx=1, dy=1, upscale=1,
                kp=None, np_=None) -> dict:
    """NativeConvParams geometry with the output size the reference's executor
    requires (op_executor.cc:410-414) and the smallest legal kp/np."""
    ow = (upscale * iw + 2 * px - dx * (kw - 1) - 1) // sx + 1
    oh = (upscale * ih + 2 * py - dy * (kh - 1) - 1) // sy + 1
    kp = kp or -(-(kw * kh * ic) // 32) * 32
    np_ = np_ or -(-oc // 32) * 32
    return dict(iw=iw, ih=ih, ic=ic, oc=oc, batch=batch, ow=ow, oh=oh, kw=kw, kh=kh, sx=sx, sy=sy, px=px,
                py=py, dx=dx, dy=dy, kp=kp, np=np_, upscale=upscale)


def conv2d(x, wperm, bias, prm: dict, round_acc_f16=False, kind="st"):
    """Oracle opcode-17 output [batch][oc][oh][ow]."""
    p = np.array([prm[f] for f in CONV_FIELDS], np.int32)
    out = np.empty((prm["batch"], prm["oc"], prm["oh"], prm["ow"]), np.float32)
    lib(kind).orc_conv2d_nchw_f16(_p(out), _p(np.ascontiguousarray(x, np.float32)), _p(wperm),
                                  _p(None if bias is None else np.ascontiguousarray(bias, np.float32)),
                                  _p(p), 1 if round_acc_f16 else 0)
    return out


def conv_case(seed, prm: dict, bias=True):
    """Seeded opcode-17 operands: x ~ N(0,1) NCHW, weight FP16 ~ N(0, 0.05)
    logical [oc][ic][kh][kw] placed in the [kp][np] K x N matrix (zero
    padding), bias ~ N(0, 0.01).  Returns x, w_logical (float, FP16 values),
    wperm, bias."""
    b, ic, ih, iw, oc, kh, kw = prm["batch"], prm["ic"], prm["ih"], prm["iw"], prm["oc"], prm["kh"], prm["kw"]
    x = normal(b * ic * ih * iw, 1.0, 0, 1, seed).reshape(b, ic, ih, iw)
    bits = f16_normal(oc * ic * kh * kw, 0.05, seed + 1).reshape(oc, ic, kh, kw)
    wkn = np.zeros((prm["kp"], prm["np"]), np.uint16)
    wkn[:ic * kh * kw, :oc] = bits.reshape(oc, ic * kh * kw).T
    bb = normal(oc, 0.01, 0, 1, seed + 2) if bias else None
    return x, bits.view(np.float16).astype(np.float32), f16_pack_permuted(wkn), bb


# ---------------------------------------------------------------- opcode 19
AUX_FIELDS = ("mode", "count", "width", "channels", "spatial", "groups", "batch", "other_count", "activation")


def model_aux(x, w, b, prm: dict, eps=1e-6, kind="st"):
    """Oracle opcode-19 output (count floats)."""
    p = np.array([prm[f] for f in AUX_FIELDS], np.int32)
    out = np.zeros(prm["count"], np.float32)
    f = lambda a: None if a is None else np.ascontiguousarray(a, np.float32)
    lib(kind).orc_model_aux(_p(out), _p(f(x)), _p(f(w)), _p(f(b)), _p(p), eps)
    return out
