"""ctypes binding of libhtp_ops_b200.so for the Python harness (tests, bench,
smoke).  The library is plain C: every call passes raw device pointers, sizes
and a cudaStream_t; torch is used by the harness only to own device memory and
streams.  Loading fails loudly when the compiled library is missing: there is
no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
LIB_PATH = os.environ.get("HTPG_LIB") or os.path.join(HERE, "libhtp_ops_b200.so")
INCLUDE = os.path.join(REPO, "include")

# error codes (include/htp_ops_b200.h)
OK, EPAYLOAD, EUNMAPPED, EHEADER = 0, -1, -2, -3
EARGS, ECAPACITY, ECONTROL, ELAUNCH, ENOPLAN = -10, -11, -12, -13, -14
EWATCHDOG, ENOMEM, ESCRATCH, EARCH = -16, -17, -18, -75
BUF_DEVICE, BUF_HOST = 0, 1

_lib = None


def build(jobs: int = 8) -> str:
    subprocess.run(["make", "-s", "-C", HERE, f"-j{jobs}"], check=True)
    return LIB_PATH


def declared_symbols() -> list[str]:
    """Function names declared in include/*.h and include/host/*.h."""
    names = []
    for root, _, files in os.walk(INCLUDE):
        for f in files:
            if not f.endswith(".h"):
                continue
            text = open(os.path.join(root, f)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            text = re.sub(r"#define[^\n]*\n", "\n", text)
            text = re.sub(r"static inline[^{]*\{.*?\n\}", "", text, flags=re.S)
            for m in re.finditer(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(([^;{]*)\)\s*;", text):
                name = m.group(1)
                if name in ("sizeof", "if", "return", "HTPB_STATIC_ASSERT", "__attribute__"):
                    continue
                names.append(name)
    return sorted(set(names))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is not built (run __graft_entry__.build()); "
                           "this library has no CPU fallback")
    L = ctypes.CDLL(LIB_PATH)
    P, I, S, U32, U64, I64 = (ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_uint32,
                              ctypes.c_uint64, ctypes.c_int64)
    sig = {
        "htpg_init": (I, [I]),
        "htpg_version": (I, []),
        "htpg_strerror": (ctypes.c_char_p, [I]),
        "htpg_last_cuda_error": (ctypes.c_char_p, []),
        "htpg_check_device": (I, [P, ctypes.POINTER(U32)]),
        "htpg_quantize_rows": (I, [P, P, P, P, I, I, P]),
        "htpg_w8a8_weights_create": (I, [P, I, I, I, I, P, ctypes.POINTER(P)]),
        "htpg_f16_weights_create": (I, [P, I, I, I, I, P, ctypes.POINTER(P)]),
        "htpg_weights_destroy": (None, [P]),
        "htpg_weights_cols": (I, [P]),
        "htpg_w8a8_run": (I, [P, P, I, P, P, I, I, I, P]),
        "htpg_f16_run": (I, [P, P, I, P, P, I, I, I, P]),
        "htpg_w8a8_run_static": (I, [P, P, I, P, P, I, I, I, P]),
        "htpg_w8a8_run_gather": (I, [P, ctypes.POINTER(P), I, I, P, P, I, I, I, P]),
        "htpg_w8a8_run_planes": (I, [P, P, P, I, P, P]),
        "htpg_conv2d_run": (I, [P, P, P, P, P, P]),
        "htpg_conv_set_chunk_bytes": (I, [S]),
        "hmx_conv2d_nchw_f16": (I, [P, P, P, P, P]),
        "htpg_model_aux_check": (I, [P, I, I]),
        "htpg_model_aux": (I, [P, P, P, P, P, P]),
        "hvx_model_aux_f32": (I, [P, P, P, P, P]),
        "htpg_ipc_export": (I, [P, P]),
        "htpg_ipc_import": (I, [P, ctypes.POINTER(P)]),
        "htpg_ipc_close": (I, [P]),
        "htpg_w8a8_linear": (I, [P, P, P, P, I, I, I, I, I, P]),
        "htpg_f16_linear": (I, [P, P, P, P, I, I, I, I, I, P]),
        "htpg_weight_cache_drop": (None, [P]),
        "htpg_weight_cache_clear": (None, []),
        "htpg_set_profiling": (I, [I]),
        "htpg_set_decode_kernel": (I, [I]),
        "htpg_set_pair_direct": (I, [I]),
        "htpg_set_pair_tail_split": (I, [I]),
        "htpg_set_qk0_decode": (I, [I]),
        "htpg_set_qdec_shape": (I, [I, I]),
        "htpg_qk0_decode_plan_info": (I, [I, I, I, I, I, ctypes.POINTER(I64)]),
        "htpg_last_phase_ms": (I, [ctypes.POINTER(ctypes.c_float)] * 3),
        "htpg_launch_count": (U64, []),
        "htpg_stream_read": (I, [P, S, P]),
        "htpg_debug_simulate_abort": (I, [U32]),
        "htpg_debug_workspaces": (I, [ctypes.POINTER(S), ctypes.POINTER(S)]),
        "htpg_w8a8_profile_fill": (I, [I, I, I, ctypes.c_double, P]),
        "htpg_plan_info": (I, [I, I, I, I, I, ctypes.POINTER(I64)]),
        "htpg_phase_timing": (I, [I]),
        "htpg_phase_timing_read": (I, [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double),
                                       ctypes.POINTER(I)]),
        "htpg_buffer_alloc": (I, [S, I, ctypes.POINTER(I), ctypes.POINTER(P)]),
        "htpg_buffer_register": (I, [I, P, S, I]),
        "htpg_buffer_release": (I, [I]),
        "htpg_buffer_touch": (I, [I]),
        "htpg_buffer_resolve": (P, [I, I64, S, ctypes.POINTER(I)]),
        "execute_op_simple": (I, [P, S]),
        "hmx_mat_mul_native_w8a8": (I, [P, P, P, I, I, I]),
        "hmx_mat_mul_native_w8a8_profiled": (I, [P, P, P, I, I, I, P]),
        "hmx_mat_mul_native_w8a8_cpu": (I, [P, P, P, I, I, I, P]),
        "hmx_mat_mul_f16_epilogue": (I, [P, P, P, P, I, I, I, I, I]),
        "hmx_mat_mul_permuted_w16a32": (I, [P, P, P, I, I, I]),
        "hmx_mat_mul_permuted_qk_0_d16a32": (I, [P, P, P, I, I, I, I]),
        "htpg_qk0_weight_bytes": (S, [I, I, I]),
        "htpg_qk0_linear": (I, [P, P, P, I, I, I, I, P]),
        "htpg_qk0_weights_create": (I, [P, I, I, I, P, ctypes.POINTER(P)]),
        "htpg_qk0_run": (I, [P, P, P, I, P]),
        "htpg_qk0_dequantize": (I, [P, P, I, I, I, P]),
        "htpg_qk0_plan_info": (I, [I, I, I, I, I, ctypes.POINTER(I64)]),
        "htp_ops_open": (I, [ctypes.c_char_p, ctypes.POINTER(U64)]),
        "htp_ops_close": (I, [U64]),
        "htp_ops_init_backend": (I, [U64]),
        "htp_ops_init_backend_fraction": (I, [U64, U32, U32]),
        "htp_ops_init_mapping_backend": (I, [U64]),
        "htp_ops_release_backend": (I, [U64]),
        "htp_ops_create_channel": (I, [U64, ctypes.c_int32, U32]),
        "htp_ops_create_channel_with_token": (I, [U64, U64, ctypes.c_int32, U32]),
        "htp_ops_destroy_channel": (I, [U64]),
        "htp_ops_rms_norm_f32": (I, [U64, I, I, I, I, I, I]),
        "htp_ops_mat_mul_permuted_w16a32": (I, [U64, I, I, I, I, I, I, I, I, I]),
        "htp_ops_mat_mul_permuted_w16a32_trace": (I, [U64, I, I, I, I, I, I, I, I, I] + [ctypes.POINTER(U64)] * 3),
        "htp_ops_test_ops": (I, [U64, ctypes.POINTER(ctypes.c_int32)]),
        "htp_ops_session_open": (I, [ctypes.POINTER(P), I, ctypes.c_char_p, I]),
        "htp_ops_default_session": (P, []),
        "htp_ops_session_init_backend": (I, [P]),
        "htp_ops_session_acquire_backend": (I, [P]),
        "htp_ops_session_release_backend": (I, [P]),
        "htp_ops_session_create_channel": (I, [P, I, ctypes.c_uint]),
        "htp_ops_session_create_channel_with_token": (I, [P, I, ctypes.c_uint]),
        "htp_ops_session_destroy_channel": (I, [P]),
        "htp_ops_session_handle": (U64, [P]),
        "htp_ops_set_active_session": (I, [P]),
        "htp_ops_set_default_session": (I, []),
        "htp_ops_session_id": (U32, [P]),
        "htp_ops_session_domain": (U32, [P]),
        "htp_ops_session_is_reserved": (I, [P]),
        "htp_ops_session_is_initialized": (I, [P]),
        "htp_ops_session_has_channel": (I, [P]),
        "htp_ops_session_close": (None, [P]),
        "open_dsp_session": (I, [I, I]),
        "close_dsp_session": (None, []),
        "get_global_handle": (U64, []),
        "init_htp_backend": (None, []),
        "release_htp_backend": (I, []),
        "create_htp_message_channel": (I, [I, ctypes.c_uint]),
        "destroy_htp_message_channel": (I, []),
        "htp_ops_rpc_rms_norm_f32": (I, [I] * 6),
        "htp_ops_rpc_mat_mul_permuted_w16a32": (I, [I] * 9),
        "htp_ops_rpc_mat_mul_permuted_w16a32_session": (I, [P] + [I] * 9),
        "htp_ops_rpc_mat_mul_permuted_w16a32_trace_session": (I, [P] + [I] * 9 + [ctypes.POINTER(U64)] * 3),
        "htp_ops_f16_epilogue_version": (I, []),
        "htp_ops_native_model_version": (I, []),
        "htp_ops_dit_aux_version": (I, []),
        "htp_ops_dit_concat_version": (I, []),
        "htp_ops_w8a8_epilogue_version": (I, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        L = lib()
        raise RuntimeError(f"{what}: {rc} ({L.htpg_strerror(rc).decode()}) "
                           f"{L.htpg_last_cuda_error().decode()}")


def ptr(t) -> int | None:
    """Device (or host) address of a torch tensor / numpy array, None for None."""
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    return t.ctypes.data


def stream_ptr(stream=None) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else stream


class Weights:
    """A prepared (repacked) weight owned by the library."""

    def __init__(self, handle: int, cols: int):
        self.handle = handle
        self.cols = cols

    def __del__(self):
        if self.handle and _lib is not None:
            _lib.htpg_weights_destroy(self.handle)
            self.handle = None


def w8a8_weights(blob_dev, k: int, n: int, n0: int = 0, n_cols: int = 0, stream=None) -> Weights:
    h = ctypes.c_void_p()
    check(lib().htpg_w8a8_weights_create(ptr(blob_dev), k, n, n0, n_cols, stream_ptr(stream),
                                         ctypes.byref(h)), "htpg_w8a8_weights_create")
    return Weights(h.value, lib().htpg_weights_cols(h.value))


def f16_weights(wperm_dev, k: int, n: int, n0: int = 0, n_cols: int = 0, stream=None) -> Weights:
    h = ctypes.c_void_p()
    check(lib().htpg_f16_weights_create(ptr(wperm_dev), k, n, n0, n_cols, stream_ptr(stream),
                                        ctypes.byref(h)), "htpg_f16_weights_create")
    return Weights(h.value, lib().htpg_weights_cols(h.value))


def w8a8_run(w: Weights, out, x, bias=None, m=None, channels=0, mode=0, ldo=0, stream=None) -> int:
    m = x.shape[0] if m is None else m
    return lib().htpg_w8a8_run(w.handle, ptr(out), ldo, ptr(x), ptr(bias), m, channels, mode,
                               stream_ptr(stream))


def f16_run(w: Weights, out, x, bias=None, m=None, channels=0, mode=0, ldo=0, stream=None) -> int:
    m = x.shape[0] if m is None else m
    return lib().htpg_f16_run(w.handle, ptr(out), ldo, ptr(x), ptr(bias), m, channels, mode,
                              stream_ptr(stream))


PLAN_FIELDS = ("swap", "bn", "splits", "tiles_a", "tiles_b", "kb_total", "kb_per_split",
               "units", "grid", "smem", "full_units", "tail_s")


def plan_info(kind: int, m: int, n: int, k: int, sms: int = 148) -> dict:
    out = (ctypes.c_int64 * 12)()
    check(lib().htpg_plan_info(kind, m, n, k, sms, out), "htpg_plan_info")
    return dict(zip(PLAN_FIELDS, list(out)))


def set_decode_kernel(which: int) -> None:
    """0: W8A8 problems with m <= 16 run the register-fed decode kernel (the
    default); 1: they run the swapped tcgen05 kernel.  Results are identical."""
    check(lib().htpg_set_decode_kernel(which), "htpg_set_decode_kernel")


def set_qk0_decode(which: int) -> None:
    """0 (default): opcode 2-4 problems with m <= 32 run the register-fed
    kernel where it is the faster one, else the tcgen05 kernel; 1: always the
    tcgen05 kernel; 2: the register-fed kernel for every m <= 32."""
    check(lib().htpg_set_qk0_decode(which), "htpg_set_qk0_decode")


def set_qdec_shape(per_sm: int = 0, tiles: int = 0) -> None:
    """Force the register-fed opcode 2-4 decode kernel's launch shape (CTAs
    per SM 1 or 2, weight tiles per CTA 16, 8 or 4); (0, 0) restores the
    planner's choice."""
    check(lib().htpg_set_qdec_shape(per_sm, tiles), "htpg_set_qdec_shape")


def set_pair_tail_split(on: bool) -> None:
    """True (default): swapped CTA-pair plans cut the tiles of a mostly idle
    last round into K pieces (exact INT32 hand-off); False: whole tiles only.
    Results are identical."""
    check(lib().htpg_set_pair_tail_split(1 if on else 0), "htpg_set_pair_tail_split")


def set_pair_direct(on: bool) -> None:
    """True (default): W8A8 CTA-pair problems with a row-major output run in the
    swapped orientation with stores straight from registers; False: the normal
    orientation with staged TMA stores.  Results are identical."""
    check(lib().htpg_set_pair_direct(1 if on else 0), "htpg_set_pair_direct")


def qk0_plan_info(weight_type: int, m: int, n: int, k: int, sms: int = 148) -> dict:
    """Plan of the fused small-M opcode 2-4 kernel."""
    out = (ctypes.c_int64 * 6)()
    check(lib().htpg_qk0_plan_info(weight_type, m, n, k, sms, out), "htpg_qk0_plan_info")
    return dict(zip(("bn", "tiles_a", "tiles_b", "kb_total", "grid", "smem"), list(out)))


def qk0_decode_plan_info(weight_type: int, m: int, n: int, k: int, sms: int = 148) -> dict:
    """Plan of the register-fed opcode 2-4 decode kernel (m <= 32)."""
    out = (ctypes.c_int64 * 8)()
    check(lib().htpg_qk0_decode_plan_info(weight_type, m, n, k, sms, out), "htpg_qk0_decode_plan_info")
    return dict(zip(("per_sm", "tiles", "ntiles", "ktiles", "splits", "grid", "slice", "smem"), list(out)))


def qk0_weights(weight_dev, weight_type: int, k: int, n: int, stream=None) -> Weights:
    """Prepared opcode 2-4 weight (stage records) from the reference's super-block stream."""
    h = ctypes.c_void_p()
    check(lib().htpg_qk0_weights_create(ptr(weight_dev), k, n, weight_type, stream_ptr(stream), ctypes.byref(h)),
          "htpg_qk0_weights_create")
    return Weights(h.value, n)


def qk0_run(w: Weights, out, x, m: int, stream=None) -> int:
    return lib().htpg_qk0_run(w.handle, ptr(out), ptr(x), m, stream_ptr(stream))


def qk0_linear(out, x, weight, weight_type: int, m: int, k: int, n: int, stream=None) -> int:
    """Opcodes 2-4 on device tensors: out[m][n] = fp16(x) * dequant(weight)."""
    return lib().htpg_qk0_linear(ptr(out), ptr(x), ptr(weight), m, k, n, weight_type, stream_ptr(stream))


def phase_timing_read() -> tuple[float, float, int]:
    a, g, n = ctypes.c_double(), ctypes.c_double(), ctypes.c_int()
    check(lib().htpg_phase_timing_read(ctypes.byref(a), ctypes.byref(g), ctypes.byref(n)),
          "htpg_phase_timing_read")
    return a.value, g.value, n.value


def check_device(stream=None) -> int:
    flags = ctypes.c_uint32(0)
    return lib().htpg_check_device(stream_ptr(stream), ctypes.byref(flags))


# ------------------------------------------------------------------ formats
# Host-side packers of the reference's weight formats (what the caller's
# offline packer produces): the W8A8 constants blob (include/op_reg.h
# W8A8Header; INT8 weights in the HMX deep N64 layout of
# src/dsp/ops/linear_w8a8.c:453-487) and the permuted FP16 tile layout
# (src/host/test.c:548-556).
def pack_w8a8_constants(w_nk, sw, inverse=None, signature: int = 0):
    """w_nk: [N][K] int8, sw: [N] float32, inverse: [K] float32 or None (ones)."""
    import numpy as np
    w_nk = np.ascontiguousarray(w_nk, np.int8)
    n, k = w_nk.shape
    assert n % 64 == 0 and k % 32 == 0
    kn = k * n
    bytes_ = 128 + kn + 8 * n + 4 * k
    blob = np.zeros(bytes_, np.uint8)
    hdr = np.zeros(10, np.uint32)
    hdr[:] = [0x38574D48, 1, k, n, 128, 128 + kn, 128 + kn + 4 * n, 128 + kn + 8 * n, bytes_, 0]
    blob[:40] = hdr.view(np.uint8)
    blob[40:48] = np.array([signature], np.uint64).view(np.uint8)
    # n = g*64 + h*32 + j, k = t*32 + q*4 + r  ->  [g][t][h][q][j][r]
    deep = w_nk.reshape(n // 64, 2, 32, k // 32, 8, 4).transpose(0, 3, 1, 4, 2, 5)
    blob[128:128 + kn] = deep.reshape(-1).view(np.uint8)
    blob[128 + kn:128 + kn + 4 * n] = np.ascontiguousarray(sw, np.float32).view(np.uint8)
    sums = w_nk.astype(np.int32).sum(axis=1).astype(np.int32)
    blob[128 + kn + 4 * n:128 + kn + 8 * n] = sums.view(np.uint8)
    inv = np.ones(k, np.float32) if inverse is None else np.ascontiguousarray(inverse, np.float32)
    blob[128 + kn + 8 * n:] = inv.view(np.uint8)
    return blob


def pack_f16_permuted(w_kn_bits):
    """w_kn_bits: [K][N] FP16 bit patterns (uint16) -> permuted 32x32 tiles."""
    import numpy as np
    w = np.ascontiguousarray(w_kn_bits, np.uint16)
    k, n = w.shape
    assert k % 32 == 0 and n % 32 == 0
    # k = t*32 + p*2 + b, n = s*32 + j  ->  [s][t][p][j][b]
    return w.reshape(k // 32, 16, 2, n // 32, 32).transpose(3, 0, 1, 4, 2).reshape(-1).copy()


# ------------------------------------------------------------------ sharding
# Column (N) tensor parallelism for the large linears: rank r owns output
# columns [r*N/w, (r+1)*N/w) -- whole 64-column groups of the constants blob --
# and the full row-major output is reassembled from the gathered shards.
def column_range(n: int, world: int, rank: int, granule: int = 64) -> tuple[int, int]:
    """(first column, columns) owned by `rank`; N must split into whole granules."""
    if n % (granule * world):
        raise ValueError(f"N={n} does not split into {world} shards of whole {granule}-column groups")
    n_loc = n // world
    return rank * n_loc, n_loc


def assemble_columns(full, gathered) -> None:
    """gathered: [world][M][N/world] shards (all-gather order) -> full: [M][N] row-major."""
    world, m, n_loc = gathered.shape
    full.view(m, world, n_loc).copy_(gathered.permute(1, 0, 2))


IPC_HANDLE_BYTES = 72


def ipc_export(t) -> bytes:
    """72-byte CUDA IPC handle (+ offset) of a device tensor's storage."""
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    check(lib().htpg_ipc_export(ptr(t), buf), "htpg_ipc_export")
    return buf.raw


def ipc_import(handle: bytes) -> int:
    """Device address, in this process, of a peer's exported buffer."""
    p = ctypes.c_void_p()
    check(lib().htpg_ipc_import(ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES), ctypes.byref(p)),
          "htpg_ipc_import")
    return p.value


# ------------------------------------------------------------------ opcode 17
CONV_FIELDS = ("iw", "ih", "ic", "oc", "batch", "ow", "oh", "kw", "kh", "sx", "sy", "px", "py", "dx", "dy",
               "kp", "np", "upscale")


def conv_params_bytes(prm: dict, output=(-1, 0), activation=(-1, 0), weight=(-1, 0), bias=(-1, 0)) -> bytes:
    """124-byte NativeConvParams (include/op_reg.h) with the timing fields zero."""
    import struct
    bufs = struct.pack("<8i", *output, *activation, *weight, *bias)
    return bufs + struct.pack("<18i", *[prm[f] for f in CONV_FIELDS]) + b"\0" * 20


# ------------------------------------------------------------------ opcode 19
AUX_FIELDS = ("mode", "count", "width", "channels", "spatial", "groups", "batch", "other_count", "activation")


def aux_params_bytes(prm: dict, eps: float = 1e-6, output=(-1, 0), input_=(-1, 0), weight=(-1, 0),
                     bias=(-1, 0)) -> bytes:
    """76-byte NativeAuxParams (include/op_reg.h), elapsed_us zero."""
    import struct
    return (struct.pack("<8i", *output, *input_, *weight, *bias) +
            struct.pack("<9i", *[prm[f] for f in AUX_FIELDS]) + struct.pack("<fi", eps, 0))
