"""Known-answer tests that pin the CPU oracle to the reference.

The reference has no golden FP32 outputs for this path; what it does pin are
integer facts checked by its HMX probe against scalar integer arithmetic
(tests/hmx-probe/integer_tests.c:79-134, study_data.h:1-21, study_dsp.c:70-86)
and the tensor layouts its kernels and host demo address
(linear_w8a8.c:117,281,453-487; src/host/test.c:548-556).  Each test below
restates one of those checks for the oracle.  The FP32 steps are pinned by
hand-computed cases of the reference formulas (linear_w8a8.c:34-59,
mat_mul.c:788-826).
"""
import numpy as np
import pytest

import oracle as O


# ------------------------------------------------------------------ layouts
def test_deep_layout_matches_probe_recipe():
    # study_dsp.c:79-84: tile (t*banks + h)*1024, inside (k/4)*128 + n*4 + k%4,
    # banks = 2 for the N64 groups; groups of 64 columns are n0*K apart
    # (linear_w8a8.c:453).
    K = 96
    for n in range(0, 192, 7):
        for k in range(K):
            g, h, j = n // 64, (n % 64) // 32, n % 32
            t = k // 32
            want = g * 64 * K + (t * 2 + h) * 1024 + ((k % 32) // 4) * 128 + j * 4 + k % 4
            assert O.lib().orc_deep_offset(K, n, k) == want


def test_permuted_f16_layout_matches_host_demo():
    # src/host/test.c:548-556
    K = 64
    for k in range(K):
        for n in range(0, 96, 5):
            i0, i1, j0, j1 = k // 32, k % 32, n // 32, n % 32
            tile = j0 * (K // 32) + i0
            want = tile * 1024 + (i1 & ~1) * 32 + j1 * 2 + (i1 & 1)
            assert O.lib().orc_f16_perm_offset(K, k, n) == want


def test_cm_activation_layout():
    # linear_w8a8.c:281 (tile base (row/64)*64*K), :117 (packed + (c/32)*2048 + r*32)
    K = 128
    for m in range(0, 200, 3):
        for k in range(0, K, 5):
            want = (m // 64) * 64 * K + (k // 32) * 2048 + (m % 64) * 32 + k % 32
            assert O.lib().orc_cm_offset(K, m, k) == want


def test_blob_round_trip_and_header():
    n, k = 192, 96
    w = O.int8_uniform(n * k, 11).reshape(n, k)
    sw = O.uniform(n, 1e-3, 1e-2, 12)
    inv = O.uniform(k, 0.5, 2.0, 13)
    blob = O.w8a8_pack(w, sw, inv, signature=0xABCDEF)
    hdr = blob[:40].view(np.uint32)
    kn = k * n
    assert list(hdr[:9]) == [0x38574D48, 1, k, n, 128, 128 + kn, 128 + kn + 4 * n,
                             128 + kn + 8 * n, 128 + kn + 8 * n + 4 * k]
    assert blob[40:48].view(np.uint64)[0] == 0xABCDEF
    np.testing.assert_array_equal(O.w8a8_unpack(blob, k, n), w)
    sums = blob[128 + kn + 4 * n:128 + kn + 8 * n].view(np.int32)
    np.testing.assert_array_equal(sums, w.astype(np.int32).sum(1))


# ------------------------------------------------------------------ integer KATs
def _accumulate(a_u8, w_s8):
    """acc[m][n] = sum_k a[m][k] * w[n][k] via the oracle."""
    return O.w8a8_accumulate(np.ascontiguousarray(a_u8, np.uint8), np.ascontiguousarray(w_s8, np.int8))


@pytest.mark.parametrize("target", [0, 1, -1, 32767, 32768, 32769, -32767, -32768, -32769, 65535,
                                    65536, 65537, -65535, -65536, -65537, 131071, 131072, 1036320,
                                    -1036320])
def test_int32_boundary_targets(target):
    # integer_tests.c:96-108: reach each target with 255*127 blocks, then a
    # remainder; the UINT8 x INT8 dot product must reproduce it exactly.
    K = 64
    a = np.zeros((1, K), np.uint8)
    w = np.zeros((1, K), np.int8)
    rem, sign, k = abs(target), (-1 if target < 0 else 1), 0
    while rem >= 32385:
        a[0, k], w[0, k] = 255, sign * 127
        rem -= 32385
        k += 1
    if rem >= 127:
        a[0, k], w[0, k] = rem // 127, sign * 127
        rem %= 127
        k += 1
    if rem:
        a[0, k], w[0, k] = rem, sign
    assert _accumulate(a, w)[0, 0] == target


@pytest.mark.parametrize("kt", [1, 2, 3, 4])
def test_zero_point_correction_with_padding(kt):
    # integer_tests.c:111-134: signed activation through zero point 128;
    # got - 128*colsum == sum (a-128)*w, with padded rows/columns and distinct
    # K tiles (depth = kt*32 - 1, the last k is padding).
    m, ncols, depth = 5, 17, kt * 32 - 1
    K, N = kt * 32, 64
    a = np.full((m, K), 128, np.uint8)            # padding codes are the zero point
    w = np.zeros((N, K), np.int8)
    for r in range(m):
        for k in range(depth):
            a[r, k] = (r * 13 + k * 17) % 256
    for k in range(depth):
        for n in range(ncols):
            w[n, k] = (k * 11 + n * 5) % 16 - 8
    acc = _accumulate(a, w)
    colsum = w.astype(np.int64).sum(1)
    expect = (a.astype(np.int64) - 128) @ w.astype(np.int64).T
    np.testing.assert_array_equal(acc.astype(np.int64) - 128 * colsum[None, :], expect)


def test_signed_accumulators_use_blob_column_sums():
    # the operator subtracts (sum_k w) << 7 taken from the constants blob
    # (linear_w8a8.c:159,168): with consistent sums this is sum (code-128)*w
    c = O.make_w8a8(6, "t", 9, 96, 128, 0.01, False, 0)
    _, codes, scales, sacc = O.w8a8_linear(c.x, c.blob, 96, 128, want_intermediates=True)
    np.testing.assert_array_equal(sacc, (codes.astype(np.int64) - 128) @ c.w.astype(np.int64).T)
    # a blob whose stored sums are off by d shifts every accumulator by -128*d
    blob = c.blob.copy()
    kn = 96 * 128
    sums = blob[128 + kn + 4 * 128:128 + kn + 8 * 128].view(np.int32)
    sums[5] += 3
    _, _, _, sacc2 = O.w8a8_linear(c.x, blob, 96, 128, want_intermediates=True)
    np.testing.assert_array_equal(sacc2[:, 5], sacc[:, 5] - 384)
    np.testing.assert_array_equal(np.delete(sacc2, 5, 1), np.delete(sacc, 5, 1))


def _study_hash(x):
    x &= 0xFFFFFFFF
    x ^= x >> 16
    x = (x * 0x7FEB352D) & 0xFFFFFFFF
    x ^= x >> 15
    x = (x * 0x846CA68B) & 0xFFFFFFFF
    return x ^ (x >> 16)


def _study_a(r, k, seed):
    if seed == 0:
        return 129
    if seed in (30, 31):
        return 255
    return _study_hash(r * 7919 + k * 13 + seed * 104729) & 255


def _study_w(k, n, seed):  # INT8 kind (study_data.h:13-20, kind == 1)
    if seed == 0:
        return 1
    if seed == 30:
        return 127
    if seed == 31:
        return -128
    if 12 <= seed < 24:
        return (_study_hash(k * 3571 + n * 23 + seed * 65537) & 255) - 128
    return (_study_hash(k * 3571 + n * 23 + seed * 65537) & 15) - 8


@pytest.mark.parametrize("seed", [0, 3, 12, 17, 23, 30, 31])
@pytest.mark.parametrize("kt", [1, 48])
def test_study_generators_raw_and_signed_sums(seed, kt):
    # study_host.c:160-187: raw = sum a*w, signed = sum (a-128)*w on the study
    # generators (M64, N64 "weight:deep", K up to 6144).  Weight -128 (seed 31)
    # is outside the [-127,127] codes of the operator but valid for the
    # accumulator.
    K, N, M = kt * 32, 64, 64
    a = np.array([[_study_a(r, k, seed) for k in range(K)] for r in range(M)], np.uint8)
    w = np.array([[_study_w(k, n, seed) for k in range(K)] for n in range(N)], np.int64)
    raw = _accumulate(a, w.astype(np.int8))
    np.testing.assert_array_equal(raw, a.astype(np.int64) @ w.T)
    colsum = w.sum(1)
    np.testing.assert_array_equal(raw.astype(np.int64) - 128 * colsum[None, :],
                                  (a.astype(np.int64) - 128) @ w.T)


# ------------------------------------------------------------------ FP32 steps
def test_quantisation_round_half_even_and_clamp():
    # scale = absmax/127 = 1 exactly: u = x + 128, RNE on ties (linear_w8a8.c:50-58)
    x = np.array([[127.0, 0.5, 1.5, -0.5, -1.5, 2.5, -127.0, 0.49999997, 126.5, -126.5]], np.float32)
    codes, scales = O.quantize_rows(x)
    assert scales[0] == np.float32(1.0)
    assert list(codes[0]) == [255, 128, 130, 128, 126, 130, 1, 128, 254, 2]


def test_quantisation_zero_and_tiny_rows():
    x = np.zeros((2, 64), np.float32)
    x[1, 3] = 1e-20
    codes, scales = O.quantize_rows(x)
    assert scales[0] == np.float32(1e-12) and scales[1] == np.float32(1e-12)
    assert (codes == 128).all()          # 1e-20 * 1e12 + 128 rounds to 128


def test_quantisation_uses_ieee_steps():
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((7, 96)) * 3).astype(np.float32)
    inv = rng.uniform(0.5, 2, 96).astype(np.float32)
    codes, scales = O.quantize_rows(x, inv)
    xs = (x * inv).astype(np.float32)
    sc = np.maximum((np.abs(xs).max(1) / np.float32(127)).astype(np.float32), np.float32(1e-12))
    np.testing.assert_array_equal(scales, sc)
    s = (np.float32(1) / sc).astype(np.float32)
    u = ((xs * s[:, None]).astype(np.float32) + np.float32(128)).astype(np.float32)
    u = np.clip(u, 1, 255)
    np.testing.assert_array_equal(codes, np.rint(u).astype(np.uint8))


@pytest.mark.parametrize("mode", [1, 2])
def test_activation_formulas(mode):
    xs = np.linspace(-12, 12, 97)
    for x in xs:
        got = O.epilogue(float(np.float32(x)), mode)
        if mode == 1:
            ref = 0.5 * x * (1 + np.tanh(np.sqrt(2 / np.pi) * (x + 0.044715 * x ** 3)))
        else:
            ref = x / (1 + np.exp(-1.702 * x))
        assert abs(got - ref) <= 1e-5 * max(1.0, abs(ref))
    assert O.epilogue(3.0, 0) == 3.0 and O.epilogue(3.0, 3) == 3.0


def test_w8a8_dequant_order_and_modes():
    # out = fl(fl(float(y) * sw) * rs) then bias, then activation; mode 3 is the
    # cropped channel-major store (mat_mul.c:847-858)
    c = O.make_w8a8(9, "t", 6, 64, 128, 0.0, True, 0)
    out, codes, scales, acc = O.w8a8_linear(c.x, c.blob, 64, 128, want_intermediates=True)
    ref = ((acc.astype(np.float32) * c.sw[None, :]).astype(np.float32) * scales[:, None]).astype(np.float32)
    np.testing.assert_array_equal(out, ref)
    withb = O.w8a8_linear(c.x, c.blob, 64, 128, bias=c.bias, mode=0)
    np.testing.assert_array_equal(withb, (ref + c.bias[None, :]).astype(np.float32))
    chw = O.w8a8_linear(c.x, c.blob, 64, 128, bias=c.bias, channels=100, mode=3)
    assert chw.shape == (100, 6)
    np.testing.assert_array_equal(chw, withb[:, :100].T)


def test_f16_epilogue_matches_fp64_reference():
    m, k, n = 9, 64, 96
    x = O.normal(m * k, 1.0, 0, 1, 21).reshape(m, k)
    w = O.f16_normal(k * n, 0.02, 22).reshape(k, n)
    wperm = O.f16_pack_permuted(w)
    got = O.f16_linear(x, wperm, k, n)
    ref = x.astype(np.float16).astype(np.float64) @ w.view(np.float16).astype(np.float64)
    assert O.max_abs_rel(got, ref) < 1e-6
    got16 = O.f16_linear(x, wperm, k, n, round_acc_f16=True)
    np.testing.assert_array_equal(got16, got.astype(np.float16).astype(np.float32))


def test_row_subset_equals_full():
    c = O.make_w8a8(4, "t", 40, 128, 192, 0.01, True, 1)
    full = O.w8a8_linear(c.x, c.blob, 128, 192, bias=c.bias, mode=1)
    rows = [0, 7, 39, 13]
    sub = O.w8a8_linear(c.x, c.blob, 128, 192, bias=c.bias, mode=1, rows=rows)
    np.testing.assert_array_equal(sub, full[rows])


def test_openmp_build_matches_single_thread():
    c = O.config_c1()
    a = O.w8a8_linear(c.x, c.blob, c.k, c.n)
    b = O.w8a8_linear(c.x, c.blob, c.k, c.n, kind="omp")
    np.testing.assert_array_equal(a, b)


def test_seeded_generators_are_deterministic():
    a = O.normal(1000, 1.0, 0.01, 20.0, 123)
    b = O.normal(1000, 1.0, 0.01, 20.0, 123)
    np.testing.assert_array_equal(a, b)
    assert abs(float(np.std(O.normal(100000, 1.0, 0, 1, 7))) - 1.0) < 0.02
    w = O.int8_uniform(100000, 3)
    assert w.min() == -127 and w.max() == 127


@pytest.mark.parametrize("m,k,n", [(70, 64, 128), (64, 32, 64), (130, 96, 192), (5, 32, 64)])
def test_plane_export_layout(m, k, n):
    """The CPU-epilogue export (linear_w8a8.c:205-227): walking each half's
    byte stream as export_plane_tile lays it out and joining plane p as byte p
    (the readout order of output_tile_impl, :153-163) gives back the
    unsigned-code accumulators sum_k code_u8 * w."""
    c = O.make_w8a8(9, "planes", m, k, n, 0.01, False, 0, inverse_range=(0.5, 2.0))
    planes, scales, acc = O.w8a8_planes(c.x, c.blob, k, n)
    pb = planes.reshape(m, n * 4)
    dec = np.zeros((m, n), np.uint32)
    for t in range((m + 63) // 64):
        rows = min(64, m - t * 64)
        for g in range(n // 64):
            for h in range(2):
                col = (g * 64 + h * 32) * 4
                stream = np.concatenate([pb[t * 64 + r, col:col + 128] for r in range(rows)])
                for p in range(4):
                    plane = stream[p * rows * 32:(p + 1) * rows * 32].reshape(rows, 32).astype(np.uint32)
                    dec[t * 64:t * 64 + rows, g * 64 + h * 32:g * 64 + h * 32 + 32] |= plane << (8 * p)
    assert np.array_equal(dec.view(np.int32), acc)
    codes, sc = O.quantize_rows(c.x, O.blob_inverse(c.blob, k, n))
    w = O.w8a8_unpack(c.blob, k, n).astype(np.int64)
    assert np.array_equal((codes.astype(np.int64) @ w.T).astype(np.int32), acc)
    assert np.array_equal(sc, scales)


def _direct_conv(x, w, bias, prm):
    """fp64 NCHW convolution on FP16-rounded operands, nearest 2x upsample."""
    up = prm["upscale"]
    xu = np.repeat(np.repeat(x.astype(np.float16).astype(np.float64), up, axis=2), up, axis=3)
    b, ic, H, W = xu.shape
    oc, _, kh, kw = w.shape
    out = np.zeros((b, oc, prm["oh"], prm["ow"]))
    for oy in range(prm["oh"]):
        for ox in range(prm["ow"]):
            for ky in range(kh):
                for kx in range(kw):
                    yy = oy * prm["sy"] - prm["py"] + ky * prm["dy"]
                    xx = ox * prm["sx"] - prm["px"] + kx * prm["dx"]
                    if 0 <= yy < H and 0 <= xx < W:
                        out[:, :, oy, ox] += xu[:, :, yy, xx] @ w[:, :, ky, kx].astype(np.float64).T
    if bias is not None:
        out += bias[None, :, None, None]
    return out


@pytest.mark.parametrize("geom", [
    dict(iw=9, ih=7, ic=3, oc=5),                                   # 3x3, pad 1
    dict(iw=6, ih=5, ic=4, oc=40, upscale=2),                       # nearest 2x upsample
    dict(iw=11, ih=9, ic=2, oc=8, sx=2, sy=2, px=0, py=0),          # stride 2, no padding
    dict(iw=10, ih=8, ic=3, oc=7, dx=2, dy=2, px=2, py=2),          # dilation 2
    dict(iw=5, ih=4, ic=33, oc=9, kw=1, kh=1, px=0, py=0, batch=2),  # 1x1, K padding, batch 2
])
def test_conv_oracle_matches_direct_convolution(geom):
    """Opcode 17 (mat_mul.c:2189-2343): the oracle's im2col (the reference's
    gather rule) + FP16 GEMM + channel-major epilogue equals a direct fp64
    convolution of the FP16-rounded operands."""
    prm = O.conv_params(**geom)
    x, wl, wperm, bias = O.conv_case(77, prm)
    got = O.conv2d(x, wperm, bias, prm)
    ref = _direct_conv(x, wl, bias, prm)
    assert got.shape == ref.shape
    assert np.max(np.abs(got - ref)) <= 1e-5 * max(1.0, np.max(np.abs(ref)))


# ---------------------------------------------------------------- opcode 19
def _sig(z):
    return 1.0 / (1.0 + np.exp(-z))


def _act(x, mode):
    x = x.astype(np.float64)
    if mode in (4, 5):
        return x * _sig(x)
    if mode == 1:
        return x * _sig(1.5957691216057308 * (x + 0.044715 * x ** 3))
    return x * _sig(1.702 * x)


def aux_cases():
    rng = np.random.default_rng(5)
    f = lambda *s: rng.standard_normal(s).astype(np.float32)
    C = []
    # (name, prm, x, w, b, reference)
    x = f(6, 96); w = f(96); b = f(96)
    for act in (0, 1):
        mu = x.astype(np.float64).mean(1, keepdims=True); var = ((x - mu) ** 2).mean(1, keepdims=True)
        y = (x - mu) / np.sqrt(var + 1e-6) * w + b
        C.append(("layernorm", dict(mode=0, count=576, width=96, channels=1, spatial=6, groups=1, batch=1,
                                     other_count=96, activation=act), x, w, b, _act(y, 4) if act else y))
    x = f(5, 64); w = f(64)
    y = x / np.sqrt((x.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6) * w
    C.append(("rmsnorm", dict(mode=1, count=320, width=64, channels=1, spatial=5, groups=1, batch=1,
                              other_count=64, activation=0), x, w, None, y))
    x = f(2, 8, 20); w = f(8); b = f(8)
    g = x.reshape(2, 4, 2 * 20).astype(np.float64)
    y = ((g - g.mean(2, keepdims=True)) / np.sqrt(g.var(2, keepdims=True) + 1e-6)).reshape(2, 8, 20)
    y = y * w[None, :, None] + b[None, :, None]
    C.append(("groupnorm", dict(mode=2, count=320, width=1, channels=8, spatial=20, groups=4, batch=2,
                                other_count=8, activation=0), x, w, b, y))
    x = f(200); w = f(50)
    C.append(("add", dict(mode=3, count=200, width=1, channels=1, spatial=1, groups=1, batch=1, other_count=50,
                          activation=0), x, w, None, x + np.tile(w, 4)))
    C.append(("mul", dict(mode=4, count=200, width=1, channels=1, spatial=1, groups=1, batch=1, other_count=50,
                          activation=0), x, w, None, x * np.tile(w, 4)))
    for mode, am in ((5, 4), (6, 1), (7, 2)):
        C.append((f"act{mode}", dict(mode=mode, count=200, width=1, channels=1, spatial=1, groups=1, batch=1,
                                     other_count=0, activation=0), x, None, None, _act(x, am)))
    x = f(2, 5, 7)
    C.append(("transpose", dict(mode=8, count=70, width=5, channels=1, spatial=7, groups=1, batch=2,
                                other_count=0, activation=0), x, None, None, x.transpose(0, 2, 1)))
    x = f(2, 6, 32)
    for shared in (False, True):
        w = f(32) if shared else f(2, 32); b = f(32) if shared else f(2, 32)
        mu = x.astype(np.float64).mean(2, keepdims=True); var = ((x - mu) ** 2).mean(2, keepdims=True)
        v = (x - mu) / np.sqrt(var + 1e-6)
        ww = w[None, None, :] if shared else w[:, None, :]; bb = b[None, None, :] if shared else b[:, None, :]
        C.append((f"modulate{int(shared)}", dict(mode=9, count=384, width=32, channels=1, spatial=6, groups=1,
                                                 batch=2, other_count=32 if shared else 64, activation=0),
                  x, w, b, v + v * ww + bb))
    x = f(2, 4, 32); w = f(2, 32); b = f(2, 4, 32)
    C.append(("gate", dict(mode=10, count=256, width=32, channels=1, spatial=4, groups=1, batch=2, other_count=64,
                           activation=0), x, w, b, x * w[:, None, :] + b))
    for groups in (1, 2):
        x = f(2, 4, 3, 8); pe = f(groups, 4, 8, 2)  # [groups][tokens][dim/2 pairs... as dim*2 floats]
        pe = pe.reshape(groups, 4, 16)
        y = np.zeros((2, 3, 4, 8))
        for bb in range(2):
            for t in range(4):
                m = pe[0 if groups == 1 else bb, t].reshape(4, 4)
                for h in range(3):
                    v = x[bb, t, h].astype(np.float64)
                    for e in range(0, 8, 2):
                        mm = m[e // 2]
                        y[bb, h, t, e] = v[e] * mm[0] + v[e + 1] * mm[1]
                        y[bb, h, t, e + 1] = v[e + 1] * mm[3] + v[e] * mm[2]
        C.append((f"rope{groups}", dict(mode=11, count=192, width=8, channels=3, spatial=4, groups=groups,
                                         batch=2, other_count=2 * 8 * 4 * groups, activation=0), x, pe, None, y))
    x = f(6, 40)
    for act in (0, 1):
        gate = x[:, :16] if act else x[:, 16:32]; up = x[:, 16:32] if act else x[:, :16]
        C.append((f"swiglu{act}", dict(mode=12, count=96, width=16, channels=40, spatial=3, groups=1, batch=2,
                                       other_count=0, activation=act), x, None, None, _act(gate, 5) * up))
        att = f(6, 8)
        C.append((f"swiglu_cat{act}", dict(mode=13, count=144, width=16, channels=40, spatial=3, groups=8, batch=2,
                                           other_count=48, activation=act), x, att, None,
                  np.concatenate([att, _act(gate, 5) * up], axis=1)))
    return C


@pytest.mark.parametrize("case", aux_cases(), ids=lambda c: c[0])
def test_model_aux_oracle(case):
    """Opcode 19 (mat_mul.c:2344-2480): each mode of the oracle against an
    independent fp64 statement of the same operation."""
    name, prm, x, w, b, ref = case
    got = O.model_aux(x, w, b, prm)
    ref = np.asarray(ref, np.float64).reshape(-1)
    assert got.shape == ref.shape
    assert np.max(np.abs(got - ref)) <= 2e-5 * max(1.0, np.max(np.abs(ref))), name


# ----------------------------------------------------------------- opcodes 2-4
# Instruction-level restatement of the reference's per-super-block
# dequantisation (mat_mul.c:389-424 for Q4_0 / IQ4_NL, :488-525 for Q8_0) on
# 128-byte HVX vectors, written from the HVX instruction definitions:
#   vlut16(u.b, v.h, 0) "nomatch": pair.lo.h[i] = v.h[2*(u.b[2i] & 15)],
#                                  pair.hi.h[i] = v.h[2*(u.b[2i+1] & 15)]
#   vunpack (ub->uh, uh->uw, b->h): elements widened in order, first half in lo
#   vlsr(ub, 4):                   each byte shifted right by four
#   qf16 multiply + conversion:    modelled as FP16 rounding of the exact product
# It checks the closed form of the C oracle (orc_qk0_element) element by element.
def _vlut16(u, table):
    return table[2 * (u[0::2] & 15)], table[2 * (u[1::2] & 15)]


def _hvx_superblock(block: np.ndarray, wtype: int) -> np.ndarray:
    ext = np.zeros(512, np.uint8)
    ext[:block.size] = block                       # vmemu reads a full vector past the block
    halves = ext[:128].view(np.uint16)             # vmemu(src[i].scales)
    table = np.zeros(64, np.uint16)
    table[0::2] = halves[:32]                      # lo of vunpack(uh -> uw)
    idx0 = np.array([0, 2] * 32 + [1, 3] * 32, np.uint8)
    s0 = _vlut16(idx0, table)
    s1 = _vlut16(idx0 + 4, table)
    scales = [s0[0], s0[1], s1[0], s1[1]]
    if wtype == O.GGML_Q8_0:
        q = ext[16:16 + 256].view(np.int8)
        vecs = [q[0:64], q[64:128], q[128:192], q[192:256]]
        vecs = [v.astype(np.float32) for v in vecs]
    else:
        levels = (np.arange(16) - 8) if wtype == O.GGML_Q4_0 else np.array(
            [-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113])
        lut = np.zeros(64, np.float16)
        lut[0:32:2] = levels
        lut = lut.view(np.uint16)
        qs = ext[16:144]
        lo = _vlut16(qs, lut)
        hi = _vlut16(qs >> 4, lut)
        vecs = [x.view(np.float16).astype(np.float32) for x in (lo[0], lo[1], hi[0], hi[1])]
    with np.errstate(over="ignore"):              # the largest scale times -127 overflows to -inf
        out = [(vecs[j] * scales[j].view(np.float16).astype(np.float32)).astype(np.float16) for j in range(4)]
    return np.concatenate(out).view(np.uint16)


@pytest.mark.parametrize("wtype", [O.GGML_Q4_0, O.GGML_Q8_0, O.GGML_IQ4_NL])
def test_qk0_superblock_matches_hvx_sequence(wtype):
    L = O.lib()
    bb = O.qk0_block_bytes(wtype)
    assert bb == (272 if wtype == O.GGML_Q8_0 else 144)
    rng = np.random.default_rng(wtype)
    special = np.array([0x0001, 0x03FF, 0x0400, 0x7BFF, 0x8001, 0x3C00, 0xBC00, 0x0000, 0x2E66, 0x1400],
                       np.uint16)                  # subnormals, the largest normal, +-1, zero
    for trial in range(60):
        block = rng.integers(0, 256, bb, dtype=np.uint8)
        sc = rng.normal(0, 0.01, 8).astype(np.float16).view(np.uint16)
        if trial % 3 == 0:
            sc = rng.choice(special, 8)
        block[:16] = sc.view(np.uint8)
        want = _hvx_superblock(block, wtype)
        got = np.array([L.orc_qk0_element(block.ctypes.data, wtype, e) for e in range(256)], np.uint16)
        np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("wtype", [O.GGML_Q4_0, O.GGML_Q8_0, O.GGML_IQ4_NL])
def test_qk0_stream_is_the_packed_f16_weight(wtype):
    """Super-block i dequantises to packed-FP16 elements [256i, 256i+256)
    (mat_mul.c:1700-1709 dequantises chunk nc*k into the FP16 weight buffer
    that core_dot_chunk_fp16 reads in the permuted tile layout)."""
    k, n = 96, 64
    bb = O.qk0_block_bytes(wtype)
    rng = np.random.default_rng(3)
    for _ in range(12):
        src = np.zeros(k * n // 256 * bb, np.uint8)
        blocks = src.reshape(-1, bb)
        sb, e = int(rng.integers(0, blocks.shape[0])), int(rng.integers(0, 256))
        blocks[sb, :16] = np.full(8, 0x3C00, np.uint16).view(np.uint8)     # all scales 1.0
        if wtype == O.GGML_Q8_0:
            blocks[sb, 16 + e] = 3
        else:
            # every other code at level 0 (Q4_0: nibble 8); IQ4_NL has no zero
            # level, so compare against the level of nibble 0 there
            fill = 0x88 if wtype == O.GGML_Q4_0 else 0x00
            blocks[:, 16:] = fill
            v, i = e // 64, e % 64
            byte = 16 + 2 * i + (v & 1)
            nib = 11                                                       # Q4_0: 3, IQ4_NL: 38
            blocks[sb, byte] = (blocks[sb, byte] & 0xF0) | nib if v < 2 else (blocks[sb, byte] & 0x0F) | (nib << 4)
        w = O.qk0_dequant(src, wtype, k, n).view(np.float16).astype(np.float32)   # [n][k]
        f = sb * 256 + e
        tile, o = divmod(f, 1024)
        kk = (tile % (k // 32)) * 32 + (o // 64) * 2 + (o & 1)
        nn = (tile // (k // 32)) * 32 + (o % 64) // 2
        assert O.lib().orc_f16_perm_offset(k, kk, nn) == f
        base = 0.0 if wtype != O.GGML_IQ4_NL else None
        if base is None:
            other = w[(np.arange(n)[:, None] != nn) | (np.arange(k)[None, :] != kk)]
            assert np.all((other == -127.0) | (other == 0.0))
            assert w[nn, kk] == 38.0
        else:
            hit = np.argwhere(w != 0)
            assert hit.tolist() == [[nn, kk]] and w[nn, kk] == 3.0


@pytest.mark.parametrize("wtype", [O.GGML_Q4_0, O.GGML_Q8_0, O.GGML_IQ4_NL])
def test_qk0_quantise_round_trip(wtype):
    k, n = 128, 96
    w = O.normal(k * n, 0.02, seed=11).reshape(k, n)
    q = O.qk0_quantize(w, wtype)
    assert q.size == O.qk0_weight_bytes(wtype, k, n)
    d = O.qk0_dequant(q, wtype, k, n).view(np.float16).astype(np.float32).T
    # scale d = the group's extreme / (-8 | 127 | -127): Q4_0 and IQ4_NL clip the
    # opposite extreme at 7d (113d), Q8_0 rounds to half a step
    bound = {O.GGML_Q4_0: 1.0 / 8, O.GGML_Q8_0: 0.5 / 127, O.GGML_IQ4_NL: 14 / 127}[wtype]
    assert np.max(np.abs(d - w)) <= bound * np.max(np.abs(w)) * 1.01


def test_qk0_linear_uses_the_dequantised_weight():
    k, n, m = 64, 96, 5
    src = O.qk0_random(O.GGML_Q4_0, k, n, seed=2)
    x = O.normal(m * k, 1.0, seed=4).reshape(m, k)
    w = O.qk0_dequant(src, O.GGML_Q4_0, k, n).view(np.float16).astype(np.float64)   # [n][k]
    xh = x.astype(np.float16).astype(np.float64)
    want = xh @ w.T
    got = O.qk0_linear(x, src, O.GGML_Q4_0, k, n)
    assert O.max_abs_rel(got, want) <= 1e-6
    got16 = O.qk0_linear(x, src, O.GGML_Q4_0, k, n, round_acc_f16=True)
    assert O.max_abs_rel(got16, want) <= 1e-3
