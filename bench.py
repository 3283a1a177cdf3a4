#!/usr/bin/env python
"""Benchmark of the B200 linear-operator path (the driver's contract).

Workload (default, every N): configuration C4 — W8A8 MLP fc1 with bias +
GELU(tanh) epilogue, M=16384 tokens, K=1536, N=6144, column-sharded over the
N GPUs (N/world columns per GPU).  For N > 1 the output exchange is fused into
the GEMM (default, --exchange fused): the epilogue stores every finished tile
into every rank's row-major [M][N] output over NVLink, and a stream-ordered
NCCL all-reduce of one token orders the step; --exchange nccl keeps the NCCL
all-gather + reassembly baseline.  One step = quantise the activation rows,
the tcgen05 INT8 GEMM with the fused dequant/bias/GELU epilogue (and its
stores to the peers).  Metric: whole-job INT8 TOPS (2*M*N*K per step / device
time, max over ranks).

* value        device-resident inputs; per-step CUDA-event time (L2 flushed
               between steps by a 256 MiB write + read-back outside the timed
               events; a bounded sleep kernel lets the host queue the timed
               steps ahead, so launch gaps are not counted).
* e2e          the same operator through the reference-facing API: an opcode-15
               request (56-byte epilogue payload) posted on the shared-memory
               message channel with host (pinned) buffers; the receiver copies
               the activation in and the output out every step.
* roofline     the GEMM kernel's algorithmic bytes / ops per launch over its
               average event-timed duration inside the timed region.
* cpu_baseline the CPU oracle (restatement of the reference arithmetic; the
               reference itself only builds for a Hexagon DSP) on a bounded row
               sample of the same workload, all host threads.

`--impl reference` times that CPU implementation alone (rank 0), as the
reference arm.
"""
from __future__ import annotations

import argparse
import ctypes
import faulthandler
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "htp-ops-lib-sd.cpp_b200")
sys.path.insert(0, PKG)

M_C4, K_C4, N_C4 = 16384, 1536, 6144
FLUSH_BYTES = 256 << 20
L2_NOTE = ("256 MiB buffer written then read back between steps (outside the timed events): "
           "the next step starts from a cold L2 holding only clean lines")
NVLINK_GBS = 770.0   # peer copy per direction measured with `bench.py --peer-copy` (771-775 GB/s; nominal 900)
SLEEP_CYCLES = 20_000_000   # ~10 ms of torch's bounded sleep kernel ahead of a timed loop


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", 0)), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi samples (200 ms) while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ inputs
# ------------------------------------------------------------------ seeded inputs
# The benchmark's seeded generator: splitmix64 streams, one per tensor, seeded
# ((0x5EED0000 + config index) << 16) | (layer << 8) | tensor; normals by
# Box-Muller on FP64 (u1 = 1 - u, u2 = u; with outliers each pair of values
# also draws one uniform per value, x20 below p), INT8 weights as
# (splitmix64 % 255) - 127, column scales U[1e-3, 1e-2).  Vectorised with
# numpy (the k-th value of a stream is mix(seed + k * 0x9E3779B97F4A7C15)).
def _splitmix(seed, count):
    import numpy as np
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + np.arange(1, count + 1, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def _unit(v):
    import numpy as np
    return (v >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)


def seeded_normal(count, sigma, outlier_p, scale, seed):
    import numpy as np
    pairs = (count + 1) // 2
    per = 4 if outlier_p > 0 else 2
    r = _splitmix(seed, pairs * per).reshape(pairs, per)
    u1, u2 = 1.0 - _unit(r[:, 0]), _unit(r[:, 1])
    rad = np.sqrt(-2.0 * np.log(u1))
    z = np.stack([rad * np.cos(2.0 * np.pi * u2), rad * np.sin(2.0 * np.pi * u2)], 1) * sigma
    if outlier_p > 0:
        z = np.where(np.stack([_unit(r[:, 2]), _unit(r[:, 3])], 1) < outlier_p, z * scale, z)
    return z.reshape(-1)[:count].astype(np.float32)


def tensor_seed(config_index, tensor, layer=0):
    return ((0x5EED0000 + config_index) << 16) | (layer << 8) | tensor


def seeded_c4_inputs(torch, dev, m, k, n, config_index=3, outlier_p=0.005):
    """C4's tensors from the benchmark's seeds (the same bytes the CPU oracle's
    generator gives): x [m][k], W int8 [n][k], column scales, bias."""
    import numpy as np
    import htpg
    x = seeded_normal(m * k, 1.0, outlier_p, 20.0, tensor_seed(config_index, 1)).reshape(m, k)
    w = ((_splitmix(tensor_seed(config_index, 2), n * k) % np.uint64(255)).astype(np.int16) - 127).astype(
        np.int8).reshape(n, k)
    sw = (1e-3 + (1e-2 - 1e-3) * _unit(_splitmix(tensor_seed(config_index, 3), n))).astype(np.float32)
    bias = seeded_normal(n, 0.01, 0.0, 1.0, tensor_seed(config_index, 4))
    blob = htpg.pack_w8a8_constants(w, sw, None, signature=tensor_seed(config_index, 2))
    return (torch.from_numpy(x).to(dev), torch.from_numpy(blob).to(dev), torch.from_numpy(bias).to(dev), blob,
            bias)


def make_c4_inputs(torch, dev, m, k, n, seed=0x5EED0003, outlier_p=0.005):
    """Seeded synthetic C4 tensors with the benchmark's value distributions:
    X ~ N(0,1) with 0.5% of entries x20, W int8 uniform [-127,127], column
    scales U[1e-3,1e-2], bias N(0,0.01)."""
    import numpy as np
    import htpg
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn(m, k, device=dev, generator=g)
    x = torch.where(torch.rand(m, k, device=dev, generator=g) < outlier_p, x * 20.0, x).contiguous()
    gc = torch.Generator()
    gc.manual_seed(seed + 1)
    w = torch.randint(-127, 128, (n, k), generator=gc, dtype=torch.int16).to(torch.int8).numpy()
    sw = (torch.rand(n, generator=gc) * 9e-3 + 1e-3).numpy().astype(np.float32)
    bias = (torch.randn(n, generator=gc) * 0.01).to(dev)
    blob = htpg.pack_w8a8_constants(w, sw, None, signature=seed)
    return x, torch.from_numpy(blob).to(dev), bias, blob


class L2Flush:
    """Evicts the L2 between timed steps: a write of a buffer twice the L2's
    size, then a read of it, so no dirty line of the flush is left for the
    next step's kernels to write back."""

    def __init__(self, torch, dev):
        self.buf = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
        self.sink = torch.empty((), dtype=torch.float32, device=dev)
        self.torch = torch

    def __call__(self):
        self.buf.zero_()
        self.torch.sum(self.buf, dim=0, out=self.sink)


# ------------------------------------------------------------------ suite
def _w8a8_operands(torch, htpg, dev, m, k, n, seed, outlier_p, bias):
    """Seeded W8A8 operands (the benchmark's value distributions) and prepared weights."""
    x, blob_dev, b, _ = make_c4_inputs(torch, dev, m, k, n, seed=seed, outlier_p=outlier_p)
    return x, htpg.w8a8_weights(blob_dev, k, n), (b if bias else None), blob_dev


def suite(torch, L, htpg, dev, flush, reps=20, only=None):
    """Per-config device times of the other benchmark configurations (one GPU): C1,
    C2, the four C3 DiT linears and the six C5 decode linears.  Each run is the
    whole operator (activation pass + GEMM), timed with CUDA events on the
    launching stream, the L2 flushed (256 MiB written and read back) before
    every run, the stream held by a bounded sleep kernel while the host queues
    the runs; the median of `reps` runs.  `host_latency_us` is one call on an
    idle GPU, host work included.  For the decode shapes `stream_us` is the
    per-linear time of back-to-back runs over six operand sets (352 MB of
    weights, more than the L2), the throughput a sequence of decode linears
    sees.  Algorithmic bytes: W8A8 4MK + KN + 4N + 4MN
    (+4N bias); F16 4MK + 2KN + 4N + 4MN."""
    import numpy as np
    hbm, bf16, _, _ = peaks()
    int8_peak = 2.0 * bf16
    stream = torch.cuda.current_stream()
    res = {}

    def timed(fn):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
        for _ in range(3):
            fn()
        # host-inclusive latency: one call at a time on an idle GPU
        lat = []
        for _ in range(5):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            fn()
            torch.cuda.synchronize()
            lat.append((time.perf_counter() - t0) * 1e6)
        # device time: a bounded sleep kernel holds the stream while the host
        # queues every run, so no run waits for its own launch
        def pass_us():
            torch.cuda._sleep(SLEEP_CYCLES)
            for a, b in ev:
                flush()
                a.record(stream)
                fn()
                b.record(stream)
            torch.cuda.synchronize()
            return statistics.median(a.elapsed_time(b) for a, b in ev) * 1e3
        us = pass_us()
        # the split between the activation pass and the GEMM comes from a second
        # pass with the library's phase events (which serialise the two kernels)
        L.htpg_phase_timing(1)
        htpg.phase_timing_read()
        pass_us()
        L.htpg_phase_timing(0)
        act_ms, gemm_ms, runs = htpg.phase_timing_read()
        return us, act_ms * 1e3 / max(runs, 1), gemm_ms * 1e3 / max(runs, 1), statistics.median(lat)

    def stream_us(fns):
        """Back-to-back runs over rotating operand sets larger than the L2 (no
        flush, no events between runs): the per-operator time of a sequence of
        linears, each reading its weight from HBM."""
        for f in fns:
            f()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        runs = 8 * len(fns)
        torch.cuda._sleep(SLEEP_CYCLES)
        a.record(stream)
        for i in range(runs):
            fns[i % len(fns)]()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b) * 1e3 / runs

    def record(name, m, k, n, timing, nbytes, peak_ops):
        us, act_us, gemm_us, lat_us = timing
        ops = 2.0 * m * n * k
        t_tc, t_hbm = ops / (peak_ops * 1e12), nbytes / (hbm * 1e9)
        res[name] = {"M": m, "K": k, "N": n, "us": us, "act_us": act_us, "gemm_us": gemm_us,
                     "host_latency_us": lat_us,
                     "TOPS": ops / us / 1e6, "GBps": nbytes / us / 1e3,
                     "tensor_frac": ops / us / 1e6 / peak_ops, "hbm_frac": nbytes / us / 1e3 / hbm,
                     "bound": "tensor" if t_tc >= t_hbm else "hbm",
                     "roofline_frac": max(t_tc, t_hbm) / (us * 1e-6)}

    def w8a8_case(name, m, k, n, seed, outlier_p, mode, bias, sets=1):
        if only and name != only:
            return
        x, w, b, keep = _w8a8_operands(torch, htpg, dev, m, k, n, seed, outlier_p, bias)
        out = torch.empty(m, n, dtype=torch.float32, device=dev)
        tm = timed(lambda: htpg.check(htpg.w8a8_run(w, out, x, b, mode=mode), name))
        nbytes = 4 * m * k + k * n + 4 * n + 4 * m * n + (4 * n if bias else 0)
        record(name, m, k, n, tm, nbytes, int8_peak)
        if sets > 1:
            ops = [(x, w, b)] + [_w8a8_operands(torch, htpg, dev, m, k, n, seed + 0x100 * i, outlier_p, bias)[:3]
                                 for i in range(1, sets)]
            t = stream_us([lambda o=o: htpg.check(htpg.w8a8_run(o[1], out, o[0], o[2], mode=mode), name)
                           for o in ops])
            res[name]["stream_us"] = t
            res[name]["stream_GBps"] = nbytes / t / 1e3
            res[name]["stream_hbm_frac"] = nbytes / t / 1e3 / hbm
            del ops
        del keep

    w8a8_case("C1", 256, 1152, 4608, 0x5EED0000, 0.01, 0, False)
    # C2: CLIP fc1 through the FP16 path, bias + QuickGELU
    m, k, n = 77, 768, 3072
    if only and only != "C2":
        m = 0
    if m:
        g = torch.Generator(device=dev)
        g.manual_seed(0x5EED0001)
        x = torch.randn(m, k, device=dev, generator=g)
        wf = (torch.randn(k, n, device=dev, generator=g) * 0.02).half()
        bias = torch.randn(n, device=dev, generator=g) * 0.01
        wperm = torch.from_numpy(htpg.pack_f16_permuted(wf.cpu().numpy().view(np.uint16)).view(np.int16)).to(dev)
        wh = htpg.f16_weights(wperm, k, n)
        out = torch.empty(m, n, dtype=torch.float32, device=dev)
        tm = timed(lambda: htpg.check(htpg.f16_run(wh, out, x, bias, mode=2), "C2"))
        record("C2", m, k, n, tm, 4 * m * k + 2 * k * n + 4 * n + 4 * m * n, bf16)
        del wh, wperm
    # C3: DiT block linears at M=4096
    for name, k, n, mode, b in (("C3_qkv", 1536, 4608, 0, False), ("C3_out", 1536, 1536, 0, False),
                                ("C3_fc1", 1536, 6144, 1, True), ("C3_fc2", 6144, 1536, 0, True)):
        w8a8_case(name, 4096, k, n, 0x5EED0002 + k + n, 0.005, mode, b)
    if not only:
        res["C3_stack_us"] = sum(res[c]["us"] for c in ("C3_qkv", "C3_out", "C3_fc1", "C3_fc2"))
    if not only or only == "C3_stack":
        # the four DiT linears back to back, as a block's forward pass runs them,
        # over two blocks' operands (~0.9 GB, more than the L2): per-stack time
        layers = ((1536, 4608, 0, False), (1536, 1536, 0, False), (1536, 6144, 1, True), (6144, 1536, 0, True))
        sets = []
        for si in range(2):
            ops = []
            for j, (k, n, mode, b) in enumerate(layers):
                x, w, bb, blob = _w8a8_operands(torch, htpg, dev, 4096, k, n, 0x5EED0102 + 0x100 * si + j, 0.005, b)
                ops.append((x, w, bb, blob, torch.empty(4096, n, dtype=torch.float32, device=dev), mode))
            sets.append(ops)

        def run_stack(ops):
            for x, w, bb, _, out, mode in ops:
                htpg.check(htpg.w8a8_run(w, out, x, bb, mode=mode), "C3 stack")

        t = stream_us([lambda o=o: run_stack(o) for o in sets])
        ops_total = sum(2.0 * 4096 * n * k for k, n, _, _ in layers)
        bytes_total = sum(4 * 4096 * k + k * n + 4 * n + 4 * 4096 * n + (4 * n if b else 0) for k, n, _, b in layers)
        res["C3_stack_stream"] = {"us": t, "TOPS": ops_total / t / 1e6, "tensor_frac": ops_total / t / 1e6 / int8_peak,
                                  "hbm_frac": bytes_total / t / 1e3 / hbm,
                                  "note": "qkv, out, fc1 (bias+GELU), fc2 (bias) back to back, each with its own "
                                          "activation pass, rotating two blocks' operands (no L2 flush)"}
        del sets
    # opcode 17: SD-VAE-decoder-shaped convolutions (512 -> 512 channels, 3x3,
    # pad 1) at 64x64, and after a nearest 2x upsample (128x128 output)
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    for name, hw, up in (("C6_conv_64", 64, 1), ("C6_upconv_128", 64, 2)):
        if only and name != only:
            continue
        ic = oc = 512
        ow = oh = hw * up
        kp, np_ = 9 * ic, oc
        g = torch.Generator(device=dev)
        g.manual_seed(0x5EED0006 + up)
        x = torch.randn(1, ic, hw, hw, device=dev, generator=g)
        wkn = (torch.randn(kp, np_, device=dev, generator=g) * 0.02).half()
        bias = torch.randn(oc, device=dev, generator=g) * 0.01
        wperm = torch.from_numpy(htpg.pack_f16_permuted(wkn.cpu().numpy().view(np.uint16)).view(np.int16)).to(dev)
        wc = htpg.f16_weights(wperm, kp, np_)
        prm = dict(iw=hw, ih=hw, ic=ic, oc=oc, batch=1, ow=ow, oh=oh, kw=3, kh=3, sx=1, sy=1, px=1, py=1, dx=1,
                   dy=1, kp=kp, np=np_, upscale=up)
        pbuf = (ctypes.c_uint8 * 124).from_buffer_copy(htpg.conv_params_bytes(prm))
        out = torch.empty(1, oc, oh, ow, device=dev)
        tm = timed(lambda: htpg.check(L.htpg_conv2d_run(wc.handle, htpg.ptr(out), htpg.ptr(x), htpg.ptr(bias), pbuf,
                                                         htpg.stream_ptr()), name))
        spatial = ow * oh
        # algorithmic bytes: input read, FP16 weight, bias, FP32 output
        record(name, spatial, kp, oc, tm, 4 * ic * hw * hw + 2 * kp * np_ + 4 * oc + 4 * oc * spatial, bf16)
        res[name]["note"] = "conv as im2col GEMM: M = output pixels, K = 9*ic, N = oc; FP16 in, FP32 accumulate"
        del wc, wperm
    # opcode 19: DiT auxiliaries around the linears (HBM-bound)
    for name, mode, rows, width, chans in (("C7_adaln_modulate", 9, 8192, 1536, 1), ("C7_swiglu", 12, 4096, 6144, 12288)):
        if only and name != only:
            continue
        g = torch.Generator(device=dev)
        g.manual_seed(0x5EED0007 + mode)
        if mode == 9:
            x = torch.randn(rows, width, device=dev, generator=g)
            w = torch.randn(2, width, device=dev, generator=g)
            b = torch.randn(2, width, device=dev, generator=g)
            prm = dict(mode=9, count=rows * width, width=width, channels=1, spatial=rows // 2, groups=1, batch=2,
                       other_count=2 * width, activation=0)
            nbytes = 8 * rows * width + 16 * width
        else:
            x = torch.randn(rows, chans, device=dev, generator=g)
            w = b = None
            prm = dict(mode=12, count=rows * width, width=width, channels=chans, spatial=rows, groups=1, batch=1,
                       other_count=0, activation=0)
            nbytes = 4 * rows * chans + 4 * rows * width
        out = torch.empty(prm["count"], device=dev)
        pbuf = (ctypes.c_uint8 * 76).from_buffer_copy(htpg.aux_params_bytes(prm))
        tm = timed(lambda: htpg.check(L.htpg_model_aux(htpg.ptr(out), htpg.ptr(x), htpg.ptr(w), htpg.ptr(b), pbuf,
                                                        htpg.stream_ptr()), name))
        us = tm[0]
        res[name] = {"rows": rows, "width": width, "us": us, "GBps": nbytes / us / 1e3, "hbm_frac": nbytes / us / 1e3 / hbm,
                     "bound": "hbm", "host_latency_us": tm[3]}
    # opcodes 2-4: ggml-block weights (Q4_0 / Q8_0 / IQ4_NL) at the LLM decode
    # shapes of C5 and one prefill shape.  Random codes and FP16 scales
    # generated on the device (the kernels have no data-dependent paths).
    # Algorithmic bytes 4MK + K*N/256*block + 4MN; FLOPs 2MNK.
    def qk0_weight(wtype, k, n, seed):
        bb = 272 if wtype == 8 else 144
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        src = torch.randint(0, 256, (k * n // 256, bb), dtype=torch.uint8, device=dev, generator=g)
        sc = (torch.randn(k * n // 256, 8, device=dev, generator=g) * 0.002).half()
        src[:, :16] = sc.view(torch.uint8)
        return src.reshape(-1).contiguous()

    for tname, wtype in (("q4_0", 2), ("q8_0", 8), ("iq4_nl", 20)):
        bb = 272 if wtype == 8 else 144
        for shape, m, k, n in (("up_M1", 1, 4096, 14336), ("down_M16", 16, 14336, 4096),
                               ("prefill_M4096", 4096, 4096, 14336)):
            name = f"C8_{tname}_{shape}"
            if (only and name != only) or (shape == "prefill_M4096" and wtype != 2):
                continue
            g = torch.Generator(device=dev)
            g.manual_seed(0x5EED0008 + wtype)
            x = torch.randn(m, k, device=dev, generator=g)
            src = qk0_weight(wtype, k, n, 0x5EED0108 + wtype)
            out = torch.empty(m, n, device=dev)
            tm = timed(lambda: htpg.check(htpg.qk0_linear(out, x, src, wtype, m, k, n), name))
            nbytes = 4 * m * k + k * n // 256 * bb + 4 * m * n
            record(name, m, k, n, tm, nbytes, bf16)
            if m <= 32:
                sets = [(x, src)] + [(x, qk0_weight(wtype, k, n, 0x5EED0208 + wtype + i)) for i in range(1, 6)]
                t = stream_us([lambda o=o: htpg.check(htpg.qk0_linear(out, o[0], o[1], wtype, m, k, n), name)
                               for o in sets])
                res[name].update(stream_us=t, stream_GBps=nbytes / t / 1e3, stream_hbm_frac=nbytes / t / 1e3 / hbm)
                for o in sets[1:]:
                    L.htpg_weight_cache_drop(htpg.ptr(o[1]))
                del sets
            # the one-call entry point caches the prepared weight by address
            L.htpg_weight_cache_drop(htpg.ptr(src))
            del src
    # C5 read ceiling: a read-only stream (the decode kernels' 32-byte loads,
    # data discarded) over one linear's weight bytes (4096 x 14336 = 58.7 MB)
    # from a cold L2, the same back to back over six buffers (352 MB, more
    # than the L2), and one launch over all 352 MB
    if not only or only == "C5_read":
        nb = 4096 * 14336
        big = torch.ones(6 * nb, dtype=torch.uint8, device=dev)
        parts = [big[i * nb:(i + 1) * nb] for i in range(6)]

        def rd(b, nbytes=nb):
            htpg.check(L.htpg_stream_read(htpg.ptr(b), nbytes, htpg.stream_ptr()), "htpg_stream_read")

        tm = timed(lambda: rd(parts[0]))
        t = stream_us([lambda b=b: rd(b) for b in parts])
        tb = timed(lambda: rd(big, 6 * nb))[0]
        res["C5_read_ceiling"] = {"bytes": nb, "us": tm[0], "GBps": nb / tm[0] / 1e3, "hbm_frac": nb / tm[0] / 1e3 / hbm,
                                  "stream_us": t, "stream_GBps": nb / t / 1e3, "stream_hbm_frac": nb / t / 1e3 / hbm,
                                  "one_launch_352MB_us": tb, "one_launch_352MB_GBps": 6 * nb / tb / 1e3,
                                  "one_launch_352MB_hbm_frac": 6 * nb / tb / 1e3 / hbm}
        del big, parts
    # C5: decode shapes, no epilogue
    for m in (1, 4, 16):
        for name, k, n in (("up", 4096, 14336), ("down", 14336, 4096)):
            w8a8_case(f"C5_{name}_M{m}", m, k, n, 0x5EED0004 + m + k, 0.0, 0, False, sets=6)
    return res


def suite_summary(res):
    """Short form of the suite: per config the device time and the fraction of
    its roofline (tensor or HBM, whichever bounds it), decode shapes also back to
    back; ordered so the C1, C2 and C3 entries come last."""
    out = {}

    def r(v, nd=3):
        return None if v is None else round(float(v), nd)

    order = sorted(res, key=lambda name: (0 if not name.startswith(("C1", "C2", "C3")) else 1, name))
    for name in order:
        v = res[name]
        if not isinstance(v, dict):
            out[name] = r(v, 1)
            continue
        e = {"us": r(v.get("us"), 1)}
        if "roofline_frac" in v:
            e["frac"] = r(v["roofline_frac"])
            e["bound"] = v.get("bound")
        elif "tensor_frac" in v:
            e["tensor_frac"] = r(v["tensor_frac"])
        if "hbm_frac" in v and "roofline_frac" not in v:
            e["hbm_frac"] = r(v["hbm_frac"])
        if "stream_us" in v:
            e["stream_us"] = r(v["stream_us"], 1)
            e["stream_hbm_frac"] = r(v["stream_hbm_frac"])
        if "one_launch_352MB_hbm_frac" in v:
            e["hbm_frac"] = r(v["hbm_frac"])
            e["one_launch_352MB_hbm_frac"] = r(v["one_launch_352MB_hbm_frac"])
        if "TOPS" in v:
            e["TOPS"] = r(v["TOPS"], 1)
        out[name] = e
    return out


# ------------------------------------------------------------------ CPU leg
_CPU_CASES = {}


def cpu_sample(k, n, rows, reps=1):
    """Time the OpenMP CPU oracle on `rows` rows of a C4-shaped problem.
    Returns (TOPS, threads, seconds)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle as O
    import numpy as np
    kind = "native"
    try:
        O.lib("native")
    except Exception:
        kind = "omp"
    # every host thread, whatever OMP_NUM_THREADS the launcher exported
    O.lib(kind).orc_set_threads(len(os.sched_getaffinity(0)))
    key = (rows, k, n)
    if key not in _CPU_CASES:
        _CPU_CASES[key] = O.make_w8a8(3, "C4-sample", rows, k, n, 0.005, True, 1)
    c = _CPU_CASES[key]
    O.w8a8_linear(c.x[:8], c.blob, k, n, bias=c.bias, mode=1, kind=kind)  # warm
    t0 = time.perf_counter()
    for _ in range(reps):
        O.w8a8_linear(c.x, c.blob, k, n, bias=c.bias, mode=1, kind=kind)
    dt = (time.perf_counter() - t0) / reps
    return 2.0 * rows * n * k / dt / 1e12, O.lib(kind).orc_threads(), dt


def check_rows(torch, x_dev, out_dev, blob_host, bias_host, k, n, rows=24):
    """The last timed step's output on sampled rows against the CPU oracle on
    the same input bytes (bias + GELU: max-abs-rel bar 2e-3)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import numpy as np
    import oracle as O
    m = x_dev.shape[0]
    sel = np.unique(np.linspace(0, m - 1, rows).astype(np.int64))
    idx = torch.from_numpy(sel).to(x_dev.device)
    xr = x_dev.index_select(0, idx).cpu().numpy()
    got = out_dev.index_select(0, idx).cpu().numpy()
    ref = O.w8a8_linear(xr, blob_host, k, n, bias=bias_host, mode=1)
    err = O.max_abs_rel(got, ref)
    return {"rows": int(len(sel)), "max_abs_rel": err, "bar": 2e-3, "ok": bool(err <= 2e-3)}


def run_reference_arm(args, rank):
    if rank != 0:
        return
    rows = args.cpu_rows
    vals = []
    threads = 1
    for i in range(args.warmup + args.steps):
        tops, threads, _ = cpu_sample(K_C4, N_C4, rows)
        if i >= args.warmup:
            vals.append(tops)
    v = statistics.median(vals)
    line = {
        "impl": "reference",
        "metric": "W8A8 linear INT8 TOPS (C4 fc1 M=16384 K=1536 N=6144 bias+GELU)",
        "value": v, "unit": "TOPS", "higher_is_better": True, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "dtype": "u8xs8->s32, f32 io",
        "data": "synthetic (seeded; C4 value distributions)",
        "config": {"workload": "C4", "M": M_C4, "K": K_C4, "N": N_C4, "epilogue": "bias+gelu_tanh"},
        "cpu_baseline": {"value": v, "unit": "TOPS", "cores": threads, "kind": "port",
                         "sample": f"{rows} of {M_C4} rows per step, all {N_C4} columns"},
        "e2e": {"value": v, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ e2e
def e2e_channel(torch, L, htpg, m, k, n, x_dev, blob_host, bias_dev, steps, warmup):
    """Opcode-15 (56-byte epilogue payload) through the message channel with
    host buffers.  Returns (seconds per step, h2d bytes, d2h bytes)."""
    import numpy as np
    msg_bytes = 4096
    fds, ptrs = {}, {}

    def alloc(name, nbytes):
        fd, p = ctypes.c_int(), ctypes.c_void_p()
        htpg.check(L.htpg_buffer_alloc(nbytes, htpg.BUF_HOST, ctypes.byref(fd), ctypes.byref(p)), name)
        fds[name], ptrs[name] = fd.value, p.value

    alloc("chan", msg_bytes)
    alloc("x", m * k * 4)
    alloc("out", m * n * 4)
    alloc("blob", blob_host.nbytes)
    alloc("bias", n * 4)
    # host copies are held in variables: a temporary's memory may be returned
    # to the OS before memmove reads it
    x_host = np.ascontiguousarray(x_dev.cpu().numpy())
    bias_host = np.ascontiguousarray(bias_dev.cpu().numpy())
    ctypes.memmove(ptrs["x"], x_host.ctypes.data, m * k * 4)
    ctypes.memmove(ptrs["blob"], blob_host.ctypes.data, blob_host.nbytes)
    ctypes.memmove(ptrs["bias"], bias_host.ctypes.data, n * 4)

    sess = ctypes.c_void_p()
    htpg.check(L.htp_ops_session_open(ctypes.byref(sess), 3, None, 0), "session_open")
    htpg.check(L.htp_ops_session_init_backend(sess), "init_backend")
    htpg.check(L.htp_ops_session_create_channel(sess, fds["chan"], msg_bytes), "create_channel")
    chan = ptrs["chan"]
    # MessageHeader(16) + 2 offsets, RequestHeader(8) + OpComputeRequest(4) + payload(56)
    hdr = 16 + 8
    payload = np.zeros(14, np.int32)
    payload[0:2] = (fds["out"], 0)
    payload[2:4] = (fds["x"], 0)
    payload[4:6] = (fds["blob"], 0)
    payload[6:10] = (m, k, n, 0)
    payload[10:12] = (fds["bias"], 0)
    payload[12:14] = (n, 1)          # channels, mode 1 = bias + GELU
    req = np.concatenate([np.array([0, 2], np.int32), np.array([15], np.int32), payload])
    state = (ctypes.c_uint8 * 8).from_address(chan)

    def post():
        ctypes.memset(chan, 0, 8)
        head = np.array([0, 0, 0, 1, hdr, hdr + req.nbytes], np.int32)  # state(8) checksum n_reqs offs
        ctypes.memmove(chan + 8, head[2:].ctypes.data, 16)
        ctypes.memmove(chan + hdr, req.ctypes.data, req.nbytes)
        state[0] = 1
        while state[1] != 1:
            pass
        rc = ctypes.c_int32.from_address(chan + hdr).value
        htpg.check(rc, "opcode 15 via channel")

    for _ in range(warmup):
        post()
    t0 = time.perf_counter()
    for _ in range(steps):
        post()
    dt = (time.perf_counter() - t0) / steps
    L.htp_ops_session_destroy_channel(sess)
    L.htp_ops_session_close(sess)
    for name in fds:
        L.htpg_buffer_release(fds[name])
    return dt, m * k * 4 + n * 4, m * n * 4


def peer_copy(gib: int = 1, reps: int = 10):
    """Copy-engine bandwidth over NVLink between GPUs 0 and 1: 1 GiB from
    GPU 0 to GPU 1 (one direction), and both directions at once (one stream
    per direction); best of `reps`, CUDA events.  One JSON line."""
    import torch
    assert torch.cuda.device_count() >= 2, "needs two visible GPUs"
    nbytes = gib << 30
    a0 = torch.empty(nbytes, dtype=torch.uint8, device="cuda:0")
    b1 = torch.empty(nbytes, dtype=torch.uint8, device="cuda:1")
    a1 = torch.empty(nbytes, dtype=torch.uint8, device="cuda:1")
    b0 = torch.empty(nbytes, dtype=torch.uint8, device="cuda:0")
    s0 = torch.cuda.Stream(device="cuda:0")
    s1 = torch.cuda.Stream(device="cuda:1")

    def one_way():
        e = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        with torch.cuda.stream(s0):
            e[0].record(s0)
            b1.copy_(a0, non_blocking=True)
            e[1].record(s0)
        torch.cuda.synchronize("cuda:0")
        torch.cuda.synchronize("cuda:1")
        return nbytes / (e[0].elapsed_time(e[1]) * 1e-3) / 1e9

    def both_ways():
        e0 = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        e1 = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        with torch.cuda.stream(s0):
            e0[0].record(s0)
            b1.copy_(a0, non_blocking=True)
            e0[1].record(s0)
        with torch.cuda.stream(s1):
            e1[0].record(s1)
            b0.copy_(a1, non_blocking=True)
            e1[1].record(s1)
        torch.cuda.synchronize("cuda:0")
        torch.cuda.synchronize("cuda:1")
        return min(nbytes / (e0[0].elapsed_time(e0[1]) * 1e-3) / 1e9, nbytes / (e1[0].elapsed_time(e1[1]) * 1e-3) / 1e9)

    for _ in range(2):
        one_way()
        both_ways()
    uni = max(one_way() for _ in range(reps))
    bi = max(both_ways() for _ in range(reps))
    print(json.dumps({"peer_copy": {"bytes": nbytes, "one_direction_GBps": uni,
                                    "each_direction_when_both_GBps": bi,
                                    "how": "torch copy_ between cuda:0 and cuda:1 (copy engine, NVLink), "
                                           f"best of {reps}, CUDA events"}}), flush=True)


# ------------------------------------------------------------------ main arm
def main():
    faulthandler.enable()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-rows", type=int, default=M_C4,
                    help="rows of the C4 problem the CPU baseline computes per sample")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-suite", action="store_true",
                    help="skip the per-config C1/C2/C3/C5 device times (one GPU only)")
    ap.add_argument("--exchange", default="fused", choices=["fused", "nccl"],
                    help="N>1: how the column blocks reach every rank")
    ap.add_argument("--suite-only", default=None,
                    help="run only this suite config (e.g. C5_up_M16) and print its timings; for profiling")
    ap.add_argument("--pair-direct", type=int, default=1, choices=[0, 1],
                    help="W8A8 CTA-pair problems: 1 swapped orientation with register stores (default), "
                         "0 normal orientation with staged TMA stores")
    ap.add_argument("--decode-kernel", default="reg", choices=["reg", "tc"],
                    help="kernel for W8A8 m <= 16: register-fed decode (default) or swapped tcgen05")
    ap.add_argument("--m", type=int, default=M_C4,
                    help="token rows; smaller values only for profiling captures (workload C4-M<m>)")
    ap.add_argument("--settle", type=float, default=1.5,
                    help="seconds of untimed load before timing (clock sampling); 0 under ncu")
    ap.add_argument("--peer-copy", action="store_true",
                    help="measure the NVLink peer-copy bandwidth between GPUs 0 and 1 (one process) and exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.peer_copy:
        peer_copy()
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank)
        return

    import torch
    import htpg
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    L = htpg.lib()
    htpg.check(L.htpg_init(local), "htpg_init")
    htpg.set_decode_kernel(0 if args.decode_kernel == "reg" else 1)
    htpg.set_pair_direct(bool(args.pair_direct))
    if args.suite_only:
        res = suite(torch, L, htpg, dev, L2Flush(torch, dev), only=args.suite_only)
        htpg.check(htpg.check_device(), "watchdog")
        print(json.dumps({"suite": res}), flush=True)
        return
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))

    m, k, n = args.m, K_C4, N_C4
    workload = "C4" if m == M_C4 else f"C4-M{m}"
    assert n % (64 * world) == 0
    n0, n_loc = htpg.column_range(n, world, rank)
    x, blob_dev, bias, blob_host, bias_host = seeded_c4_inputs(torch, dev, m, k, n)
    w = htpg.w8a8_weights(blob_dev, k, n, n0=n0, n_cols=n_loc)
    bias_loc = bias[n0:n0 + n_loc].contiguous()
    out_loc = torch.empty(m, n_loc, dtype=torch.float32, device=dev)
    fused = world > 1 and args.exchange == "fused"
    gathered = torch.empty(world * m, n_loc, dtype=torch.float32, device=dev) if world > 1 and not fused else None
    full = torch.empty(m, n, dtype=torch.float32, device=dev) if world > 1 else None
    flush = L2Flush(torch, dev)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    peers = []
    if fused:
        # every rank's [M][N] output, mapped into this process; this rank's
        # GEMM stores its column block into all of them
        handles = [None] * world
        dist.all_gather_object(handles, htpg.ipc_export(full))
        peers = [htpg.ipc_import(handles[p]) for p in range(world) if p != rank]
        outs = (ctypes.c_void_p * world)(full.data_ptr() + 4 * n0, *[q + 4 * n0 for q in peers])
        token = torch.zeros(1, dtype=torch.float32, device=dev)

    def step():
        if fused:
            htpg.check(L.htpg_w8a8_run_gather(w.handle, outs, world, n, htpg.ptr(x), htpg.ptr(bias_loc), m, n_loc,
                                              1, sp), "htpg_w8a8_run_gather")
            # stream-ordered: completes once every rank's stores have landed
            dist.all_reduce(token)
            return
        htpg.check(L.htpg_w8a8_run(w.handle, htpg.ptr(out_loc), 0, htpg.ptr(x), htpg.ptr(bias_loc), m, n_loc,
                                   1, sp), "htpg_w8a8_run")
        if world > 1:
            dist.all_gather_into_tensor(gathered, out_loc)
            htpg.assemble_columns(full, gathered.view(world, m, n_loc))

    for _ in range(args.warmup):
        flush()
        step()
    torch.cuda.synchronize()
    htpg.check(htpg.check_device(), "watchdog")

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    L.htpg_phase_timing(1)
    htpg.phase_timing_read()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    # settle steps: keep the GPU under this load for ~1.5 s before timing so the
    # 200 ms clock samples describe the timed steps; every rank runs the same count
    t0 = time.perf_counter()
    for _ in range(5):
        flush()
        step()
    torch.cuda.synchronize()
    per = max((time.perf_counter() - t0) / 5, 1e-5)
    cnt = torch.tensor([min(int(args.settle / per), 20000)], dtype=torch.int64, device=dev)
    if dist:
        dist.all_reduce(cnt, op=dist.ReduceOp.MAX)
    settle = int(cnt.item())
    with ClockSampler(local) as clocks:
        for i in range(settle):
            flush()
            step()
            if i % 64 == 63:
                htpg.phase_timing_read()   # keeps the pending event list short
        torch.cuda.synchronize()
        htpg.phase_timing_read()
        launches0 = L.htpg_launch_count()
        torch.cuda._sleep(SLEEP_CYCLES)       # the host queues the timed steps meanwhile
        for i in range(args.steps):
            flush()                            # L2 flush outside the timed events
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        torch.cuda.synchronize()
    launches = L.htpg_launch_count() - launches0
    if dist:
        dist.barrier()
    L.htpg_phase_timing(0)
    shard_ms = None
    if world > 1:
        # the GEMM phase alone: each rank computes its column shard (what a
        # row-parallel next layer consumes), no exchange; same timing rules
        def shard_step():
            htpg.check(L.htpg_w8a8_run(w.handle, htpg.ptr(out_loc), 0, htpg.ptr(x), htpg.ptr(bias_loc), m, n_loc,
                                       1, sp), "htpg_w8a8_run")
        for _ in range(3):
            flush()
            shard_step()
        dist.barrier()
        torch.cuda.synchronize()
        s_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in range(args.steps)]
        torch.cuda._sleep(SLEEP_CYCLES)
        for a, b in s_ev:
            flush()
            a.record(stream)
            shard_step()
            b.record(stream)
        torch.cuda.synchronize()
        ts = torch.tensor([sum(a.elapsed_time(b) for a, b in s_ev)], dtype=torch.float64, device=dev)
        dist.all_reduce(ts, op=dist.ReduceOp.MAX)
        shard_ms = float(ts.item()) / args.steps
    act_ms, gemm_ms, runs = htpg.phase_timing_read()
    total_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    htpg.check(htpg.check_device(), "watchdog")

    ms_per_step = total_ms / args.steps
    ops = 2.0 * m * n * k
    value = ops / (ms_per_step * 1e-3) / 1e12

    hbm, bf16, bf16_sus, peak_kind = peaks()
    int8_peak = 2.0 * bf16  # no measured INT8 GEMM: 2x the measured dense BF16 (B200: INT8 = 2x BF16 rate)
    gemm_avg_ms = gemm_ms / max(runs, 1)
    act_avg_ms = act_ms / max(runs, 1)
    gemm_bytes = m * k + k * n_loc + 4 * n_loc * 2 + 4 * m + 4 * m * n_loc
    gemm_ops = 2.0 * m * n_loc * k
    t_hbm = gemm_bytes / (hbm * 1e9)
    t_tc = gemm_ops / (int8_peak * 1e12)
    # with the fused exchange the GEMM phase also stores every tile into the
    # world-1 peers: each rank sends (and receives) (world-1)/world of the FP32
    # output over NVLink, against the measured 770 GB/s per direction
    link_bytes = (world - 1) * 4 * m * n_loc if (world > 1 and fused) else 0
    t_link = link_bytes / (NVLINK_GBS * 1e9)
    if t_link > max(t_tc, t_hbm):
        roof = {"bound": "nvlink", "achieved": link_bytes / (gemm_avg_ms * 1e-3) / 1e9, "peak": NVLINK_GBS,
                "unit": "GB/s"}
    elif t_tc >= t_hbm:
        roof = {"bound": "tensor", "achieved": gemm_ops / (gemm_avg_ms * 1e-3) / 1e12, "peak": int8_peak,
                "unit": "TFLOP/s"}
    else:
        roof = {"bound": "hbm", "achieved": gemm_bytes / (gemm_avg_ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    if link_bytes:
        roof["nvlink_bytes_per_rank"] = link_bytes
        roof["nvlink_frac"] = link_bytes / (gemm_avg_ms * 1e-3) / 1e9 / NVLINK_GBS
    roof["traffic"] = None
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            tr = json.load(f).get(f"C4_w{world}")
            roof["traffic"] = tr
    except Exception:
        pass
    plan = htpg.plan_info(0, m, n_loc, k) if not (world > 1 and fused) else None
    if plan is None:
        roof["kernel"] = "gemm2_kernel<I8,256,false> (CTA-pair tcgen05 kind::i8, TMA stores to every rank)"
    elif plan["swap"] == 3:
        roof["kernel"] = (f"gemm2_kernel<I8,{plan['bn']},true> (CTA-pair tcgen05 kind::i8, swapped orientation, "
                          "fused dequant/bias/GELU, stores from registers)")
    elif plan["swap"] == 0 and plan["tiles_a"] == (m + 255) // 256:
        roof["kernel"] = (f"gemm2_kernel<I8,{plan['bn']},false> (CTA-pair tcgen05 kind::i8 + fused "
                          "dequant/bias/GELU, TMA stores)")
    else:
        roof["kernel"] = f"gemm_kernel<I8,{plan['bn']},false> (tcgen05 kind::i8 + fused dequant/bias/GELU)"
    roof["peak_source"] = f"hbm {peak_kind} burst copy; tensor = 2 x {peak_kind} dense BF16 burst"
    roof["hbm_frac"] = gemm_bytes / (gemm_avg_ms * 1e-3) / 1e9 / hbm
    roof["tensor_frac"] = gemm_ops / (gemm_avg_ms * 1e-3) / 1e12 / int8_peak
    roof["gemm_us"] = gemm_avg_ms * 1e3
    roof["quant_us"] = act_avg_ms * 1e3
    roof["algorithmic_bytes"] = gemm_bytes

    line = {
        "metric": "W8A8 linear INT8 TOPS (C4 fc1 M=16384 K=1536 N=6144 bias+GELU)",
        "value": value, "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "u8xs8->s32 (int8 tensor cores), f32 io",
        "data": ("synthetic: C4 value distributions from the benchmark's splitmix64 seeds (config 3); "
                 "the CPU baseline computes on the same bytes"),
        "config": {"workload": workload, "M": m, "K": k, "N": n, "N_per_gpu": n_loc,
                   "epilogue": "bias+gelu_tanh", "parallelism": f"tp{world} (columns)" if world > 1 else "single",
                   "exchange": (None if world == 1 else
                                "fused: the GEMM epilogue TMA-stores each tile into every rank's [M][N] output "
                                "over NVLink (CUDA IPC); NCCL all-reduce of a token orders the step" if fused else
                                "nccl all_gather + reassembly"),
                   "l2": L2_NOTE},
        "roofline": roof,
        "gpu_launches": int(launches),
        "clocks": clocks.summary(),
    }
    if shard_ms is not None:
        line["shard_only"] = {"value": ops / (shard_ms * 1e-3) / 1e12, "unit": "TOPS", "ms_per_step": shard_ms,
                              "note": "the same steps without the output exchange: every rank computes its "
                                      "[M][N/world] column shard (the input of a row-parallel next layer); "
                                      "max over ranks; not the headline value"}

    if rank == 0 and world == 1 and not args.no_e2e:
        dt, h2d, d2h = e2e_channel(torch, L, htpg, m, k, n, x, blob_host, bias, max(3, args.steps // 4), 2)
        line["e2e"] = {"value": ops / dt / 1e12, "unit": "TOPS", "h2d_bytes_per_step": h2d,
                       "d2h_bytes_per_step": d2h, "path": "message channel, opcode 15 (56-byte payload), "
                       "pinned host buffers"}
    elif world > 1 and not args.no_e2e:
        # C-ABI run of this rank's column shard with host buffers: the pinned
        # activation goes in every step on every rank, rank 0 reads the whole
        # gathered output back; device time per step, max over ranks.
        x_host = x.cpu().pin_memory()
        out_host = torch.empty(m, n, dtype=torch.float32).pin_memory() if rank == 0 else None
        e2e_steps = max(3, args.steps // 4)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(e2e_steps)]

        def e2e_step():
            x.copy_(x_host, non_blocking=True)
            step()
            if rank == 0:
                out_host.copy_(full, non_blocking=True)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        dist.barrier()
        for a, b in ev:
            a.record(stream)
            e2e_step()
            b.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([sum(a.elapsed_time(b) for a, b in ev) / e2e_steps], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        line["e2e"] = {"value": ops / (float(t.item()) * 1e-3) / 1e12, "unit": "TOPS",
                       "h2d_bytes_per_step": m * k * 4, "d2h_bytes_per_step": m * n * 4,
                       "path": ("C ABI htpg_w8a8_run_gather per rank (fused output exchange over NVLink)"
                                if fused else "C ABI htpg_w8a8_run per rank + NCCL all-gather") +
                               "; pinned host activation in (every rank), full output out (rank 0)"}
    if world == 1 and not args.no_suite:
        line["suite"] = suite(torch, L, htpg, dev, flush)
    if rank == 0 and world == 1 and not args.no_cpu:
        tops, threads, secs = cpu_sample(k, n, args.cpu_rows)
        line["cpu_baseline"] = {"value": tops, "unit": "TOPS", "cores": threads, "kind": "port",
                                "sample": f"{args.cpu_rows} of {m} rows, all {n} columns ({secs:.2f} s)"}
        line["cpu_baseline"]["check"] = check_rows(torch, x, out_loc, blob_host, bias_host, k, n)
    if world > 1:
        # the assembled output against one GPU computing all N columns
        torch.cuda.synchronize()
        if rank == 0:
            w_all = htpg.w8a8_weights(blob_dev, k, n)
            ref = torch.empty(m, n, dtype=torch.float32, device=dev)
            htpg.check(L.htpg_w8a8_run(w_all.handle, htpg.ptr(ref), 0, htpg.ptr(x), htpg.ptr(bias), m, n, 1, sp),
                       "reference run")
            torch.cuda.synchronize()
            line["config"]["check"] = {"vs_single_gpu_max_abs_diff": float((ref - full).abs().max().item()),
                                       "bit_exact": bool(torch.equal(ref.view(torch.int32), full.view(torch.int32)))}
            del w_all, ref
        dist.barrier()
        for q in peers:
            htpg.check(L.htpg_ipc_close(q), "htpg_ipc_close")
    if "suite" in line:
        # the per-config figures in short form, last on the line so that a
        # reader keeping only the line's tail still sees them (C1-C3 last)
        full = line.pop("suite")
        line["suite"] = full
        line["suite_summary"] = suite_summary(full)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
