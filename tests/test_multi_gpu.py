"""Column-sharded W8A8 linear with the fused output exchange on 2 GPUs.

Each rank prepares its column block of the weight, maps every rank's [M][N]
output through CUDA IPC and runs htpg_w8a8_run_gather: its epilogue stores
each tile into all of them.  The single-destination CTA-pair shapes of this
test run the swapped orientation in the single-GPU reference run and the
normal orientation (TMA stores) in the exchange, so the comparison also
checks the two orientations against each other.  After a stream-ordered all-reduce of a token the
assembled output must equal, bit for bit, one GPU computing all N columns.
Skipped when fewer than two GPUs are visible.
"""
import ctypes
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import sys
    import datetime
    here = os.path.dirname(os.path.abspath(__file__))
    for sub in ("../htp-ops-lib-sd.cpp_b200", "../oracle", ".."):
        sys.path.insert(0, os.path.join(here, sub))
    import torch.distributed as dist
    import htpg
    import bench
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    L = htpg.lib()
    htpg.check(L.htpg_init(rank), "htpg_init")
    results = {}
    peers = []
    try:
        cases = [(1000, 512, 1280, 1), (300, 768, 1024, 0), (4100, 256, 4608, 2), (2048, 1536, 3072, 1)]
        for (m, k, n, mode) in cases:
            x, blob, bias, _ = bench.make_c4_inputs(torch, dev, m, k, n, seed=0x5EED0100 + m)
            n0, nl = htpg.column_range(n, world, rank)
            w = htpg.w8a8_weights(blob, k, n, n0=n0, n_cols=nl)
            bias_loc = bias[n0:n0 + nl].contiguous()
            full = torch.full((m, n), float("nan"), device=dev)
            handles = [None] * world
            dist.all_gather_object(handles, htpg.ipc_export(full))
            peers = [htpg.ipc_import(handles[p]) for p in range(world) if p != rank]
            outs = (ctypes.c_void_p * world)(full.data_ptr() + 4 * n0, *[p + 4 * n0 for p in peers])
            sp = torch.cuda.current_stream().cuda_stream
            for _ in range(2):   # twice: the second run overwrites the first in place
                htpg.check(L.htpg_w8a8_run_gather(w.handle, outs, world, n, htpg.ptr(x), htpg.ptr(bias_loc),
                                                  m, nl, mode, sp), "htpg_w8a8_run_gather")
                token = torch.zeros(1, device=dev)
                dist.all_reduce(token)
            torch.cuda.synchronize()
            w_all = htpg.w8a8_weights(blob, k, n)
            ref = torch.empty(m, n, device=dev)
            htpg.check(htpg.w8a8_run(w_all, ref, x, bias, mode=mode), "single-GPU run")
            torch.cuda.synchronize()
            results[(m, k, n, mode)] = bool(torch.equal(ref.view(torch.int32), full.view(torch.int32)))
            dist.barrier()
            for p in peers:
                htpg.check(L.htpg_ipc_close(p), "htpg_ipc_close")
            peers = []
        # several destinations need the TMA-store epilogue: small M is refused
        x = torch.randn(16, 256, device=dev)
        _, blob, _, _ = bench.make_c4_inputs(torch, dev, 16, 256, 256)
        w = htpg.w8a8_weights(blob, 256, 256)
        a = torch.empty(16, 256, device=dev)
        b = torch.empty(16, 256, device=dev)
        outs2 = (ctypes.c_void_p * 2)(a.data_ptr(), b.data_ptr())
        results["small_m_refused"] = L.htpg_w8a8_run_gather(w.handle, outs2, 2, 256, htpg.ptr(x), None, 16, 0, 0,
                                                            None) == htpg.ECAPACITY
        results["watchdog"] = htpg.check_device() == 0
        q.put((rank, results))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_exchange_matches_single_gpu():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for _ in range(2):
        rank, res = q.get(timeout=10)
        assert all(res.values()), (rank, res)
