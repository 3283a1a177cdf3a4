"""Column-sharded linear across ranks (gloo, CPU): the N-split layout used for
multi-GPU runs.  Each rank computes its column shard (here with the CPU oracle,
from a constants blob holding only its columns), the shards are all-gathered
and reassembled into the row-major output, which must equal the unsharded
result exactly: row quantisation depends only on the row, never on N.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, m, k, n, mode, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for sub in ("../htp-ops-lib-sd.cpp_b200", "../oracle"):
        sys.path.insert(0, os.path.join(here, sub))
    import htpg
    import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = O.make_w8a8(3, "shard", m, k, n, 0.005, True, mode)
        n0, nl = htpg.column_range(n, world, rank)
        blob = O.w8a8_pack(c.w[n0:n0 + nl], c.sw[n0:n0 + nl], None)
        shard = O.w8a8_linear(c.x, blob, k, nl, bias=c.bias[n0:n0 + nl], mode=mode)
        gathered = torch.empty(world * m, nl)
        dist.all_gather_into_tensor(gathered, torch.from_numpy(shard))
        full = torch.empty(m, n)
        htpg.assemble_columns(full, gathered.view(world, m, nl))
        if rank == 0:
            ref = O.w8a8_linear(c.x, c.blob, k, n, bias=c.bias, mode=mode)
            q.put(bool(np.array_equal(full.numpy().view(np.uint32), ref.view(np.uint32))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,mode", [(2, 1), (4, 0)])
def test_column_shards_reassemble_exactly(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, 40, 256, 512, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert q.get(timeout=5) is True


def test_column_range_rules():
    import htpg
    assert htpg.column_range(6144, 8, 3) == (2304, 768)
    with pytest.raises(ValueError):
        htpg.column_range(6144, 5, 0)
    with pytest.raises(ValueError):
        htpg.column_range(192, 2, 0)   # 96 columns is not whole 64-column groups
