"""Multi-GPU tests of the peer-memory all-reduce (two ranks, one process per GPU).

Skipped unless the machine has at least two GPUs.  Ranks exchange IPC handles
over a gloo process group on 127.0.0.1; the all-reduce itself runs on NVLink.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime
    import torch
    import torch.distributed as dist
    import blog_b200 as Q
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        Q.init(rank)
        s = torch.cuda.Stream()
        Q.set_stream(s.cuda_stream)

        def exchange(h):
            out = [None] * world
            dist.all_gather_object(out, h)
            return out
        comm = Q.Comm(rank, world, 4096, 4, exchange)
        res = []
        with torch.cuda.stream(s):
            for step in range(3):
                for slot, n in enumerate((3584, 1, 4096, 777)):
                    base = torch.arange(n, dtype=torch.float32, device="cuda") * 0.25
                    buf = base * (rank + 1) + step + slot
                    Q.set_stream(s.cuda_stream)
                    comm.allreduce(buf.data_ptr(), n, slot)
                    torch.cuda.synchronize()
                    # rank order sum: sum_r (base*(r+1) + step + slot)
                    want = sum(base * (r + 1) + step + slot for r in range(world))
                    res.append(bool(torch.equal(buf, want)))
                comm.step()
        torch.cuda.synchronize()
        Q.check_device()
        dist.barrier()
        comm.close()
        dist.destroy_process_group()
        q.put((rank, all(res), len(res)))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, False, repr(e)))


def test_peer_allreduce_two_ranks():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, info in out:
        assert ok, (rank, info)
