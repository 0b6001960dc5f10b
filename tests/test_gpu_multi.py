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


def _tp_chain_worker(rank, world, port, q, mlp=False):
    import datetime
    import numpy as np
    import torch
    import torch.distributed as dist
    import blog_b200 as Q
    import oracle as O
    from gpu_util import make_weights
    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        Q.init(rank)
        Q.set_stream(torch.cuda.current_stream().cuda_stream)
        H, QW, KV, F, V = 2048, 2048, 256, 4096, 5000
        rb = lambda k: O.row_bytes(O.Q4_K, k)
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to("cuda")
        rng = np.random.default_rng(5)
        full = {n: make_weights(O.Q4_K, r, k, seed=400 + i) for i, (n, r, k) in enumerate(
            (("wq", QW, H), ("wk", KV, H), ("wv", KV, H), ("wo", H, QW), ("wg", F, H), ("wu", F, H), ("wd", H, F),
             ("lm", V, H)))}
        ln1, ln2, lnf = [(1 + 0.1 * rng.standard_normal(H)).astype(np.float32) for _ in range(3)]
        bq = (0.01 * rng.standard_normal(QW + 2 * KV)).astype(np.float32)
        h0 = rng.standard_normal(H).astype(np.float32)

        def rows(w, lo, hi):
            return w[lo:hi]

        def kblocks(w, b0, b1):  # row-parallel shard: whole 256-element blocks of every row
            return w[:, b0 * 144:b1 * 144]

        def split(n, parts, g):
            nb = n // g
            cuts = [(r * nb) // parts for r in range(parts + 1)]
            return cuts[rank] * g, cuts[rank + 1] * g

        def build(W, qlo, qhi, klo, khi, flo, fhi, vlo, vhi, comm_world):
            keep = []
            dv = lambda a: keep.append(d(a)) or keep[-1]
            t = {"h": dv(h0.copy()), "qkv": torch.zeros((qhi - qlo) + 2 * (khi - klo), device="cuda"),
                 "act": torch.zeros(fhi - flo, device="cuda"), "logits": torch.zeros(vhi - vlo, device="cuda"),
                 "tok": torch.full((1,), -1, dtype=torch.int32, device="cuda")}
            wq, wk, wv = dv(rows(W["wq"], qlo, qhi)), dv(rows(W["wk"], klo, khi)), dv(rows(W["wv"], klo, khi))
            wo = dv(kblocks(W["wo"], qlo // 256, qhi // 256))
            wg, wu = dv(rows(W["wg"], flo, fhi)), dv(rows(W["wu"], flo, fhi))
            wd = dv(kblocks(W["wd"], flo // 256, fhi // 256))
            wl = dv(rows(W["lm"], vlo, vhi))
            b = dv(np.concatenate([bq[qlo:qhi], bq[QW + klo:QW + khi], bq[QW + KV + klo:QW + KV + khi]]))
            g1, g2, gf = dv(ln1), dv(ln2), dv(lnf)
            hp = t["h"].data_ptr()
            red = comm_world > 1
            ops = []
            for _ in range(2):
                ops.append(Q.chain_op(Q.OP_STORE, [wq.data_ptr(), wk.data_ptr(), wv.data_ptr()], [rb(H)] * 3,
                                      [qhi - qlo, khi - klo, khi - klo], H, hp, t["qkv"].data_ptr(), g1.data_ptr(),
                                      1e-6, b.data_ptr()))
                ops.append(Q.chain_op(Q.OP_ADD, [wo.data_ptr()], [rb(qhi - qlo)], [H], qhi - qlo, t["qkv"].data_ptr(),
                                      hp, reduce=red))
                if mlp:  # gate/up + down as one op; with comm_world > 1 its partials are summed over ranks
                    ops.append(Q.chain_op(Q.OP_MLP, [wg.data_ptr(), wu.data_ptr(), wd.data_ptr()],
                                          [rb(H), rb(H), rb(fhi - flo)], [fhi - flo, fhi - flo, H], H, hp, hp,
                                          g2.data_ptr(), 1e-6))
                    continue
                ops.append(Q.chain_op(Q.OP_SWIGLU, [wg.data_ptr(), wu.data_ptr()], [rb(H)] * 2, [fhi - flo] * 2, H, hp,
                                      t["act"].data_ptr(), g2.data_ptr(), 1e-6))
                ops.append(Q.chain_op(Q.OP_ADD, [wd.data_ptr()], [rb(fhi - flo)], [H], fhi - flo, t["act"].data_ptr(),
                                      hp, reduce=red))
            ops.append(Q.chain_op(Q.OP_STORE, [wl.data_ptr()], [rb(H)], [vhi - vlo], H, hp, t["logits"].data_ptr(),
                                  gf.data_ptr(), 1e-6, argmax_idx=t["tok"].data_ptr(), argmax_offset=vlo))
            return t, ops, keep

        def exchange(hnd):
            out = [None] * world
            dist.all_gather_object(out, hnd)
            return out
        qlo, qhi = split(QW, world, 256)
        klo, khi = split(KV, world, 32)
        flo, fhi = split(F, world, 256)
        vlo, vhi = split(V, world, 8)
        t, ops, keep = build(full, qlo, qhi, klo, khi, flo, fhi, vlo, vhi, world)
        chain = Q.GemvChain(ops, rank, world, exchange)
        res = []
        for _ in range(3):  # replays
            t["h"].copy_(d(h0))
            chain.run()
            torch.cuda.synchronize()
            res.append((t["h"].cpu().numpy().copy(), int(t["tok"].cpu()[0])))
        Q.check_device()
        ok_rep = all(np.array_equal(r[0].view(np.uint32), res[0][0].view(np.uint32)) and r[1] == res[0][1] for r in res)
        hs = [None] * world
        dist.all_gather_object(hs, (res[0][0], res[0][1]))
        ok_rank = all(np.array_equal(x[0].view(np.uint32), hs[0][0].view(np.uint32)) and x[1] == hs[0][1] for x in hs)
        ok = ok_rep and ok_rank
        info = "replicas agree" if ok else (
            f"replays differ: {[float(np.abs(r[0] - res[0][0]).max()) for r in res]}" if not ok_rep else
            f"ranks differ: {[float(np.abs(x[0] - hs[0][0]).max()) for x in hs]}")
        if rank == 0 and ok:  # against the single-GPU chain with the whole matrices
            t1, ops1, keep1 = build(full, 0, QW, 0, KV, 0, F, 0, V, 1)
            c1 = Q.GemvChain(ops1)
            c1.run()
            torch.cuda.synchronize()
            h1, tok1 = t1["h"].cpu().numpy(), int(t1["tok"].cpu()[0])
            err = float(np.linalg.norm(res[0][0].astype(np.float64) - h1) / np.linalg.norm(h1))
            ok = err < 1e-5 and tok1 == res[0][1]
            info = f"rel err {err:.2e}, tokens {res[0][1]} vs {tok1}"
            c1.close()
        dist.barrier()
        chain.close()
        dist.destroy_process_group()
        q.put((rank, ok, info))
    except Exception as e:  # report to the parent instead of hanging it
        import traceback
        q.put((rank, False, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_chain_matches_single_gpu(world, mlp=False):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_chain_worker, args=(r, world, port, q, mlp)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, info in out:
        assert ok, (rank, info)


def _ep_worker(rank, world, port, q):
    import datetime
    import numpy as np
    import torch
    import torch.distributed as dist
    import blog_b200 as Q
    try:
        import bench
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        Q.init(rank)
        Q.set_stream(torch.cuda.current_stream().cuda_stream)
        # two layers: the dense layer 0 and one MoE layer, batch 8
        st = bench.MoEStack(Q, torch, rank, world, 8, layers=2)

        def moe_layer(stk):
            L = stk.layers[1]
            stk.xn.copy_(torch.randn(stk.xn.shape, generator=torch.Generator().manual_seed(3)).to("cuda"))
            Q.quant_gemv_ex(bench.QK, L["wr"].data_ptr(), Q.row_bytes(bench.QK, bench.DS_H), stk.xn.data_ptr(),
                            bench.DS_H, stk.logits.data_ptr(), bench.DS_E, bench.DS_E, bench.DS_H, stk.T)
            stk.moe.zero_()
            stk.routed(L)
            torch.cuda.synchronize()
            return stk.moe.cpu().numpy().copy(), stk.idx.cpu().numpy().copy()
        part, idx = moe_layer(st)
        parts = [None] * world
        dist.all_gather_object(parts, part)
        ep = np.sum(np.stack(parts).astype(np.float64), axis=0)
        ok, info = True, ""
        if rank == 0:
            del st
            torch.cuda.empty_cache()
            one = bench.MoEStack(Q, torch, 0, 1, 8, layers=2)
            full, idx1 = moe_layer(one)
            err = float(np.linalg.norm(ep - full) / np.linalg.norm(full))
            ok = err < 1e-5 and np.array_equal(idx, idx1)
            info = f"EP{world} vs 1 GPU: rel err {err:.2e}"
        Q.check_device()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok, info))
    except Exception:
        import traceback
        q.put((rank, False, traceback.format_exc()))


def test_expert_parallel_moe_layer_matches_single_gpu():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=400) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, info in out:
        assert ok, (rank, info)
