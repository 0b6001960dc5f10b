"""Failure detection without a GPU fault: a tensor-parallel chain whose peer never runs.

Rank 0 of a world-2 chain is launched alone on one GPU.  Its exchange buffer and the
"peer's" buffer are both ordinary local allocations, and nothing ever writes rank 1's
partial sums: every wait for them is a wait on a flag nothing sets.  The kernel must give
up after its bounded wait (about 5 s), record the error in the device error word and
return; ql_check_device then reports QL_EDEVICE, and the context stays usable (a normal
launch afterwards gives correct results).  Only one kernel runs: no two launches ever
wait on each other."""
import ctypes as C
import time

import numpy as np
import pytest

import blog_b200 as Q
import oracle as O
from gpu_util import dev, host, make_weights, rel_l2

pytestmark = pytest.mark.gpu
H, QW, KV, V = 2048, 2048, 256, 1000


def test_tp_chain_peer_that_never_arrives_reports_edevice():
    import torch
    torch.cuda.init()
    Q.init(0)
    Q.set_stream(torch.cuda.current_stream().cuda_stream)
    rb = lambda k: O.row_bytes(O.Q4_K, k)
    wq, wk, wv = (dev(make_weights(O.Q4_K, r, H, seed=500 + i)) for i, r in enumerate((QW, KV, KV)))
    wo = dev(make_weights(O.Q4_K, H, QW, seed=504))
    lm = dev(make_weights(O.Q4_K, V, H, seed=505))
    g = dev(np.ones(H, np.float32))
    h = dev(np.random.default_rng(1).standard_normal(H).astype(np.float32))
    qkv = torch.zeros(QW + 2 * KV, device="cuda:0")
    logits = torch.zeros(V, device="cuda:0")
    tok = torch.full((1,), -1, dtype=torch.int32, device="cuda:0")
    ops = [Q.chain_op(Q.OP_STORE, [wq.data_ptr(), wk.data_ptr(), wv.data_ptr()], [rb(H)] * 3, [QW, KV, KV], H,
                      h.data_ptr(), qkv.data_ptr(), g.data_ptr(), 1e-6),
           Q.chain_op(Q.OP_ADD, [wo.data_ptr()], [rb(QW)], [H], QW, qkv.data_ptr(), h.data_ptr(), reduce=True),
           Q.chain_op(Q.OP_STORE, [lm.data_ptr()], [rb(H)], [V], H, h.data_ptr(), logits.data_ptr(), g.data_ptr(),
                      1e-6, argmax_idx=tok.data_ptr())]
    arr = (Q.ChainOp * len(ops))(*ops)
    L = Q.lib()
    nbytes = L.ql_gemv_chain_exchange_bytes(C.cast(arr, C.c_void_p), len(ops), 2)
    assert nbytes > 0
    bufs = [torch.zeros(nbytes // 8 + 32, dtype=torch.int64, device="cuda:0") for _ in range(2)]
    ptrs = (C.c_void_p * 2)(bufs[0].data_ptr(), bufs[1].data_ptr())
    handle = C.c_void_p()
    assert L.ql_gemv_chain_create_tp(C.cast(arr, C.c_void_p), len(ops), 0, 2, C.cast(ptrs, C.c_void_p),
                                     C.byref(handle)) == Q.QL_OK, L.ql_last_error()
    try:
        t0 = time.time()
        assert L.ql_gemv_chain_run(handle) == Q.QL_OK, L.ql_last_error()
        st = L.ql_check_device()
        waited = time.time() - t0
        assert st == Q.QL_EDEVICE, (st, L.ql_last_error())
        assert b"bounded wait" in L.ql_last_error()
        assert 1.0 < waited < 60.0, waited
    finally:
        assert L.ql_gemv_chain_destroy(handle) == Q.QL_OK
    # the context is still usable: an ordinary launch gives the right answer
    x = np.random.default_rng(2).standard_normal((1, H)).astype(np.float32)
    y = torch.zeros(QW, device="cuda:0")
    w = make_weights(O.Q4_K, QW, H, seed=500)
    Q.quant_gemv(O.Q4_K, wq.data_ptr(), rb(H), dev(x).data_ptr(), y.data_ptr(), QW, H, 1)
    assert rel_l2(host(y), O.gemv(O.Q4_K, w, rb(H), x, QW, H, 1, order=1)[0]) < 1e-5
    Q.check_device()
