"""Pins the CPU oracle against the reference's own CUDA kernels.

oracle/_ref/libref_local_llm.so is AI/codes/local-llm's kernel.cu + launch.cu
compiled unchanged for sm_100a by oracle/Makefile.  On the same inputs:
  * dequant-to-f16 must agree bit for bit with the oracle;
  * the reference's warp-per-row GEMV must agree bit for bit with the oracle's
    restatement of its summation order (order=0);
  * router indices must agree exactly (weights: the reference uses the __expf
    intrinsic, the oracle expf, so they agree to a few ulp) -- and this
    library's router must agree with the reference's bit for bit;
  * embeddings and argmax must agree exactly.
"""
import numpy as np
import pytest

import blog_b200 as Q
import oracle as O
from gpu_util import dev, host, make_weights, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    import torch
    R = O.ref_lib()
    if R is None:
        pytest.fail("oracle/_ref/libref_local_llm.so is missing (built by `make -C oracle` where the reference exists)")
    torch.cuda.init()
    R.ref_set_stream(torch.cuda.current_stream().cuda_stream)
    Q.init(0)
    Q.set_stream(torch.cuda.current_stream().cuda_stream)
    return R


@pytest.mark.parametrize("t,fn", [(O.Q4_K, "ref_dequantize_q4k"), (O.Q8_0, "ref_dequantize_q80"),
                                  (O.Q5_0, "ref_dequantize_q50"), (O.Q6_K, "ref_dequantize_q6k")])
def test_reference_dequant_equals_oracle(ref, t, fn):
    import torch
    w = make_weights(t, 128, 1024, seed=5 + t)
    n = 128 * 1024
    out = torch.empty(n, dtype=torch.int16, device="cuda:0")
    getattr(ref, fn)(dev(w).data_ptr(), out.data_ptr(), n)
    assert ref.ref_last_error() == 0
    assert np.array_equal(host(out).view(np.uint16), O.dequant_f16(t, w.reshape(-1), n))


@pytest.mark.parametrize("t,n,k,m", [(O.Q4_K, 256, 4096, 1), (O.Q4_K, 64, 2048, 3), (O.Q8_0, 200, 896, 1),
                                     (O.Q5_0, 128, 1408, 2), (O.Q6_K, 64, 1024, 1)])
def test_reference_gemv_equals_oracle_lane_order(ref, t, n, k, m):
    import torch
    w = make_weights(t, n, k, seed=n + k)
    x = np.random.default_rng(n).standard_normal((m, k)).astype(np.float32)
    y = torch.empty((m, n), device="cuda:0")
    rb = O.row_bytes(t, k)
    ref.ref_quant_gemv(t, dev(w).data_ptr(), rb, dev(x).data_ptr(), y.data_ptr(), n, k, m)
    assert ref.ref_last_error() == 0
    got = host(y)
    assert np.array_equal(got.view(np.uint32), O.gemv(t, w, rb, x, n, k, m, order=0).view(np.uint32))
    # and this library's engine agrees with the reference kernel to fp32 accuracy
    y2 = torch.empty((m, n), device="cuda:0")
    Q.quant_gemv(t, dev(w).data_ptr(), rb, dev(x).data_ptr(), y2.data_ptr(), n, k, m)
    assert rel_l2(host(y2), got) < 1e-5


def test_reference_router_equals_oracle_and_library(ref):
    import torch
    rng = np.random.default_rng(3)
    lg = rng.standard_normal((64, 64)).astype(np.float32)
    lg[1, :] = 0.25
    lg[2, [3, 30, 50]] = 7.0
    lg[3, ::3] = np.nan
    T, E, k = 64, 64, 6
    ri = torch.empty((T, k), dtype=torch.int32, device="cuda:0")
    rw = torch.empty((T, k), device="cuda:0")
    ref.ref_moe_router_topk(dev(lg).data_ptr(), ri.data_ptr(), rw.data_ptr(), T, E, k, 1.0)
    li = torch.empty((T, k), dtype=torch.int32, device="cuda:0")
    lw = torch.empty((T, k), device="cuda:0")
    Q.moe_router_topk(dev(lg).data_ptr(), li.data_ptr(), lw.data_ptr(), T, E, k, 1.0)
    oi, ow = O.router_topk(lg, k, 1.0)
    assert np.array_equal(host(ri), oi)
    np.testing.assert_allclose(host(rw), ow, rtol=2e-6, atol=1e-7)
    assert np.array_equal(host(li), host(ri))
    assert np.array_equal(host(lw).view(np.uint32), host(rw).view(np.uint32))


def test_reference_moe_gather_combine_close_to_oracle(ref):
    import torch
    t, E, F, K, H, k = O.Q4_K, 4, 256, 512, 512, 3
    g, u = make_weights(t, E * F, K, seed=1), make_weights(t, E * F, K, seed=2)
    d = make_weights(t, E * H, F, seed=3)
    x = np.random.default_rng(4).standard_normal(K).astype(np.float32)
    ids = np.array([2, 0, 3], np.int32)
    rwt = np.array([0.5, 0.3, 0.2], np.float32)
    rbk, rbf = O.row_bytes(t, K), O.row_bytes(t, F)
    act = torch.empty((k, F), device="cuda:0")
    ref.ref_quant_swiglu_indexed(t, dev(g).data_ptr(), dev(u).data_ptr(), F * rbk, F * rbk, rbk, rbk,
                                 dev(x).data_ptr(), dev(ids).data_ptr(), act.data_ptr(), k, F, K)
    oact = O.swiglu_indexed(t, g, u, F * rbk, F * rbk, rbk, rbk, x, ids, k, F, K, order=0)
    assert rel_l2(host(act), oact) < 1e-6
    out = dev(np.zeros(H, np.float32))
    ref.ref_quant_down_ordered(t, dev(d).data_ptr(), H * rbf, rbf, act.data_ptr(), dev(ids).data_ptr(),
                               dev(rwt).data_ptr(), out.data_ptr(), k, H, F)
    oout = O.down_indexed_ordered(t, d, H * rbf, rbf, host(act), ids, rwt, np.zeros(H, np.float32), k, H, F, order=0)
    assert np.array_equal(host(out).view(np.uint32), oout.view(np.uint32))


def test_reference_embedding_and_argmax(ref):
    import torch
    t, V, H = O.Q4_K, 512, 1024
    tab = make_weights(t, V, H, seed=9)
    ids = np.array([0, 511, 17, 17], np.int32)
    out = torch.empty((4, H), device="cuda:0")
    ref.ref_quant_embedding(t, dev(ids).data_ptr(), out.data_ptr(), dev(tab).data_ptr(), O.row_bytes(t, H), H, 4)
    assert np.array_equal(host(out).view(np.uint32), O.embedding(t, ids, tab, O.row_bytes(t, H), H).view(np.uint32))
    v = np.random.default_rng(5).standard_normal(152064).astype(np.float32)
    v[[100, 90000]] = 50.0
    oi = torch.empty(1, dtype=torch.int32, device="cuda:0")
    ref.ref_argmax(dev(v).data_ptr(), v.size, oi.data_ptr())
    assert int(host(oi)[0]) == O.argmax(v) == 100
