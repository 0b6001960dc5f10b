"""The persistent GEMV chain (one cooperative launch for a decoder stack) against
the same ops run one launch at a time through the per-op entry points.

The per-op launches compute exact fp32 products on the CUDA cores; the chain runs the
Q4_K blocks on the integer tensor cores against activations staged as 21-bit fixed-point
limbs per 256-element block, and splits every op over all SMs (stream-K).  Results agree
within 1e-5 relative L2, and the fused argmax is exact on the chain's own logits."""
import numpy as np
import pytest

import blog_b200 as Q
import oracle as O
from gpu_util import dev, host, make_weights, rel_l2

pytestmark = pytest.mark.gpu
H, QW, KV, F, V, LAYERS, EPS = 2048, 2048, 256, 4096, 5000, 2, 1e-6


@pytest.fixture(scope="module", autouse=True)
def _stream():
    import torch
    torch.cuda.init()
    Q.init(0)
    Q.set_stream(torch.cuda.current_stream().cuda_stream)
    yield
    Q.check_device()


def _stack(torch):
    rng = np.random.default_rng(5)
    rb = lambda k: O.row_bytes(O.Q4_K, k)
    layers = []
    for l in range(LAYERS):
        L = {n: dev(make_weights(O.Q4_K, r, k, seed=300 + 10 * l + i))
             for i, (n, r, k) in enumerate((("wq", QW, H), ("wk", KV, H), ("wv", KV, H), ("wo", H, QW),
                                            ("wg", F, H), ("wu", F, H), ("wd", H, F)))}
        L["ln1"] = dev((1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
        L["ln2"] = dev((1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
        L["b"] = dev((0.01 * rng.standard_normal(QW + 2 * KV)).astype(np.float32))
        layers.append(L)
    lm = dev(make_weights(O.Q4_K, V, H, seed=399))
    lnf = dev((1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
    return layers, lm, lnf, rb


def _bufs(torch, h0):
    return {"h": dev(h0.copy()), "qkv": torch.zeros(QW + 2 * KV, device="cuda:0"),
            "act": torch.zeros(F, device="cuda:0"), "logits": torch.zeros(V, device="cuda:0"),
            "tok": torch.full((1,), -1, dtype=torch.int32, device="cuda:0")}


def _per_op(torch, layers, lm, lnf, rb, b):
    h = b["h"].data_ptr()
    for L in layers:
        Q.quant_gemv_stacked_ex(O.Q4_K, [L["wq"].data_ptr(), L["wk"].data_ptr(), L["wv"].data_ptr()], [rb(H)] * 3,
                                [QW, KV, KV], h, H, b["qkv"].data_ptr(), QW + 2 * KV, H, 1, L["ln1"].data_ptr(), EPS,
                                L["b"].data_ptr())
        Q.quant_gemv_ex(O.Q4_K, L["wo"].data_ptr(), rb(QW), b["qkv"].data_ptr(), QW, h, H, H, QW, 1, accumulate=True)
        Q.quant_swiglu_ex(O.Q4_K, L["wg"].data_ptr(), L["wu"].data_ptr(), rb(H), rb(H), h, H, b["act"].data_ptr(), F,
                          F, H, 1, L["ln2"].data_ptr(), EPS)
        Q.quant_gemv_ex(O.Q4_K, L["wd"].data_ptr(), rb(F), b["act"].data_ptr(), F, h, H, H, F, 1, accumulate=True)
    Q.quant_gemv_ex(O.Q4_K, lm.data_ptr(), rb(H), h, H, b["logits"].data_ptr(), V, V, H, 1, lnf.data_ptr(), EPS)


def _chain_ops(layers, lm, lnf, rb, b, with_logits=True, mlp=False):
    h = b["h"].data_ptr()
    ops = []
    for L in layers:
        ops.append(Q.chain_op(Q.OP_STORE, [L["wq"].data_ptr(), L["wk"].data_ptr(), L["wv"].data_ptr()], [rb(H)] * 3,
                              [QW, KV, KV], H, h, b["qkv"].data_ptr(), L["ln1"].data_ptr(), EPS, L["b"].data_ptr()))
        ops.append(Q.chain_op(Q.OP_ADD, [L["wo"].data_ptr()], [rb(QW)], [H], QW, b["qkv"].data_ptr(), h))
        if mlp:  # gate/up SwiGLU and down + residual as one op (split over the FFN)
            ops.append(Q.chain_op(Q.OP_MLP, [L["wg"].data_ptr(), L["wu"].data_ptr(), L["wd"].data_ptr()],
                                  [rb(H), rb(H), rb(F)], [F, F, H], H, h, h, L["ln2"].data_ptr(), EPS))
            continue
        ops.append(Q.chain_op(Q.OP_SWIGLU, [L["wg"].data_ptr(), L["wu"].data_ptr()], [rb(H)] * 2, [F, F], H, h,
                              b["act"].data_ptr(), L["ln2"].data_ptr(), EPS))
        ops.append(Q.chain_op(Q.OP_ADD, [L["wd"].data_ptr()], [rb(F)], [H], F, b["act"].data_ptr(), h))
    ops.append(Q.chain_op(Q.OP_STORE, [lm.data_ptr()], [rb(H)], [V], H, h,
                          b["logits"].data_ptr() if with_logits else None, lnf.data_ptr(), EPS,
                          argmax_idx=b["tok"].data_ptr()))
    return ops


def test_chain_matches_per_op_launches():
    import torch
    layers, lm, lnf, rb = _stack(torch)
    h0 = np.random.default_rng(6).standard_normal(H).astype(np.float32)
    ref = _bufs(torch, h0)
    _per_op(torch, layers, lm, lnf, rb, ref)
    got = _bufs(torch, h0)
    chain = Q.GemvChain(_chain_ops(layers, lm, lnf, rb, got))
    try:
        chain.run()
        for k in ("qkv", "act", "h", "logits"):
            assert rel_l2(host(got[k]), host(ref[k])) < 1e-5, k
        lg = host(got["logits"])
        assert host(got["tok"])[0] == int(np.argmax(lg))
        # replays (graph-style: monotonic counters, no resets) give identical results
        for _ in range(3):
            got["h"].copy_(dev(h0))
            chain.run()
        assert np.array_equal(host(got["logits"]).view(np.uint32), lg.view(np.uint32))
        assert host(got["tok"])[0] == int(np.argmax(lg))
    finally:
        chain.close()


def test_chain_fused_mlp_matches_per_op_launches():
    import torch
    layers, lm, lnf, rb = _stack(torch)
    h0 = np.random.default_rng(8).standard_normal(H).astype(np.float32)
    ref = _bufs(torch, h0)
    _per_op(torch, layers, lm, lnf, rb, ref)
    got = _bufs(torch, h0)
    chain = Q.GemvChain(_chain_ops(layers, lm, lnf, rb, got, mlp=True))
    try:
        chain.run()
        for k in ("qkv", "h", "logits"):
            assert rel_l2(host(got[k]), host(ref[k])) < 1e-5, k
        lg = host(got["logits"])
        assert host(got["tok"])[0] == int(np.argmax(lg))
        # the split-K partial sums add in fixed point: replays are bit-identical
        for _ in range(3):
            got["h"].copy_(dev(h0))
            chain.run()
        assert np.array_equal(host(got["logits"]).view(np.uint32), lg.view(np.uint32))
    finally:
        chain.close()


def test_chain_fused_mlp_rejects_unseeded_residual():
    import torch
    layers, lm, lnf, rb = _stack(torch)
    b = _bufs(torch, np.zeros(H, np.float32))
    L = layers[0]
    h = b["h"].data_ptr()
    mlp = Q.chain_op(Q.OP_MLP, [L["wg"].data_ptr(), L["wu"].data_ptr(), L["wd"].data_ptr()], [rb(H), rb(H), rb(F)],
                     [F, F, H], H, h, h, L["ln2"].data_ptr(), EPS)
    lmop = Q.chain_op(Q.OP_STORE, [lm.data_ptr()], [rb(H)], [V], H, h, b["logits"].data_ptr(), lnf.data_ptr(), EPS)
    with pytest.raises(Q.QLError):  # no ADD op of the chain wrote the residual first
        Q.GemvChain([mlp, lmop])


def test_chain_captured_in_graph():
    import torch
    layers, lm, lnf, rb = _stack(torch)
    h0 = np.random.default_rng(7).standard_normal(H).astype(np.float32)
    b = _bufs(torch, h0)
    h_in = dev(h0)
    chain = Q.GemvChain(_chain_ops(layers, lm, lnf, rb, b, with_logits=False))
    try:
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            Q.set_stream(s.cuda_stream)
            b["h"].copy_(h_in)
            chain.run()
            torch.cuda.synchronize()
            first = int(host(b["tok"])[0])
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                b["h"].copy_(h_in)
                chain.run()
            for _ in range(5):
                g.replay()
            torch.cuda.synchronize()
        Q.set_stream(torch.cuda.current_stream().cuda_stream)
        assert int(host(b["tok"])[0]) == first
        del g
    finally:
        Q.set_stream(torch.cuda.current_stream().cuda_stream)
        chain.close()
