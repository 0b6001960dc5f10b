"""The batched decode chain (ql_gemv_chain_create_batch: up to 32 tokens per launch on the
tensor cores) against the CPU oracle.

Each token of the batch runs the decode stack of the one-token chain (stacked q/k/v with
RMSNorm and bias, o + residual, gate/up SwiGLU with RMSNorm, down + residual, LM head with
RMSNorm and a greedy argmax per token).  The oracle (oracle.linear_stack_batch) uses the
exact dequantized weights and float64 accumulation.  The kernel rounds weights and
activations to f16 and accumulates in fp32.  Bars: every linear on its own (one-op chains
of each kind) within 1e-3 relative L2, the north-star tolerance for a linear output; the
whole 2-layer stack (9 linears feeding each other through the residual stream, so the
per-linear errors compound) within 2.5e-3.  Greedy tokens must equal the argmax of the
kernel's own logits, and the oracle's token wherever the oracle's top-2 margin exceeds ten
times the logits' error."""
import numpy as np
import pytest

import blog_b200 as Q
import oracle as O
from gpu_util import dev, host, rel_l2

pytestmark = pytest.mark.gpu
EPS = 1e-6


@pytest.fixture(scope="module", autouse=True)
def _stream():
    import torch
    torch.cuda.init()
    Q.init(0)
    Q.set_stream(torch.cuda.current_stream().cuda_stream)
    O.set_threads(O.host_cores())
    yield
    Q.check_device()


def _model(H, QW, KV, F, V, layers, seed):
    import torch
    rng = np.random.default_rng(seed)

    def synth(rows, k, s):
        w = torch.empty((rows, Q.row_bytes(Q.Q4_K, k)), dtype=torch.uint8, device="cuda:0")
        Q.synth_quantized(Q.Q4_K, s, rows, k, 0.02, w.data_ptr())
        return w
    dl, hl = [], []
    for l in range(layers):
        D = {n: synth(r, k, seed * 100 + 10 * l + i) for i, (n, r, k) in enumerate(
            (("wq", QW, H), ("wk", KV, H), ("wv", KV, H), ("wo", H, QW), ("wg", F, H), ("wu", F, H), ("wd", H, F)))}
        Hh = {n: host(w) for n, w in D.items()}
        for n in ("ln1", "ln2"):
            Hh[n] = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
            D[n] = dev(Hh[n])
        Hh["bqkv"] = (0.01 * rng.standard_normal(QW + 2 * KV)).astype(np.float32)
        D["bqkv"] = dev(Hh["bqkv"])
        dl.append(D)
        hl.append(Hh)
    lm = synth(V, H, seed * 100 + 99)
    lnf = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    return {"dev": dl, "host": hl, "lm": lm, "lm_h": host(lm), "lnf": dev(lnf), "lnf_h": lnf,
            "dims": (H, QW, KV, F, V)}


THETA = 1e6


def _positions(M):
    return (5 + 3 * np.arange(M)).astype(np.int32)


def _run(m, M, h0, replays=1, head_dim=128):
    """The stack as one batched chain, RoPE on q and k (rows of whole heads) at _positions(M)."""
    import torch
    H, QW, KV, F, V = m["dims"]
    rb = lambda k: Q.row_bytes(Q.Q4_K, k)
    b = {"h": dev(h0.copy()), "qkv": torch.zeros((M, QW + 2 * KV), device="cuda:0"),
         "act": torch.zeros((M, F), device="cuda:0"), "logits": torch.zeros((M, V), device="cuda:0"),
         "tok": torch.full((M,), -1, dtype=torch.int32, device="cuda:0"), "pos": dev(_positions(M))}
    hp, ops = b["h"].data_ptr(), []
    for L in m["dev"]:
        ops.append(Q.chain_op(Q.OP_STORE, [L["wq"].data_ptr(), L["wk"].data_ptr(), L["wv"].data_ptr()], [rb(H)] * 3,
                              [QW, KV, KV], H, hp, b["qkv"].data_ptr(), L["ln1"].data_ptr(), EPS, L["bqkv"].data_ptr(),
                              x_stride=H, y_stride=QW + 2 * KV, rope_pos=b["pos"].data_ptr(), rope_theta=THETA,
                              rope_rows=QW + KV, head_dim=head_dim))
        ops.append(Q.chain_op(Q.OP_ADD, [L["wo"].data_ptr()], [rb(QW)], [H], QW, b["qkv"].data_ptr(), hp,
                              x_stride=QW + 2 * KV, y_stride=H))
        ops.append(Q.chain_op(Q.OP_SWIGLU, [L["wg"].data_ptr(), L["wu"].data_ptr()], [rb(H)] * 2, [F, F], H, hp,
                              b["act"].data_ptr(), L["ln2"].data_ptr(), EPS, x_stride=H, y_stride=F))
        ops.append(Q.chain_op(Q.OP_ADD, [L["wd"].data_ptr()], [rb(F)], [H], F, b["act"].data_ptr(), hp,
                              x_stride=F, y_stride=H))
    ops.append(Q.chain_op(Q.OP_STORE, [m["lm"].data_ptr()], [rb(H)], [V], H, hp, b["logits"].data_ptr(),
                          m["lnf"].data_ptr(), EPS, argmax_idx=b["tok"].data_ptr(), x_stride=H, y_stride=V))
    chain = Q.GemvChain(ops, tokens=M)
    outs = []
    try:
        for _ in range(replays):
            b["h"].copy_(dev(h0))
            chain.run()
            outs.append((host(b["h"]).copy(), host(b["logits"]).copy(), host(b["tok"]).copy()))
        Q.check_device()
    finally:
        chain.close()
    return outs


def _check(m, M, h0, outs, bar=2.5e-3, head_dim=128):
    H, QW, KV, F, V = m["dims"]
    h_ref, lg_ref = O.linear_stack_batch(m["host"], m["lm_h"], m["lnf_h"], h0, eps=EPS,
                                         rope_args=(_positions(M), THETA, head_dim, QW + KV))
    h, lg, tok = outs[0]
    e_h, e_lg = rel_l2(h, h_ref), rel_l2(lg, lg_ref)
    print(f"batched chain M={M}: h rel_l2 {e_h:.2e}, logits rel_l2 {e_lg:.2e}")
    assert e_h < bar and e_lg < bar
    for i in range(M):
        assert tok[i] == int(np.argmax(lg[i])), i
        top2 = np.sort(lg_ref[i])[-2:]
        err = float(np.max(np.abs(lg[i] - lg_ref[i])))
        if top2[1] - top2[0] > 10 * err:
            assert tok[i] == int(np.argmax(lg_ref[i])), (i, tok[i], int(np.argmax(lg_ref[i])))
    for h2, lg2, tok2 in outs[1:]:  # replays: deterministic, bit for bit
        assert np.array_equal(h2.view(np.uint32), h.view(np.uint32))
        assert np.array_equal(lg2.view(np.uint32), lg.view(np.uint32))
        assert np.array_equal(tok2, tok)


@pytest.mark.parametrize("M", [1, 8, 20, 32])
def test_batched_chain_small_shapes(M):
    m = _model(2048, 2048, 256, 4096, 5000, 2, seed=41)
    h0 = np.random.default_rng(M).standard_normal((M, 2048)).astype(np.float32)
    _check(m, M, h0, _run(m, M, h0, replays=3))


def test_batched_chain_qwen2_7b_shapes():
    m = _model(3584, 3584, 512, 18944, 152064, 2, seed=43)
    M = 32
    h0 = np.random.default_rng(9).standard_normal((M, 3584)).astype(np.float32)
    _check(m, M, h0, _run(m, M, h0, replays=2))


@pytest.mark.parametrize("op", ["qkv", "o", "gate", "up", "swiglu", "down", "lmhead"])
def test_batched_chain_each_linear(op):
    """One linear of each kind as a one-op batched chain (32 tokens) against the oracle.  The
    SwiGLU op's output is SiLU(gate) * up, the product of two linear outputs (each checked here on
    its own as a STORE op at 1e-3), so its bar is 1.5e-3."""
    import torch
    H, QW, KV, F, V, M = 3584, 3584, 512, 18944, 152064, 32
    m = _model(H, QW, KV, F, V, 1, seed=45)
    L, Lh = m["dev"][0], m["host"][0]
    rb = lambda k: Q.row_bytes(Q.Q4_K, k)
    rng = np.random.default_rng(46)
    k_in = {"qkv": H, "o": QW, "gate": H, "up": H, "swiglu": H, "down": F, "lmhead": H}[op]
    x = rng.standard_normal((M, k_in)).astype(np.float32)
    xd = dev(x)
    xn = O.rmsnorm(x, Lh["ln1"] if op == "qkv" else Lh["ln2"] if op in ("swiglu", "gate", "up") else m["lnf_h"],
                   EPS)
    W = lambda w, k: O._dq(Q.Q4_K, w, k)
    if op == "qkv":
        y = torch.zeros((M, QW + 2 * KV), device="cuda:0")
        opd = Q.chain_op(Q.OP_STORE, [L["wq"].data_ptr(), L["wk"].data_ptr(), L["wv"].data_ptr()], [rb(H)] * 3,
                         [QW, KV, KV], H, xd.data_ptr(), y.data_ptr(), L["ln1"].data_ptr(), EPS, L["bqkv"].data_ptr())
        ref = np.concatenate([xn @ W(Lh[n], H).T for n in ("wq", "wk", "wv")], axis=1) + Lh["bqkv"]
    elif op in ("o", "down"):
        base = rng.standard_normal((M, H)).astype(np.float32)
        y = dev(base)
        w = "wo" if op == "o" else "wd"
        opd = Q.chain_op(Q.OP_ADD, [L[w].data_ptr()], [rb(k_in)], [H], k_in, xd.data_ptr(), y.data_ptr())
        ref = base + x.astype(np.float64) @ W(Lh[w], k_in).T
    elif op in ("gate", "up"):
        w = "wg" if op == "gate" else "wu"
        y = torch.zeros((M, F), device="cuda:0")
        opd = Q.chain_op(Q.OP_STORE, [L[w].data_ptr()], [rb(H)], [F], H, xd.data_ptr(), y.data_ptr(),
                         L["ln2"].data_ptr(), EPS)
        ref = xn @ W(Lh[w], H).T
    elif op == "swiglu":
        y = torch.zeros((M, F), device="cuda:0")
        opd = Q.chain_op(Q.OP_SWIGLU, [L["wg"].data_ptr(), L["wu"].data_ptr()], [rb(H)] * 2, [F, F], H,
                         xd.data_ptr(), y.data_ptr(), L["ln2"].data_ptr(), EPS)
        gv, uv = xn @ W(Lh["wg"], H).T, xn @ W(Lh["wu"], H).T
        ref = gv / (1 + np.exp(-gv)) * uv
    else:
        y = torch.zeros((M, V), device="cuda:0")
        tok = torch.full((M,), -1, dtype=torch.int32, device="cuda:0")
        opd = Q.chain_op(Q.OP_STORE, [m["lm"].data_ptr()], [rb(H)], [V], H, xd.data_ptr(), y.data_ptr(),
                         m["lnf"].data_ptr(), EPS, argmax_idx=tok.data_ptr())
        ref = xn @ O._dq(Q.Q4_K, m["lm_h"], H).T
    chain = Q.GemvChain([opd], tokens=M)
    try:
        chain.run()
        got = host(y)
        Q.check_device()
    finally:
        chain.close()
    err = rel_l2(got, ref) if op not in ("o", "down") else rel_l2(got - base, ref - base)
    print(f"batched chain, one {op} linear, 32 tokens: rel_l2 {err:.2e}")
    assert err < (1.5e-3 if op == "swiglu" else 1e-3)
    if op == "lmhead":
        assert np.array_equal(host(tok), np.argmax(got, axis=1).astype(np.int32))


def test_batched_chain_rejects_unsupported_ops():
    import torch
    m = _model(2048, 2048, 256, 4096, 5000, 1, seed=44)
    L = m["dev"][0]
    rb = Q.row_bytes(Q.Q4_K, 2048)
    h = torch.zeros((4, 2048), device="cuda:0")
    mlp = Q.chain_op(Q.OP_MLP, [L["wg"].data_ptr(), L["wu"].data_ptr(), L["wd"].data_ptr()],
                     [rb, rb, Q.row_bytes(Q.Q4_K, 4096)], [4096, 4096, 2048], 2048, h.data_ptr(), h.data_ptr(),
                     L["ln2"].data_ptr(), EPS)
    with pytest.raises(Q.QLError):
        Q.GemvChain([mlp], tokens=4)
    st = Q.chain_op(Q.OP_STORE, [L["wq"].data_ptr()], [rb], [2048], 2048, h.data_ptr(), h.data_ptr())
    with pytest.raises(Q.QLError):
        Q.GemvChain([st], tokens=33)
