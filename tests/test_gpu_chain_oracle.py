"""The benchmarked decode path against the CPU oracle at the Qwen2-7B shapes it is
benchmarked on (hidden 3584, q 3584, k/v 512, FFN 18944, vocabulary 152064), and a
32-token greedy loop against the oracle's greedy loop.

The device runs the persistent chain kernel exactly as bench.py builds it for one GPU:
stacked q/k/v with RMSNorm and bias, o + residual, the fused MLP op (gate/up SwiGLU and
down + residual split over the FFN, fixed-point residual), then RMSNorm + LM head + fused
argmax; a greedy step feeds the token through the quantized embedding
(ql_quant_embedding) into the next chain launch, all on the device.  The oracle restates
the same steps on the CPU (oracle.linear_stack_token, double accumulation).  Bars: linear
outputs within 1e-3 relative L2 (measured ~1e-6), identical
greedy tokens for 32 steps (on a mismatch the test reports the oracle's logit margin).
Weights are N(0, 0.02) quantized to Q4_K by the library's device quantizer and copied to
the host, so both sides read the same bytes."""
import numpy as np
import pytest

import blog_b200 as Q
import oracle as O
from gpu_util import dev, host, rel_l2

pytestmark = pytest.mark.gpu
H, QW, KV, F, V, LAYERS, EPS = 3584, 3584, 512, 18944, 152064, 2, 1e-6


@pytest.fixture(scope="module")
def model():
    import torch
    torch.cuda.init()
    Q.init(0)
    Q.set_stream(torch.cuda.current_stream().cuda_stream)
    O.set_threads(O.host_cores())
    rng = np.random.default_rng(21)

    def synth(rows, k, seed):
        w = torch.empty((rows, Q.row_bytes(Q.Q4_K, k)), dtype=torch.uint8, device="cuda:0")
        Q.synth_quantized(Q.Q4_K, seed, rows, k, 0.02, w.data_ptr())
        return w
    dl, hl = [], []
    for l in range(LAYERS):
        D = {n: synth(r, k, 7000 + 10 * l + i) for i, (n, r, k) in enumerate(
            (("wq", QW, H), ("wk", KV, H), ("wv", KV, H), ("wo", H, QW), ("wg", F, H), ("wu", F, H), ("wd", H, F)))}
        Hh = {n: host(w) for n, w in D.items()}
        for n in ("ln1", "ln2"):
            Hh[n] = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
            D[n] = dev(Hh[n])
        Hh["bqkv"] = (0.01 * rng.standard_normal(QW + 2 * KV)).astype(np.float32)
        D["bqkv"] = dev(Hh["bqkv"])
        dl.append(D)
        hl.append(Hh)
    lm, table = synth(V, H, 7999), synth(V, H, 7998)
    lnf = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    m = {"dev": dl, "host": hl, "lm": lm, "lm_h": host(lm), "table": table, "table_h": host(table),
         "lnf": dev(lnf), "lnf_h": lnf}
    yield m
    Q.check_device()


THETA, HEAD = 1e6, 128


def _chain(m, b, rope=False):
    """The bench's one-GPU op list: qkv (RoPE on q and k when rope), o + residual, fused MLP per
    layer; LM head + argmax."""
    rb = lambda k: Q.row_bytes(Q.Q4_K, k)
    h, ops = b["h"].data_ptr(), []
    rk = dict(rope_pos=b["pos"].data_ptr(), rope_theta=THETA, rope_rows=QW + KV, head_dim=HEAD) if rope else {}
    for L in m["dev"]:
        ops.append(Q.chain_op(Q.OP_STORE, [L["wq"].data_ptr(), L["wk"].data_ptr(), L["wv"].data_ptr()], [rb(H)] * 3,
                              [QW, KV, KV], H, h, b["qkv"].data_ptr(), L["ln1"].data_ptr(), EPS, L["bqkv"].data_ptr(),
                              **rk))
        ops.append(Q.chain_op(Q.OP_ADD, [L["wo"].data_ptr()], [rb(QW)], [H], QW, b["qkv"].data_ptr(), h))
        ops.append(Q.chain_op(Q.OP_MLP, [L["wg"].data_ptr(), L["wu"].data_ptr(), L["wd"].data_ptr()],
                              [rb(H), rb(H), rb(F)], [F, F, H], H, h, h, L["ln2"].data_ptr(), EPS))
    ops.append(Q.chain_op(Q.OP_STORE, [m["lm"].data_ptr()], [rb(H)], [V], H, h, b["logits"].data_ptr(),
                          m["lnf"].data_ptr(), EPS, argmax_idx=b["tok"].data_ptr()))
    return Q.GemvChain(ops)


def _bufs(torch):
    return {"h": torch.zeros(H, device="cuda:0"), "qkv": torch.zeros(QW + 2 * KV, device="cuda:0"),
            "logits": torch.zeros(V, device="cuda:0"), "tok": torch.full((1,), -1, dtype=torch.int32, device="cuda:0"),
            "pos": torch.zeros(1, dtype=torch.int32, device="cuda:0")}


@pytest.mark.parametrize("rope", [False, True])
def test_chain_matches_oracle_at_qwen2_7b_shapes(model, rope):
    import torch
    b = _bufs(torch)
    b["pos"].fill_(37)
    h0 = np.random.default_rng(22).standard_normal(H).astype(np.float32)
    chain = _chain(model, b, rope)
    try:
        b["h"].copy_(dev(h0))
        chain.run()
        h_dev, lg_dev, tok_dev = host(b["h"]), host(b["logits"]), int(host(b["tok"])[0])
        qkv_dev = host(b["qkv"])
        Q.check_device()
    finally:
        chain.close()
    ra = (37, THETA, HEAD, QW + KV) if rope else None
    h_ref, lg_ref, tok_ref = O.linear_stack_token(model["host"], model["lm_h"], model["lnf_h"], h0, eps=EPS,
                                                  rope_args=ra)
    if rope:  # the last layer's q/k/v output, rotated, against the oracle's
        L = model["host"][-1]
        hl = O.linear_stack_token(model["host"][:-1], model["lm_h"], model["lnf_h"], h0, eps=EPS, rope_args=ra,
                                  with_logits=False)[0]
        xn = O.rmsnorm(hl.reshape(1, -1), L["ln1"], EPS)
        qkv_ref = np.concatenate([O.gemv(Q.Q4_K, L[n], L[n].shape[1], xn, L[n].shape[0], H, 1, 1)
                                  for n in ("wq", "wk", "wv")], axis=1) + L["bqkv"]
        qkv_ref = O.rope(qkv_ref, 37, THETA, HEAD, QW + KV)[0]
        e_qkv = rel_l2(qkv_dev, qkv_ref)
        print(f"fused RoPE q/k/v at position 37: rel_l2 {e_qkv:.2e}")
        assert e_qkv < 1e-4
    e_h, e_lg = rel_l2(h_dev, h_ref), rel_l2(lg_dev, lg_ref)
    print(f"chain vs oracle at Qwen2-7B shapes: h rel_l2 {e_h:.2e}, logits rel_l2 {e_lg:.2e}, tokens {tok_dev}/{tok_ref}")
    assert e_h < 1e-3 and e_lg < 1e-3
    assert tok_dev == int(np.argmax(lg_dev))  # the fused argmax is exact on the chain's own logits
    top2 = np.sort(lg_ref)[-2:]
    assert tok_dev == tok_ref, f"token {tok_dev} vs oracle {tok_ref} (oracle margin {top2[1] - top2[0]:.3e})"


def test_greedy_32_tokens_match_oracle(model):
    """32 greedy steps, RoPE on q and k at position = step (the position is a device int, as in
    the reference's graph-captured decode)."""
    import torch
    steps = 32
    b = _bufs(torch)
    first = int(np.random.default_rng(23).integers(0, V))
    hist = torch.zeros(steps, dtype=torch.int32, device="cuda:0")
    b["tok"].fill_(first)
    rbh = Q.row_bytes(Q.Q4_K, H)
    chain = _chain(model, b, rope=True)
    try:
        for i in range(steps):  # token -> embedding -> stack -> argmax -> token, no host round trip
            b["pos"].fill_(i)
            Q.quant_embedding(Q.Q4_K, b["tok"].data_ptr(), b["h"].data_ptr(), model["table"].data_ptr(), rbh, H, 1)
            chain.run()
            hist[i:i + 1].copy_(b["tok"])
        got = [int(t) for t in host(hist)]
        Q.check_device()
    finally:
        chain.close()
    want, margins = O.greedy_decode(model["host"], model["lm_h"], model["lnf_h"], model["table_h"], first, steps,
                                    eps=EPS, rope=(THETA, HEAD, QW + KV))
    print(f"greedy tokens: {got[:8]}..., distinct {len(set(got))}, smallest oracle margin {min(margins):.3e}")
    if got != want:
        i = next(j for j in range(steps) if got[j] != want[j])
        pytest.fail(f"first mismatch at step {i}: device {got[i]} vs oracle {want[i]} "
                    f"(oracle top-2 margin there {margins[i]:.3e})")
