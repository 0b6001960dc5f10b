"""CPU: the oracle's decode-stack step and greedy loop (the checker of the GPU chain and
greedy-parity tests) against an independent float64 numpy restatement built on the
oracle's bit-exact dequantizer."""
import numpy as np

import oracle as O

H, QW, KV, F, V = 512, 512, 64, 1024, 700


def _model(seed=3):
    rng = np.random.default_rng(seed)
    q = lambda r, k, s: O.quantize(O.Q4_K, O.randn(s, r * k, 0.02).reshape(r, k))
    layers = []
    for l in range(2):
        L = {n: q(r, k, 50 + 10 * l + i) for i, (n, r, k) in enumerate(
            (("wq", QW, H), ("wk", KV, H), ("wv", KV, H), ("wo", H, QW), ("wg", F, H), ("wu", F, H), ("wd", H, F)))}
        L["ln1"] = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        L["ln2"] = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
        L["bqkv"] = (0.01 * rng.standard_normal(QW + 2 * KV)).astype(np.float32)
        layers.append(L)
    lm, table = q(V, H, 98), q(V, H, 99)
    lnf = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    return layers, lm, lnf, table


def _numpy_token(layers, lm, lnf, h, eps=1e-6):
    W = lambda w, k: O.dequant_rows(O.Q4_K, w, k).astype(np.float64)
    norm = lambda x, g: x / np.sqrt(np.mean(x * x) + eps) * g
    h = h.astype(np.float64)
    for L in layers:
        xn = norm(h, L["ln1"])
        qkv = np.concatenate([W(L[n], H) @ xn for n in ("wq", "wk", "wv")]) + L["bqkv"]
        h = h + W(L["wo"], QW) @ qkv[:QW]
        xn = norm(h, L["ln2"])
        gv, uv = W(L["wg"], H) @ xn, W(L["wu"], H) @ xn
        h = h + W(L["wd"], F) @ (gv / (1 + np.exp(-gv)) * uv)
    return h, W(lm, H) @ norm(h, lnf)


def test_linear_stack_token_matches_numpy():
    layers, lm, lnf, _ = _model()
    h0 = np.random.default_rng(4).standard_normal(H).astype(np.float32)
    h, logits, tok = O.linear_stack_token(layers, lm, lnf, h0)
    h_ref, lg_ref = _numpy_token(layers, lm, lnf, h0)
    assert np.linalg.norm(h - h_ref) / np.linalg.norm(h_ref) < 1e-6
    assert np.linalg.norm(logits - lg_ref) / np.linalg.norm(lg_ref) < 1e-6
    assert tok == int(np.argmax(lg_ref))


def test_greedy_decode_follows_embedding_rows():
    layers, lm, lnf, table = _model()
    toks, margins = O.greedy_decode(layers, lm, lnf, table, 5, 6)
    assert len(toks) == 6 and all(m >= 0 for m in margins)
    tok = 5
    for want in toks:  # the loop feeds each token's embedding row into the next step
        h = O.dequant_rows(O.Q4_K, table[tok:tok + 1], H)[0]
        _, lg = _numpy_token(layers, lm, lnf, h)
        tok = int(np.argmax(lg))
        assert tok == want


def test_linear_stack_batch_matches_per_token():
    layers, lm, lnf, _ = _model()
    hb = np.random.default_rng(6).standard_normal((3, H)).astype(np.float32)
    h, lg = O.linear_stack_batch(layers, lm, lnf, hb)
    for i in range(3):
        h1, lg1 = _numpy_token(layers, lm, lnf, hb[i])
        assert np.allclose(h[i], h1, rtol=1e-12, atol=1e-12)
        assert np.allclose(lg[i], lg1, rtol=1e-12, atol=1e-12)
