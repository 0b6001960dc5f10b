"""The oracle's decode attention (restating full_attn_attend_head, kernel.cu:355-430) against a
direct numpy evaluation: softmax over the causal window, GQA head mapping, output gate, f32 and
bf16 caches.  CPU only."""
import numpy as np

import oracle as O


def _numpy(q, gate, k, v, tokens, nh, kvh, hd, start):
    out = np.zeros((tokens, nh * hd))
    for t in range(tokens):
        for h in range(nh):
            kh = h // (nh // kvh)
            n = start + t + 1
            kk = k[:n].reshape(n, kvh, hd)[:, kh].astype(np.float64)
            vv = v[:n].reshape(n, kvh, hd)[:, kh].astype(np.float64)
            s = kk @ q[t, h * hd:(h + 1) * hd].astype(np.float64) / np.sqrt(hd)
            p = np.exp(s - s.max())
            p /= p.sum()
            g = gate[t, h * hd:(h + 1) * hd].astype(np.float64)
            out[t, h * hd:(h + 1) * hd] = (p @ vv) / (1 + np.exp(-g))
    return out


def test_oracle_attention_matches_numpy():
    rng = np.random.default_rng(5)
    tokens, nh, kvh, hd, ms, start = 3, 6, 2, 16, 40, 20
    q = rng.standard_normal((tokens, nh * hd)).astype(np.float32)
    gate = rng.standard_normal((tokens, nh * hd)).astype(np.float32)
    k = rng.standard_normal((ms, kvh * hd)).astype(np.float32)
    v = rng.standard_normal((ms, kvh * hd)).astype(np.float32)
    got = O.attention_attend(q, gate, k, v, False, tokens, nh, kvh, hd, start)
    want = _numpy(q, gate, k, v, tokens, nh, kvh, hd, start)
    assert np.max(np.abs(got - want)) < 1e-6
    # bf16 cache: the top 16 bits of each f32
    kb, vb = (k.view(np.uint32) >> 16).astype(np.uint16), (v.view(np.uint32) >> 16).astype(np.uint16)
    kf, vf = ((b.astype(np.uint32) << 16).view(np.float32) for b in (kb, vb))
    got = O.attention_attend(q, gate, kb, vb, True, tokens, nh, kvh, hd, start)
    want = _numpy(q, gate, kf, vf, tokens, nh, kvh, hd, start)
    assert np.max(np.abs(got - want)) < 1e-6
