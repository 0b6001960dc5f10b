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


def _q8_1_numpy(x, raw):
    """Q8_1 blocks restated in numpy float32 (quantize_q8_1_kernel, kernel.cu:1679-1720)."""
    m, k = x.shape
    bpr = (k + 31) // 32
    out = np.zeros((m, bpr * 36), np.uint8)
    for r in range(m):
        for b in range(bpr):
            v = np.zeros(32, np.float32)
            seg = x[r, b * 32:min(k, b * 32 + 32)]
            v[:len(seg)] = seg
            amax = np.float32(np.max(np.abs(v)))
            d = np.float32(amax / np.float32(127.0)) if amax > 0 else np.float32(0)
            idv = np.float32(np.float32(1.0) / d) if d > 0 else np.float32(0)
            t = v.copy()
            o = 16
            while o:
                t[:o] = t[:o] + t[o:2 * o]
                o //= 2
            q = np.clip(np.rint(v * idv), -127, 127).astype(np.int32)  # rint: round half to even
            s = t[0] if raw else np.float32(d * np.float32(q.sum()))
            blk = out[r, b * 36:(b + 1) * 36]
            blk[0:2] = np.array([d], np.float16).view(np.uint8)
            blk[2:4] = np.array([s], np.float16).view(np.uint8)
            blk[4:36] = q.astype(np.int8).view(np.uint8)
    return out


def test_oracle_quantize_q8_1_matches_numpy():
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((3, 200)) * 3).astype(np.float32)
    x[1, 32:64] = 0.0
    for raw in (False, True):
        assert np.array_equal(O.quantize_q8_1(x, raw), _q8_1_numpy(x, raw))
