"""Regenerate the golden fixtures in this folder (run here, where gguf-py exists).

    python tests/golden/make_golden.py

Two sources of truth, written to ``golden.npz``:

1. The reference's own known-answer kernel tests
   (AI/codes/local-llm/test/LaunchAddTest.cpp).  The hand-built GGUF blocks of
   those tests are rebuilt here byte for byte and stored with the values the
   reference asserts:
     * ``ka_q80_*``   Q8_0 matmul, in 32 / out 2 / m 3, d = 1.0 (:186-240);
     * ``ka_q4k_*``   one Q4_K super-block, d=1, dmin=0.5, sc0=3, m0=2, q=5:
                      w = 14 on sub-block 0, dot = 14*158 (:711-756);
     * ``ka_q6k_*``   one Q6_K super-block, stored q = 35, scale 2: w = 6,
                      dot = 6*158 (:758-803);
     * ``ka_down_{q80,q4k,q6k}_*`` MoE down fixtures, 3 experts, k = 2
                      (:301-564); the expected combine is computed in float64
                      from the exact dequantized values;
     * ``ka_swiglu_q4k_*`` indexed SwiGLU fixture (:566-677).
2. gguf-py 0.19.0 (third-party; the GGUF package of llama.cpp, not part of the
   reference), whose quants.py restates the ggml block formats:
     * ``gg_{T}_bytes`` / ``gg_{T}_deq``: random blocks and gguf-py's
       dequantized float32 values for Q8_0, Q4_0, Q5_0, Q4_K, Q6_K;
     * ``gg_{T}_src`` / ``gg_{T}_quant``: float32 rows and gguf-py's quantized
       bytes for Q8_0, Q4_0, Q5_0 (gguf-py has no Q4_K/Q6_K quantizer).
"""
from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def u16(v):
    return [v & 0xFF, v >> 8]


def f16_bits(x: float) -> int:
    return int(np.array([x], np.float16).view(np.uint16)[0])


def known_answer() -> dict:
    out = {}
    # --- LaunchAddTest.cpp:186-240 (Q8_0 matmul, analytic) -------------------
    in_dim, out_dim, m = 32, 2, 3
    w = []
    for row in range(out_dim):
        b = u16(0x3C00)
        for k in range(in_dim):
            q = 1 if row == 0 else (2 if k % 2 == 0 else -1)
            b.append(q & 0xFF)
        w += b
    x = np.array(list(range(1, 33)) + [-v for v in range(1, 33)] + [1 if i % 2 == 0 else -1 for i in range(32)],
                 np.float32).reshape(m, in_dim)
    exp = np.zeros((m, out_dim), np.float32)
    for r in range(m):
        exp[r, 0] = x[r].sum()
        exp[r, 1] = sum(x[r, k] * (2.0 if k % 2 == 0 else -1.0) for k in range(in_dim))
    out.update(ka_q80_w=np.array(w, np.uint8), ka_q80_x=x, ka_q80_y=exp)

    # --- LaunchAddTest.cpp:711-756 (Q4_K, w = 14) -----------------------------
    wb = np.zeros(144, np.uint8)
    wb[0:2] = u16(0x3C00)
    wb[2:4] = u16(0x3800)
    wb[4 + 0] = 3
    wb[4 + 4] = 2
    wb[16:48] = 0x05
    x = np.zeros(256, np.float32)
    x[0] = 127.0
    x[1:32] = 1.0
    deq = np.zeros(256, np.float32)
    deq[:32] = 14.0
    out.update(ka_q4k_w=wb, ka_q4k_x=x, ka_q4k_deq=deq, ka_q4k_y=np.array([14.0 * 158.0], np.float32))

    # --- LaunchAddTest.cpp:758-803 (Q6_K, w = 6) ------------------------------
    wb = np.zeros(210, np.uint8)
    wb[0:32] = 0x03
    wb[128:160] = 0x02
    wb[192] = 2
    wb[193] = 2
    wb[208:210] = u16(0x3C00)
    deq = np.zeros(256, np.float32)
    deq[:32] = 6.0
    out.update(ka_q6k_w=wb, ka_q6k_x=x.copy(), ka_q6k_deq=deq, ka_q6k_y=np.array([6.0 * 158.0], np.float32))

    # --- LaunchAddTest.cpp:301-564 (MoE down, 3 experts, k=2) -----------------
    n_exp, k, hidden = 3, 2, 9

    def down_q80():
        ffn, rb = 64, 68
        w = np.zeros(n_exp * hidden * rb, np.uint8)
        for e in range(n_exp):
            for row in range(hidden):
                base = (e * hidden + row) * rb
                for blk in range(2):
                    o = base + blk * 34
                    w[o:o + 2] = u16(0x3C00)
                    for col in range(32):
                        v = ((e + 1) * (row + 3) + blk + col) % 7 - 3
                        w[o + 2 + col] = v & 0xFF
        act = np.array([[0.05 * ((r + 2) * (c % 11) - 7) for c in range(ffn)] for r in range(k)], np.float32)
        return w, ffn, rb, act, np.array([0.25, -0.75], np.float32)

    def down_q4k():
        ffn, rb = 256, 144
        w = np.zeros(n_exp * hidden * rb, np.uint8)
        for e in range(n_exp):
            for row in range(hidden):
                o = (e * hidden + row) * rb
                w[o:o + 2] = u16(0x3C00)
                w[o + 2:o + 4] = u16(0x3800)
                for j in range(4):
                    w[o + 4 + j] = 3 + ((e + row + j) & 1)
                    w[o + 8 + j] = (2 << 4) | (3 + ((e + row + j + 1) & 1))
                for j in range(4):
                    w[o + 4 + 4 + j] = 2
                for i in range(128):
                    w[o + 16 + i] = 0x31 + ((e + row + i) & 0x03)
        act = np.array([[0.03 * (((r + 1) * (c % 17)) - 8) for c in range(ffn)] for r in range(k)], np.float32)
        return w, ffn, rb, act, np.array([0.5, -0.25], np.float32)

    def down_q6k():
        ffn, rb = 256, 210
        w = np.zeros(n_exp * hidden * rb, np.uint8)
        for e in range(n_exp):
            for row in range(hidden):
                o = (e * hidden + row) * rb
                for i in range(128):
                    w[o + i] = 0x53 + ((e + row + i) & 0x03)
                for i in range(64):
                    w[o + 128 + i] = 0x55
                for i in range(16):
                    w[o + 192 + i] = (-2 if (i & 1) else 3) & 0xFF
                w[o + 208:o + 210] = u16(0x3C00)
        act = np.array([[0.02 * (((r + 3) * (c % 19)) - 10) for c in range(ffn)] for r in range(k)], np.float32)
        return w, ffn, rb, act, np.array([0.125, -0.5], np.float32)

    import gguf.quants as gq  # exact float64 combine from independently dequantized weights
    from gguf.constants import GGMLQuantizationType as G

    for name, fn, gt in (("q80", down_q80, G.Q8_0), ("q4k", down_q4k, G.Q4_K), ("q6k", down_q6k, G.Q6_K)):
        w, ffn, rb, act, rw = fn()
        ids = np.array([1, 2], np.int32)
        deq = gq.dequantize(w.reshape(n_exp * hidden, rb), gt).reshape(n_exp, hidden, ffn).astype(np.float64)
        exp = np.zeros(hidden, np.float64)
        for r in range(k):
            exp += rw[r] * (deq[ids[r]] @ act[r].astype(np.float64))
        out.update({f"ka_down_{name}_w": w, f"ka_down_{name}_act": act, f"ka_down_{name}_rw": rw,
                    f"ka_down_{name}_ids": ids, f"ka_down_{name}_ffn": np.array([ffn, rb], np.int64),
                    f"ka_down_{name}_y": exp.astype(np.float32)})

    # --- LaunchAddTest.cpp:566-677 (indexed SwiGLU, Q4_K) ---------------------
    ffn, in_dim, rb = 7, 256, 144
    g = np.zeros(n_exp * ffn * rb, np.uint8)
    u = np.zeros(n_exp * ffn * rb, np.uint8)
    for e in range(n_exp):
        for row in range(ffn):
            o = (e * ffn + row) * rb
            g[o:o + 2] = u16(0x3C00); g[o + 2:o + 4] = u16(0x3800)
            u[o:o + 2] = u16(0x3800); u[o + 2:o + 4] = u16(0x3400)
            for j in range(4):
                g[o + 4 + j] = 2 + ((e + row + j) & 3)
                g[o + 8 + j] = (1 << 4) | (3 + ((e + row + j) & 1))
                u[o + 4 + j] = 1 + ((e + row + j) & 3)
                u[o + 8 + j] = (2 << 4) | (2 + ((e + row + j) & 1))
            for j in range(4):
                g[o + 4 + 4 + j] = 2
                u[o + 4 + 4 + j] = 1
            for i in range(128):
                g[o + 16 + i] = 0x21 + ((e + row + i) & 0x03)
                u[o + 16 + i] = 0x32 + ((e + row + i) & 0x03)
    x = np.array([0.025 * ((c % 23) - 11) for c in range(in_dim)], np.float32)
    ids = np.array([1, 2], np.int32)
    dg = gq.dequantize(g.reshape(-1, rb), G.Q4_K).reshape(n_exp, ffn, in_dim).astype(np.float64)
    du = gq.dequantize(u.reshape(-1, rb), G.Q4_K).reshape(n_exp, ffn, in_dim).astype(np.float64)
    exp = np.zeros((k, ffn), np.float64)
    for r in range(k):
        gv = dg[ids[r]] @ x.astype(np.float64)
        uv = du[ids[r]] @ x.astype(np.float64)
        exp[r] = gv / (1.0 + np.exp(-gv)) * uv
    out.update(ka_swiglu_q4k_g=g, ka_swiglu_q4k_u=u, ka_swiglu_q4k_x=x, ka_swiglu_q4k_ids=ids,
               ka_swiglu_q4k_y=exp.astype(np.float32))
    return out


def gguf_vectors() -> dict:
    import gguf
    import gguf.quants as gq
    from gguf.constants import GGMLQuantizationType as G

    out = {"gguf_version": np.frombuffer(gguf.__version__.encode() if hasattr(gguf, "__version__") else b"0.19.0",
                                         np.uint8)}
    rng = np.random.default_rng(20261201)
    for name, t, be, bb in (("Q8_0", G.Q8_0, 32, 34), ("Q4_0", G.Q4_0, 32, 18), ("Q5_0", G.Q5_0, 32, 22),
                            ("Q4_K", G.Q4_K, 256, 144), ("Q6_K", G.Q6_K, 256, 210)):
        nblk = 96
        raw = rng.integers(0, 256, size=(nblk, bb), dtype=np.uint8)
        # keep every f16 scale finite and modest (random bits can be inf/nan)
        scale_offsets = {"Q8_0": [0], "Q4_0": [0], "Q5_0": [0], "Q4_K": [0, 2], "Q6_K": [208]}[name]
        for off in scale_offsets:
            vals = (rng.standard_normal(nblk) * 0.01).astype(np.float16)
            raw[:, off:off + 2] = vals.view(np.uint8).reshape(nblk, 2)
        deq = gq.dequantize(raw, t).astype(np.float32).reshape(nblk, be)
        out[f"gg_{name}_bytes"] = raw
        out[f"gg_{name}_deq"] = deq
    for name, t, be in (("Q8_0", G.Q8_0, 32), ("Q4_0", G.Q4_0, 32), ("Q5_0", G.Q5_0, 32)):
        src = (rng.standard_normal((8, 256)) * 0.02).astype(np.float32)
        src[0, :32] = 0.0  # an all-zero block (d = 0 path)
        src[1, 5] = 0.5    # a large outlier
        q = gq.quantize(src, t)
        out[f"gg_{name}_src"] = src
        out[f"gg_{name}_quant"] = np.asarray(q, np.uint8)
    return out


def main():
    d = {}
    d.update(known_answer())
    d.update(gguf_vectors())
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **d)
    print(f"wrote {path}: {len(d)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
