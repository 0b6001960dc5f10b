"""The CPU oracle pinned against golden vectors (CPU only).

Sources: the reference's own known-answer kernel tests (LaunchAddTest.cpp,
rebuilt in tests/golden/make_golden.py) and gguf-py 0.19.0 vectors.
"""
import numpy as np
import pytest

import oracle as O

TYPES = {"Q8_0": O.Q8_0, "Q4_0": O.Q4_0, "Q5_0": O.Q5_0, "Q4_K": O.Q4_K, "Q6_K": O.Q6_K}


def test_f16_roundtrip_all_bits():
    bits = np.arange(65536, dtype=np.uint16)
    finite = np.isfinite(bits.view(np.float16))
    lib = O.lib()
    dec = np.array([lib.orc_f16_to_f32(int(b)) for b in bits[::97]], np.float32)
    ref = bits[::97].view(np.float16).astype(np.float32)
    m = finite[::97]
    assert np.array_equal(dec[m].view(np.uint32), ref[m].view(np.uint32))
    # encode: RNE, equal to numpy's float32 -> float16 cast on random and edge values
    vals = np.concatenate([O.randn(5, 4000, 3.0), O.randn(6, 2000, 1e-5), O.randn(7, 1000, 3e4),
                           np.array([65504, 65519.99, 65520, 2**-25, 2**-24, 1.5 * 2**-25, 0.0, -0.0], np.float32)])
    enc = np.array([lib.orc_f32_to_f16(float(v)) for v in vals], np.uint16)
    assert np.array_equal(enc, vals.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("name", list(TYPES))
def test_dequant_matches_gguf_py(golden, name):
    t = TYPES[name]
    raw = golden[f"gg_{name}_bytes"]
    exp = golden[f"gg_{name}_deq"]
    be, bb = O.BLOCK[t]
    got = O.dequant_rows(t, raw.reshape(-1), be * raw.shape[0], rb=bb * raw.shape[0]).reshape(exp.shape)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32)), name


@pytest.mark.parametrize("name", ["Q8_0", "Q4_0", "Q5_0"])
def test_quantizer_matches_gguf_py(golden, name):
    t = TYPES[name]
    src = golden[f"gg_{name}_src"]
    exp = golden[f"gg_{name}_quant"]
    got = O.quantize(t, src)
    assert np.array_equal(got.reshape(-1), exp.reshape(-1)), name


def test_q4k_quantizer_roundtrip():
    x = O.randn(11, 64 * 256, 0.02).reshape(64, 256)
    q = O.quantize(O.Q4_K, x)
    d = O.dequant_rows(O.Q4_K, q, 256)
    # 4-bit affine per 32 elements: error bounded by half a step of each sub-block
    step = (x.reshape(64, 8, 32).max(-1) - np.minimum(x.reshape(64, 8, 32).min(-1), 0)) / 15
    err = np.abs(d - x).reshape(64, 8, 32).max(-1)
    assert np.all(err <= step * 0.75 + 2e-3)


def test_known_answer_q80_matmul(golden):
    w, x, y = golden["ka_q80_w"], golden["ka_q80_x"], golden["ka_q80_y"]
    got = O.gemv(O.Q8_0, w, 34, x, 2, 32, 3)
    np.testing.assert_allclose(got, y, atol=1e-5)


def test_known_answer_q4k_scale_min(golden):
    w, x = golden["ka_q4k_w"], golden["ka_q4k_x"]
    deq = O.dequant_rows(O.Q4_K, w, 256)
    assert np.array_equal(deq[0], golden["ka_q4k_deq"])
    got = O.gemv(O.Q4_K, w, 144, x, 1, 256, 1)
    assert got[0, 0] == golden["ka_q4k_y"][0]  # 14 * 158 exactly


def test_known_answer_q6k_scale_groups(golden):
    w, x = golden["ka_q6k_w"], golden["ka_q6k_x"]
    deq = O.dequant_rows(O.Q6_K, w, 256)
    assert np.array_equal(deq[0], golden["ka_q6k_deq"])
    got = O.gemv(O.Q6_K, w, 210, x, 1, 256, 1)
    assert got[0, 0] == golden["ka_q6k_y"][0]  # 6 * 158 exactly


@pytest.mark.parametrize("name,t", [("q80", O.Q8_0), ("q4k", O.Q4_K), ("q6k", O.Q6_K)])
def test_known_answer_moe_down(golden, name, t):
    w = golden[f"ka_down_{name}_w"]
    act, rw, ids = golden[f"ka_down_{name}_act"], golden[f"ka_down_{name}_rw"], golden[f"ka_down_{name}_ids"]
    ffn, rb = (int(v) for v in golden[f"ka_down_{name}_ffn"])
    hidden = 9
    out = O.down_indexed_ordered(t, w, hidden * rb, rb, act, ids, rw, np.zeros(hidden, np.float32), 2, hidden, ffn)
    np.testing.assert_allclose(out, golden[f"ka_down_{name}_y"], rtol=1e-5, atol=1e-4)


def test_known_answer_swiglu_indexed(golden):
    g, u, x, ids = (golden[f"ka_swiglu_q4k_{s}"] for s in ("g", "u", "x", "ids"))
    act = O.swiglu_indexed(O.Q4_K, g, u, 7 * 144, 7 * 144, 144, 144, x, ids, 2, 7, 256)
    np.testing.assert_allclose(act, golden["ka_swiglu_q4k_y"], rtol=1e-5, atol=1e-5)


def test_dequant_f16_is_rne_of_f32():
    for t in (O.Q8_0, O.Q4_0, O.Q5_0, O.Q4_K):
        x = O.randn(3, 4 * 256, 0.05).reshape(4, 256)
        q = O.quantize(t, x)
        f32 = O.dequant_rows(t, q, 256).reshape(-1)
        f16 = O.dequant_f16(t, q.reshape(-1), f32.size)
        assert np.array_equal(f16, f32.astype(np.float16).view(np.uint16))


def test_lane_order_matches_f64_to_tolerance():
    rng = np.random.default_rng(0)
    for t in (O.Q8_0, O.Q4_0, O.Q4_K, O.Q5_0):
        w = O.quantize(t, O.randn(1, 64 * 512, 0.02).reshape(64, 512))
        x = rng.standard_normal((2, 512)).astype(np.float32)
        a = O.gemv(t, w, O.row_bytes(t, 512), x, 64, 512, 2, order=0)
        b = O.gemv(t, w, O.row_bytes(t, 512), x, 64, 512, 2, order=1)
        assert np.linalg.norm(a - b) / np.linalg.norm(b) < 1e-6


def test_router_topk_semantics():
    # ties pick the lowest expert id; non-finite logits are never preferred
    lg = np.zeros((3, 8), np.float32)
    lg[0] = [1, 3, 3, 2, -1, 0, 3, 1]
    lg[1] = [np.nan, 5, np.inf, -np.inf, 4, 4, 0, 0]
    lg[2] = [np.nan] * 8
    idx, w = O.router_topk(lg, 3, 1.0)
    assert idx[0].tolist() == [1, 2, 6]
    assert idx[1].tolist() == [1, 4, 5]
    assert idx[2].tolist() == [0, 1, 2] and np.all(w[2] == 0)
    p = np.exp(lg[0] - lg[0].max()); p /= p.sum()
    np.testing.assert_allclose(w[0], p[[1, 2, 6]], rtol=1e-6)


def test_argmax_lowest_index_on_ties():
    v = np.array([0, 5, 1, 5, np.nan, 5], np.float32)
    assert O.argmax(v) == 1
