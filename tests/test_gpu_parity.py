"""Parity of the B200 kernels (called through the C ABI) with the CPU oracle.

Bars: dequantized values, routing indices, embeddings and argmax are
bit-exact; linear outputs are within 1e-5 relative L2 of the oracle's
double-precision accumulation (the north-star bound is 1e-3; the kernels
accumulate in fp32).
"""
import numpy as np
import pytest

import blog_b200 as Q
import oracle as O
from gpu_util import dev, host, make_weights, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-5


@pytest.fixture(scope="module", autouse=True)
def _stream():
    import torch
    torch.cuda.init()
    Q.init(0)
    Q.set_stream(torch.cuda.current_stream().cuda_stream)
    yield
    Q.check_device()


def _x(seed, m, k):
    return np.random.default_rng(seed).standard_normal((m, k)).astype(np.float32)


# ---- dequant: bit-exact ------------------------------------------------------
@pytest.mark.parametrize("name", ["Q8_0", "Q4_0", "Q5_0", "Q4_K", "Q6_K"])
def test_dequant_f16_bit_exact_on_gguf_vectors(golden, name):
    import torch
    t = {"Q8_0": O.Q8_0, "Q4_0": O.Q4_0, "Q5_0": O.Q5_0, "Q4_K": O.Q4_K, "Q6_K": O.Q6_K}[name]
    raw = golden[f"gg_{name}_bytes"]
    n = raw.shape[0] * O.BLOCK[t][0]
    out = torch.empty(n, dtype=torch.int16, device="cuda:0")
    Q.dequantize_to_f16(t, dev(raw).data_ptr(), out.data_ptr(), n)
    got = host(out).view(np.uint16)
    assert np.array_equal(got, O.dequant_f16(t, raw.reshape(-1), n))
    # and the f16 values are the gguf-py float32 values rounded once
    assert np.array_equal(got, golden[f"gg_{name}_deq"].reshape(-1).astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("t", [O.Q8_0, O.Q4_0, O.Q5_0, O.Q4_K, O.Q6_K])
def test_dequant_f16_bit_exact_random(t):
    import torch
    w = make_weights(t, 64, 1024, seed=t + 100)
    n = 64 * 1024
    out = torch.empty(n, dtype=torch.int16, device="cuda:0")
    Q.dequantize_to_f16(t, dev(w).data_ptr(), out.data_ptr(), n)
    assert np.array_equal(host(out).view(np.uint16), O.dequant_f16(t, w.reshape(-1), n))


# ---- GEMV / matmul -------------------------------------------------------------
SHAPES = [
    (O.Q4_K, 64, 256, 1), (O.Q4_K, 4096, 4096, 1), (O.Q4_K, 3584, 18944, 1), (O.Q4_K, 4096, 4096, 4),
    (O.Q4_K, 100, 512, 3), (O.Q4_K, 1, 256, 1), (O.Q4_K, 18944, 3584, 2),
    (O.Q8_0, 896, 896, 1), (O.Q8_0, 4864, 896, 1), (O.Q8_0, 37, 4864, 2), (O.Q8_0, 2, 32, 3), (O.Q8_0, 4096, 4096, 4),
    (O.Q4_0, 4096, 4096, 1), (O.Q4_0, 1024, 29568, 1), (O.Q4_0, 33, 8192, 2), (O.Q4_0, 11008, 4096, 1),
    (O.Q5_0, 2048, 1408, 1), (O.Q5_0, 64, 10944, 2), (O.Q5_0, 70, 96, 1),
    # rows a multiple of 16 bytes: tensor-map staging of the 32-element formats (stages that start
    # mid 16-byte chunk, ragged last row group, 72B-shape q projection)
    (O.Q5_0, 256, 4096, 1), (O.Q5_0, 100, 2048, 3), (O.Q8_0, 4096, 4096, 1), (O.Q4_0, 8192, 8192, 1),
    (O.Q4_0, 4640, 4096, 2),
    # rows a multiple of 8 (not 16) bytes: row pairs staged as one super-row (72B down projection,
    # 0.5B's K = 896 projections and LM head rows)
    (O.Q4_0, 8192, 29568, 1), (O.Q8_0, 4864, 896, 3), (O.Q8_0, 151936, 896, 1), (O.Q8_0, 64, 1792, 2),
    (O.Q6_K, 64, 2048, 1), (O.Q6_K, 300, 512, 2),
]


@pytest.mark.parametrize("t,n,k,m", SHAPES)
def test_gemv_matches_oracle(t, n, k, m):
    import torch
    w = make_weights(t, n, k, seed=n * 7 + k)
    x = _x(n + k + m, m, k)
    y = torch.full((m, n), float("nan"), device="cuda:0")
    rb = O.row_bytes(t, k)
    Q.quant_gemv(t, dev(w).data_ptr(), rb, dev(x).data_ptr(), y.data_ptr(), n, k, m)
    ref = O.gemv(t, w, rb, x, n, k, m, order=1)
    got = host(y)
    assert np.isfinite(got).all()
    assert rel_l2(got, ref) < TOL


@pytest.mark.parametrize("t", [O.Q4_K, O.Q8_0])
def test_matmul_many_tokens(t):
    import torch
    n, k, m = 512, 2048, 7
    w = make_weights(t, n, k, seed=3)
    x = _x(4, m, k)
    y = torch.empty((m, n), device="cuda:0")
    rb = O.row_bytes(t, k)
    Q.quant_matmul(t, dev(w).data_ptr(), rb, dev(x).data_ptr(), y.data_ptr(), n, k, m)
    assert rel_l2(host(y), O.gemv(t, w, rb, x, n, k, m, order=1)) < TOL


def test_repeated_calls_are_deterministic():
    import torch
    t, n, k = O.Q4_K, 3584, 18944  # stream-K splits every row group over several CTAs
    w = dev(make_weights(t, n, k, seed=9))
    x = dev(_x(10, 1, k))
    ys = []
    for _ in range(3):
        y = torch.empty(n, device="cuda:0")
        Q.quant_gemv(t, w.data_ptr(), O.row_bytes(t, k), x.data_ptr(), y.data_ptr(), n, k, 1)
        ys.append(host(y))
    assert np.array_equal(ys[0].view(np.uint32), ys[1].view(np.uint32))
    assert np.array_equal(ys[0].view(np.uint32), ys[2].view(np.uint32))


@pytest.mark.parametrize("t,n,k", [(O.Q4_K, 2048, 2816), (O.Q8_0, 896, 4864), (O.Q5_0, 2048, 1408)])
def test_gemv_add(t, n, k):
    import torch
    w = make_weights(t, n, k, seed=11)
    x = _x(12, 1, k)
    y0 = _x(13, 1, n)[0]
    y = dev(y0.copy())
    rb = O.row_bytes(t, k)
    Q.quant_gemv_add(t, dev(w).data_ptr(), rb, dev(x).data_ptr(), y.data_ptr(), n, k)
    ref = y0 + O.gemv(t, w, rb, x, n, k, 1, order=1)[0]
    assert rel_l2(host(y), ref) < TOL


@pytest.mark.parametrize("t,f,k,m", [(O.Q4_K, 2816, 2048, 1), (O.Q4_K, 18944, 3584, 1), (O.Q8_0, 4864, 896, 2),
                                     (O.Q4_0, 1000, 1024, 3), (O.Q4_0, 2048, 4096, 1), (O.Q8_0, 1024, 4096, 2)])
def test_swiglu(t, f, k, m):
    import torch
    g = make_weights(t, f, k, seed=21)
    u = make_weights(t, f, k, seed=22)
    x = _x(23, m, k)
    act = torch.empty((m, f), device="cuda:0")
    rb = O.row_bytes(t, k)
    if m == 1:
        Q.quant_swiglu(t, dev(g).data_ptr(), dev(u).data_ptr(), rb, rb, dev(x).data_ptr(), act.data_ptr(), f, k)
    else:
        Q.quant_swiglu_ex(t, dev(g).data_ptr(), dev(u).data_ptr(), rb, rb, dev(x).data_ptr(), k, act.data_ptr(), f, f,
                          k, m)
    gv = O.gemv(t, g, rb, x, f, k, m, order=1).astype(np.float64)
    uv = O.gemv(t, u, rb, x, f, k, m, order=1).astype(np.float64)
    ref = gv / (1.0 + np.exp(-gv)) * uv
    assert rel_l2(host(act), ref) < TOL


def test_gemv_ex_fused_rmsnorm_bias_accumulate():
    import torch
    t, n, k, m, eps = O.Q4_K, 512, 3584, 2, 1e-6
    w = make_weights(t, n, k, seed=31)
    x = _x(32, m, k) * 3.0
    gamma = (1.0 + 0.1 * _x(33, 1, k)[0]).astype(np.float32)
    bias = _x(34, 1, n)[0]
    y0 = _x(35, m, n)
    y = dev(y0.copy())
    rb = O.row_bytes(t, k)
    Q.quant_gemv_ex(t, dev(w).data_ptr(), rb, dev(x).data_ptr(), k, y.data_ptr(), n, n, k, m, dev(gamma).data_ptr(),
                    eps, dev(bias).data_ptr(), accumulate=True)
    xn = O.rmsnorm(x, gamma, eps)
    ref = y0 + O.gemv(t, w, rb, xn, n, k, m, order=1) + bias[None, :]
    assert rel_l2(host(y), ref) < TOL


@pytest.mark.parametrize("t,rows,k", [(O.Q4_K, (3584, 512, 512), 3584), (O.Q8_0, (896, 128, 128), 896),
                                      (O.Q4_K, (64, 50), 2048), (O.Q5_0, (32, 32, 7), 1408),
                                      (O.Q4_0, (1024, 128, 128), 4096)])
def test_stacked_qkv_matches_separate(t, rows, k):
    """Fused q/k/v (stacked sources) with RMSNorm and bias equals the separate projections."""
    import torch
    m, eps = 2, 1e-6
    ws = [make_weights(t, n, k, seed=200 + i) for i, n in enumerate(rows)]
    x = _x(210, m, k)
    gamma = (1.0 + 0.1 * _x(211, 1, k)[0]).astype(np.float32)
    total = sum(rows)
    bias = _x(212, 1, total)[0]
    y = torch.full((m, total), float("nan"), device="cuda:0")
    rb = O.row_bytes(t, k)
    Q.quant_gemv_stacked_ex(t, [dev(w).data_ptr() for w in ws], [rb] * len(ws), list(rows), dev(x).data_ptr(), k,
                            y.data_ptr(), total, k, m, dev(gamma).data_ptr(), eps, dev(bias).data_ptr())
    xn = O.rmsnorm(x, gamma, eps)
    ref = np.concatenate([O.gemv(t, w, rb, xn, n, k, m, order=1) for w, n in zip(ws, rows)], axis=1) + bias[None, :]
    assert rel_l2(host(y), ref) < TOL


def test_lm_head_full_size_row_subset():
    """151936 x 4096 Q4_K (350 MB): every output row computed, 512 checked."""
    import torch
    t, n, k = O.Q4_K, 151936, 4096
    rb = O.row_bytes(t, k)
    w = torch.empty((n, rb), dtype=torch.uint8, device="cuda:0")
    Q.synth_quantized(t, 77, n, k, 0.02, w.data_ptr())
    x = _x(78, 1, k)
    y = torch.empty(n, device="cuda:0")
    Q.quant_gemv(t, w.data_ptr(), rb, dev(x).data_ptr(), y.data_ptr(), n, k, 1)
    rows = np.sort(np.random.default_rng(79).choice(n, 512, replace=False))
    wsub = host(w[torch.from_numpy(rows).to("cuda:0")])
    ref = O.gemv(t, wsub, rb, x, len(rows), k, 1, order=1)[0]
    assert rel_l2(host(y)[rows], ref) < TOL


# ---- MoE -------------------------------------------------------------------------
def test_swiglu_indexed_with_skipped_route():
    import torch
    t, E, F, K, k = O.Q4_K, 8, 1408, 2048, 6
    g = make_weights(t, E * F, K, seed=41)
    u = make_weights(t, E * F, K, seed=42)
    x = _x(43, 1, K)[0]
    ids = np.array([3, 7, -1, 0, 5, 3], np.int32)
    rb = O.row_bytes(t, K)
    eb = F * rb
    act = torch.full((k, F), float("nan"), device="cuda:0")
    Q.quant_swiglu_indexed(t, dev(g).data_ptr(), dev(u).data_ptr(), eb, eb, rb, rb, dev(x).data_ptr(),
                           dev(ids).data_ptr(), act.data_ptr(), k, F, K)
    ref = O.swiglu_indexed(t, g, u, eb, eb, rb, rb, x, ids, k, F, K, order=1)
    got = host(act)
    assert np.all(got[2] == 0.0)
    assert rel_l2(got, ref) < TOL


@pytest.mark.parametrize("t", [O.Q5_0, O.Q8_0, O.Q4_0])
def test_down_ordered_with_skipped_route(t):
    import torch
    E, H, F, k = 8, 2048, 1408, 6
    d = make_weights(t, E * H, F, seed=51 + t)
    act = _x(52, k, F)
    ids = np.array([2, -1, 6, 1, 7, 2], np.int32)
    rw = np.abs(_x(53, 1, k)[0]).astype(np.float32)
    out0 = _x(54, 1, H)[0]
    rb = O.row_bytes(t, F)
    eb = H * rb
    out = dev(out0.copy())
    Q.quant_down_f32_indexed_accum_ordered(t, dev(d).data_ptr(), eb, rb, dev(act).data_ptr(), dev(ids).data_ptr(),
                                           dev(rw).data_ptr(), out.data_ptr(), k, H, F)
    ref = O.down_indexed_ordered(t, d, eb, rb, act, ids, rw, out0, k, H, F, order=1)
    assert rel_l2(host(out), ref) < TOL


def test_down_ordered_q4k():
    import torch
    t, E, H, F, k = O.Q4_K, 4, 512, 2048, 3
    d = make_weights(t, E * H, F, seed=61)
    act = _x(62, k, F)
    ids = np.array([3, 0, 2], np.int32)
    rw = np.array([0.5, -0.25, 0.125], np.float32)
    rb = O.row_bytes(t, F)
    out = dev(np.zeros(H, np.float32))
    Q.quant_down_f32_indexed_accum_ordered(t, dev(d).data_ptr(), H * rb, rb, dev(act).data_ptr(), dev(ids).data_ptr(),
                                           dev(rw).data_ptr(), out.data_ptr(), k, H, F)
    ref = O.down_indexed_ordered(t, d, H * rb, rb, act, ids, rw, np.zeros(H, np.float32), k, H, F, order=1)
    assert rel_l2(host(out), ref) < TOL


def _router_logits():
    rng = np.random.default_rng(71)
    lg = rng.standard_normal((64, 64)).astype(np.float32)
    lg[1, :] = 0.5                      # all tied
    lg[2, [5, 9, 40]] = 9.0             # ties at the top
    lg[3, :] = np.nan                   # nothing finite
    lg[4, ::2] = -np.inf
    lg[5, 10] = np.inf                  # +inf is non-finite -> treated as -inf
    lg[6, :60] = np.nan                 # fewer finite logits than k
    return lg


@pytest.mark.parametrize("E,k", [(64, 6), (8, 2), (40, 8)])
def test_router_topk_matches_oracle(E, k):
    import torch
    lg = np.ascontiguousarray(_router_logits()[:, :E])
    T = lg.shape[0]
    idx = torch.empty((T, k), dtype=torch.int32, device="cuda:0")
    w = torch.empty((T, k), device="cuda:0")
    Q.moe_router_topk(dev(lg).data_ptr(), idx.data_ptr(), w.data_ptr(), T, E, k, 1.0)
    ri, rw = O.router_topk(lg, k, 1.0)
    assert np.array_equal(host(idx), ri)
    np.testing.assert_allclose(host(w), rw, rtol=2e-6, atol=1e-7)


def test_embedding_bit_exact():
    import torch
    for t in (O.Q4_K, O.Q8_0, O.Q6_K, O.Q5_0, O.Q4_0):
        V, H = 1000, 512
        tab = make_weights(t, V, H, seed=81 + t)
        ids = np.array([0, 999, 5, 5, 512], np.int32)
        out = torch.empty((len(ids), H), device="cuda:0")
        Q.quant_embedding(t, dev(ids).data_ptr(), out.data_ptr(), dev(tab).data_ptr(), O.row_bytes(t, H), H, len(ids))
        ref = O.embedding(t, ids, tab, O.row_bytes(t, H), H)
        assert np.array_equal(host(out).view(np.uint32), ref.view(np.uint32)), t


@pytest.mark.parametrize("n", [1, 1000, 151936, 152064])
def test_argmax(n):
    import torch
    v = _x(91, 1, n)[0]
    if n > 10:
        v[[7, n // 2, n - 3]] = v.max() + 1.0  # ties: lowest index wins
        v[3] = np.nan
    out = torch.empty(1, dtype=torch.int32, device="cuda:0")
    Q.argmax(dev(v).data_ptr(), n, out.data_ptr())
    assert int(host(out)[0]) == O.argmax(v)


# ---- the reference's known-answer blocks, through the C ABI --------------------
def test_known_answers_through_capi(golden):
    import torch
    y = torch.empty((3, 2), device="cuda:0")
    Q.quant_matmul(O.Q8_0, dev(golden["ka_q80_w"]).data_ptr(), 34, dev(golden["ka_q80_x"]).data_ptr(), y.data_ptr(),
                   2, 32, 3)
    np.testing.assert_allclose(host(y), golden["ka_q80_y"], atol=1e-5)
    for name, t, rb in (("q4k", O.Q4_K, 144), ("q6k", O.Q6_K, 210)):
        y1 = torch.empty(1, device="cuda:0")
        Q.quant_gemv(t, dev(golden[f"ka_{name}_w"]).data_ptr(), rb, dev(golden[f"ka_{name}_x"]).data_ptr(),
                     y1.data_ptr(), 1, 256, 1)
        assert float(host(y1)[0]) == float(golden[f"ka_{name}_y"][0])
    for name, t in (("q80", O.Q8_0), ("q4k", O.Q4_K), ("q6k", O.Q6_K)):
        ffn, rb = (int(v) for v in golden[f"ka_down_{name}_ffn"])
        out = dev(np.zeros(9, np.float32))
        Q.quant_down_f32_indexed_accum_ordered(t, dev(golden[f"ka_down_{name}_w"]).data_ptr(), 9 * rb, rb,
                                               dev(golden[f"ka_down_{name}_act"]).data_ptr(),
                                               dev(golden[f"ka_down_{name}_ids"]).data_ptr(),
                                               dev(golden[f"ka_down_{name}_rw"]).data_ptr(), out.data_ptr(), 2, 9, ffn)
        np.testing.assert_allclose(host(out), golden[f"ka_down_{name}_y"], rtol=1e-5, atol=1e-4)
    act = torch.empty((2, 7), device="cuda:0")
    Q.quant_swiglu_indexed(O.Q4_K, dev(golden["ka_swiglu_q4k_g"]).data_ptr(), dev(golden["ka_swiglu_q4k_u"]).data_ptr(),
                           7 * 144, 7 * 144, 144, 144, dev(golden["ka_swiglu_q4k_x"]).data_ptr(),
                           dev(golden["ka_swiglu_q4k_ids"]).data_ptr(), act.data_ptr(), 2, 7, 256)
    np.testing.assert_allclose(host(act), golden["ka_swiglu_q4k_y"], rtol=1e-5, atol=1e-5)


def test_device_error_word_clean():
    Q.check_device()


# ---- fused LM head + greedy argmax ---------------------------------------------------
def _key_index(keys):
    keys = np.asarray(keys, np.uint64)
    return np.where(keys == 0, 0, (np.uint64(0xFFFFFFFF) - (keys & np.uint64(0xFFFFFFFF)))).astype(np.int64)


@pytest.mark.parametrize("m", [1, 3, 16])  # GEMV engine (1, 3) and tensor-core path (16)
def test_lm_head_argmax_matches_logits(m):
    import torch
    t, n, k, eps = O.Q4_K, 30000, 1024, 1e-6
    w = make_weights(t, n, k, seed=201)
    x = _x(202, m, k)
    gamma = (1.0 + 0.1 * _x(203, 1, k)[0]).astype(np.float32)
    rb = O.row_bytes(t, k)
    logits = torch.empty((m, n), device="cuda:0")
    idx = torch.full((m,), -1, dtype=torch.int32, device="cuda:0")
    key = torch.zeros((m,), dtype=torch.int64, device="cuda:0")
    for _ in range(2):  # the second launch checks that the keys were reset
        Q.quant_gemv_argmax_ex(t, dev(w).data_ptr(), rb, dev(x).data_ptr(), k, logits.data_ptr(), n, n, k, m,
                               dev(gamma).data_ptr(), eps, 0, idx.data_ptr(), key.data_ptr())
        lg = host(logits)
        want = np.argmax(lg, axis=1)  # first occurrence = lowest index on ties
        assert np.array_equal(host(idx), want)
        assert np.array_equal(_key_index(host(key).view(np.uint64)), want)


def test_lm_head_argmax_vocabulary_shards_combine():
    import torch
    t, n, k, m = O.Q4_K, 20000, 512, 2
    w = make_weights(t, n, k, seed=211)
    x = _x(212, m, k)
    rb = O.row_bytes(t, k)
    full_idx = torch.empty((m,), dtype=torch.int32, device="cuda:0")
    Q.quant_gemv_argmax_ex(t, dev(w).data_ptr(), rb, dev(x).data_ptr(), k, None, 0, n, k, m, None, 0.0, 0,
                           full_idx.data_ptr(), None)
    keys = []
    for lo, hi in ((0, 9984), (9984, n)):  # two vocabulary shards, 32-row aligned
        kk = torch.zeros((m,), dtype=torch.int64, device="cuda:0")
        Q.quant_gemv_argmax_ex(t, dev(np.ascontiguousarray(w[lo:hi])).data_ptr(), rb, dev(x).data_ptr(), k, None, 0,
                               hi - lo, k, m, None, 0.0, lo, None, kk.data_ptr())
        keys.append(host(kk).view(np.uint64))
    comb = np.maximum(keys[0], keys[1])
    assert np.array_equal(_key_index(comb), host(full_idx))


@pytest.mark.parametrize("m", [1, 16])
def test_lm_head_argmax_nan_rows_select_zero(m):
    import torch
    t, n, k = O.Q4_K, 4096, 512
    w = make_weights(t, n, k, seed=221)
    x = _x(222, m, k)
    x[0, :] = np.nan
    rb = O.row_bytes(t, k)
    idx = torch.full((m,), -1, dtype=torch.int32, device="cuda:0")
    logits = torch.empty((m, n), device="cuda:0")
    Q.quant_gemv_argmax_ex(t, dev(w).data_ptr(), rb, dev(x).data_ptr(), k, logits.data_ptr(), n, n, k, m, None, 0.0,
                           0, idx.data_ptr(), None)
    got = host(idx)
    assert got[0] == 0
    assert np.array_equal(got[1:], np.argmax(host(logits)[1:], axis=1))
