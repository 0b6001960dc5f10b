"""Grouped routed experts (ql_moe_swiglu_grouped / ql_moe_down_grouped_accum_ordered) against
the oracle's per-token restatement of the reference ops (quant_swiglu_indexed_kernel,
kernel.cu:1339-1385; quant_down_f32_indexed_accum_ordered_kernel, kernel.cu:2252-2287), run
token by token as RoutedExperts.cpp:80-118 does.

The grouped path feeds the tensor cores exact integer quants and the activations as two f16 limbs
(hi + lo, exact to ~2^-22), and applies each block's scale (and Q4_K's min) in fp32, so it is
held to 1e-5 relative L2 against the oracle's exact decode (measured 1e-7 .. 6e-7), two orders
inside the north-star linear bound of 1e-3."""
import numpy as np
import pytest

import blog_b200 as Q
import oracle as O
from gpu_util import dev, host, make_weights, rel_l2

pytestmark = pytest.mark.gpu
FP32_CLASS = 1e-5


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


def _routes(seed, T, k, E):
    """k distinct experts per token (a top-k router's output)."""
    rng = np.random.default_rng(seed)
    return np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)


def _local(ids, e_begin, n):
    le = ids - e_begin
    return np.where((le >= 0) & (le < n), le, -1).astype(np.int32)


def grouped_swiglu(t, g, u, eb, rb, x, ids, e_begin, n, F, K):
    import torch
    T, k = ids.shape
    act = torch.full((T * k, F), float("nan"), device="cuda:0")
    gd, ud = dev(g), dev(u)
    Q.moe_swiglu_grouped(t, gd.data_ptr() + e_begin * eb, ud.data_ptr() + e_begin * eb, eb, eb, rb, rb,
                         dev(x).data_ptr(), K, dev(ids).data_ptr(), e_begin, n, act.data_ptr(), T, k, F, K)
    return host(act).reshape(T, k, F)


def oracle_swiglu(t, g, u, eb, rb, x, ids, e_begin, n, F, K):
    T, k = ids.shape
    lid = _local(ids, e_begin, n)
    gs, us = g[e_begin * (eb // rb):], u[e_begin * (eb // rb):]
    return np.stack([O.swiglu_indexed(t, gs, us, eb, eb, rb, rb, x[i], lid[i], k, F, K, order=1).reshape(k, F)
                     for i in range(T)])


def grouped_down(t, d, eb, rb, act, ids, e_begin, n, rw, out0, H, F):
    T, k = ids.shape
    out = dev(out0.copy())
    Q.moe_down_grouped_accum_ordered(t, dev(d).data_ptr() + e_begin * eb, eb, rb, dev(act).data_ptr(),
                                     dev(ids).data_ptr(), e_begin, n, dev(rw).data_ptr(), out.data_ptr(), H, T, k,
                                     H, F)
    return host(out)


def oracle_down(t, d, eb, rb, act, ids, e_begin, n, rw, out0, H, F):
    T, k = ids.shape
    lid = _local(ids, e_begin, n)
    ds = d[e_begin * (eb // rb):]
    a3 = act.reshape(T, k, F)
    return np.stack([O.down_indexed_ordered(t, ds, eb, rb, a3[i], lid[i], rw[i], out0[i], k, H, F, order=1)
                     for i in range(T)])


@pytest.mark.parametrize("e_begin,n", [(0, 16), (4, 8)])
def test_grouped_deepseek_shapes(e_begin, n):
    """DeepSeek-V2-Lite expert shapes (gate/up Q4_K 1408 x 2048, down Q5_0 2048 x 1408, top-6),
    64 tokens over 16 experts; (4, 8) holds experts 4..11 only, as one rank of expert parallelism."""
    E, F, H, T, k = 16, 1408, 2048, 64, 6
    tg, td = O.Q4_K, O.Q5_0
    g, u = make_weights(tg, E * F, H, seed=301), make_weights(tg, E * F, H, seed=302)
    d = make_weights(td, E * H, F, seed=303)
    rbg, rbd = O.row_bytes(tg, H), O.row_bytes(td, F)
    x = _x(304, T, H)
    ids = _routes(305, T, k, E)
    act = grouped_swiglu(tg, g, u, F * rbg, rbg, x, ids, e_begin, n, F, H)
    assert Q.last_launch_count() == 3  # activation prep + expert buckets + one grouped launch
    ref = oracle_swiglu(tg, g, u, F * rbg, rbg, x, ids, e_begin, n, F, H)
    skipped = _local(ids, e_begin, n) < 0
    assert np.all(act[skipped] == 0.0)
    err = rel_l2(act, ref)
    print(f"grouped SwiGLU (experts {e_begin}..{e_begin + n - 1}): rel_l2 {err:.2e}")
    assert err < FP32_CLASS
    rw = np.abs(_x(306, T, k)).astype(np.float32)
    out0 = _x(307, T, H)
    a2 = ref.reshape(T * k, F).astype(np.float32)
    got = grouped_down(td, d, H * rbd, rbd, a2, ids, e_begin, n, rw, out0, H, F)
    assert Q.last_launch_count() == 4  # activation prep + expert buckets + grouped launch + ordered combine
    want = oracle_down(td, d, H * rbd, rbd, a2, ids, e_begin, n, rw, out0, H, F)
    err = rel_l2(got - out0, want - out0)
    print(f"grouped down + ordered combine (experts {e_begin}..{e_begin + n - 1}): rel_l2 {err:.2e}")
    assert err < FP32_CLASS


@pytest.mark.parametrize("t", [O.Q4_0, O.Q5_0, O.Q8_0])
def test_grouped_formats_ragged(t):
    """32-element formats with rows on 2-byte boundaries (K = 288: 9 blocks), ragged row tiles
    (F = 296 gate/up rows, H = 200 down rows) and more tokens per expert than one pass (T 150,
    k 2 over 4 experts: ~75 per expert, three passes of 32)."""
    E, K, F, H, T, k = 4, 288, 296, 200, 150, 2
    g, u = make_weights(t, E * F, K, seed=311 + t), make_weights(t, E * F, K, seed=312 + t)
    rb = O.row_bytes(t, K)
    x = _x(313, T, K)
    ids = _routes(314, T, k, E)
    act = grouped_swiglu(t, g, u, F * rb, rb, x, ids, 0, E, F, K)
    ref = oracle_swiglu(t, g, u, F * rb, rb, x, ids, 0, E, F, K)
    print(f"type {t} grouped SwiGLU rel_l2 {rel_l2(act, ref):.2e}")
    assert rel_l2(act, ref) < FP32_CLASS
    d = make_weights(t, E * H, K, seed=315 + t)  # down with ffn_dim = K
    a2 = _x(316, T * k, K)
    rw = _x(317, T, k)
    out0 = np.zeros((T, H), np.float32)
    got = grouped_down(t, d, H * rb, rb, a2, ids, 0, E, rw, out0, H, K)
    want = oracle_down(t, d, H * rb, rb, a2, ids, 0, E, rw, out0, H, K)
    print(f"type {t} grouped down rel_l2 {rel_l2(got, want):.2e}")
    assert rel_l2(got, want) < FP32_CLASS


def test_grouped_long_rows_run_per_token():
    """Rows too long for the grouped kernel's shared-memory slabs (Q8_0, in_dim 4096: 4352 B) run
    the per-token indexed launches: same results as the oracle, one launch per token + id remap."""
    t, E, F, K, T, k = O.Q8_0, 4, 64, 4096, 5, 2
    g, u = make_weights(t, E * F, K, seed=321), make_weights(t, E * F, K, seed=322)
    rb = O.row_bytes(t, K)
    x = _x(323, T, K)
    ids = _routes(324, T, k, E)
    ids[1, 0] = 9  # an id outside this call's experts: skipped
    act = grouped_swiglu(t, g, u, F * rb, rb, x, ids, 0, E, F, K)
    assert Q.last_launch_count() == 1 + T
    ref = oracle_swiglu(t, g, u, F * rb, rb, x, ids, 0, E, F, K)
    assert np.all(act[1, 0] == 0.0)
    assert rel_l2(act, ref) < 1e-5  # the per-token engine decodes exactly in fp32
    H = 96
    d = make_weights(t, E * H, K, seed=325)
    a2 = _x(326, T * k, K)
    rw = _x(327, T, k)
    out0 = _x(328, T, H)
    got = grouped_down(t, d, H * rb, rb, a2, ids, 0, E, rw, out0, H, K)
    assert Q.last_launch_count() == 1 + T
    want = oracle_down(t, d, H * rb, rb, a2, ids, 0, E, rw, out0, H, K)
    assert rel_l2(got, want) < 1e-5


def test_grouped_no_routes_and_bad_args():
    """Every route outside this call's experts: act all zeros, out unchanged; bad sizes raise."""
    import torch
    t, E, F, K, T, k = O.Q4_K, 4, 64, 256, 8, 2
    g = make_weights(t, E * F, K, seed=331)
    rb = O.row_bytes(t, K)
    ids = np.full((T, k), 7, np.int32)
    act = grouped_swiglu(t, g, g, F * rb, rb, _x(332, T, K), ids, 0, E, F, K)
    assert np.all(act == 0.0)
    out0 = _x(333, T, 32)
    d = make_weights(t, E * 32, K, seed=334)
    got = grouped_down(t, d, 32 * rb, rb, _x(335, T * k, K), ids, 0, E, np.ones((T, k), np.float32), out0, 32, K)
    assert np.array_equal(got, out0)
    with pytest.raises(Q.QLError) as e:
        Q.moe_swiglu_grouped(O.Q6_K, dev(g).data_ptr(), dev(g).data_ptr(), 1, 1, 1, 1, 0, K, 0, 0, E, 0, T, k, F, K)
    assert e.value.status == Q.QL_EINVAL
    y = torch.empty(1, device="cuda:0")
    with pytest.raises(Q.QLError) as e:
        Q.moe_down_grouped_accum_ordered(t, dev(d).data_ptr(), 32 * rb, rb, y.data_ptr(), y.data_ptr(), 0, 0,
                                         y.data_ptr(), y.data_ptr(), 32, T, k, 32, K)
    assert e.value.status == Q.QL_EINVAL


@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_shards_sum_to_the_full_layer(world):
    """Expert parallelism as the bench runs it, on one GPU: rank r holds experts [r E / W, (r + 1) E / W)
    (its packed weights and its expert range), computes the routed SwiGLU and down + ordered combine
    for all tokens, and the ranks' outputs are summed (the all-reduce).  The sum matches the one-call
    result over all experts (float reassociation of the per-token route sums only) and the oracle."""
    E, F, H, T, k = 16, 1408, 2048, 64, 6
    tg, td = O.Q4_K, O.Q5_0
    g, u = make_weights(tg, E * F, H, seed=341), make_weights(tg, E * F, H, seed=342)
    d = make_weights(td, E * H, F, seed=343)
    rbg, rbd = O.row_bytes(tg, H), O.row_bytes(td, F)
    x = _x(344, T, H)
    ids = _routes(345, T, k, E)
    rw = np.abs(_x(346, T, k)).astype(np.float32)
    zero = np.zeros((T, H), np.float32)
    full_act = grouped_swiglu(tg, g, u, F * rbg, rbg, x, ids, 0, E, F, H).reshape(T * k, F)
    full = grouped_down(td, d, H * rbd, rbd, full_act, ids, 0, E, rw, zero, H, F)
    total = np.zeros((T, H), np.float64)
    for r in range(world):
        e0, e1 = r * E // world, (r + 1) * E // world
        act = grouped_swiglu(tg, g, u, F * rbg, rbg, x, ids, e0, e1 - e0, F, H).reshape(T * k, F)
        total += grouped_down(td, d, H * rbd, rbd, act, ids, e0, e1 - e0, rw, zero, H, F)
    err = rel_l2(total, full)
    print(f"EP{world} shards summed vs one call over all experts: rel_l2 {err:.2e}")
    assert err < 1e-6
    want = oracle_down(td, d, H * rbd, rbd, oracle_swiglu(tg, g, u, F * rbg, rbg, x, ids, 0, E, F, H)
                       .reshape(T * k, F).astype(np.float32), ids, 0, E, rw, zero, H, F)
    assert rel_l2(total, want) < FP32_CLASS
