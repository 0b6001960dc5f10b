"""Parity of the tcgen05 prefill GEMM (Q4_K, Q4_0 and Q8_0, called through the C ABI).

The tensor-core path rounds each activation row (after an exact power-of-two
scale) and each dequantized weight to f16 and accumulates in fp32 on the tensor
cores.  Two bars:
  * against the CPU oracle's double-precision result on the exact weights:
    within the north-star linear bound, 1e-3 relative L2 (measured ~2e-4);
  * against a float64 evaluation of the same f16 operands (weights rounded as
    f16(n * f16(d*sc) - f16(dmin*m)), activations as f16(x * 2^k)): within
    1e-5, i.e. the kernel adds nothing beyond fp32 accumulation order.
"""
import numpy as np
import pytest

import blog_b200 as Q
import oracle as O
from gpu_util import dev, host, make_weights, rel_l2

pytestmark = pytest.mark.gpu
NORTH_STAR = 1e-3
EXACT_F16_OPERANDS = 1e-5


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


def q4k_f16_operand(w, n, k):
    """The weights exactly as the tensor-core dequantizer rounds them (float64 array [n, k])."""
    b = w.reshape(n, k // 256, 144)
    d = b[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float64)
    dmin = b[..., 2:4].copy().view(np.float16)[..., 0].astype(np.float64)
    s = b[..., 4:16].astype(np.int64)
    qs = b[..., 16:144].astype(np.int64)
    out = np.empty((n, k // 256, 256), np.float64)
    for j in range(8):  # q4k_scale_min (reference kernel.cu:913-921)
        if j < 4:
            sc, mn = s[..., j] & 63, s[..., j + 4] & 63
        else:
            sc = (s[..., j + 4] & 0xF) | ((s[..., j - 4] >> 6) << 4)
            mn = (s[..., j + 4] >> 4) | ((s[..., j] >> 6) << 4)
        D = (d * sc).astype(np.float16).astype(np.float64)
        M = (dmin * mn).astype(np.float16).astype(np.float64)
        p = j // 2
        nib = (qs[..., 32 * p:32 * p + 32] >> (4 * (j & 1))) & 0xF
        out[..., 32 * j:32 * j + 32] = (nib * D[..., None] - M[..., None]).astype(np.float16)
    return out.reshape(n, k)


def q40_f16_operand(w, n, k):
    """Q4_0 weights as the tensor-core dequantizer rounds them: f16(d * (q - 8)), one rounding."""
    b = w.reshape(n, k // 32, 18)
    d = b[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float64)
    qs = b[..., 2:18].astype(np.int64)
    q = np.concatenate([qs & 0xF, qs >> 4], axis=-1)  # elements 0..15 low nibbles, 16..31 high
    return (d[..., None] * (q - 8)).astype(np.float16).astype(np.float64).reshape(n, k)


def q80_f16_operand(w, n, k):
    """Q8_0 weights as the tensor-core dequantizer rounds them: f16(d * q), one rounding."""
    b = w.reshape(n, k // 32, 34)
    d = b[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float64)
    q = b[..., 2:34].copy().view(np.int8).astype(np.float64)
    return (d[..., None] * q).astype(np.float16).astype(np.float64).reshape(n, k)


def f16_operand(t, w, n, k):
    if t == O.Q8_0:
        return q80_f16_operand(w, n, k)
    return q40_f16_operand(w, n, k) if t == O.Q4_0 else q4k_f16_operand(w, n, k)


def act_f16_operand(x, gamma=None, eps=0.0):
    """Activations as the tensor-core path sees them: f16(x * g * 2^k) * 2^-k (* RMSNorm factor)."""
    xg = x.astype(np.float64) * (gamma.astype(np.float64)[None, :] if gamma is not None else 1.0)
    xg = xg.astype(np.float32)
    out = np.empty_like(xg, dtype=np.float64)
    for r in range(x.shape[0]):
        mx = float(np.max(np.abs(xg[r]))) if xg.shape[1] else 0.0
        kk = 0
        if mx > 0 and np.isfinite(mx):
            kk = min(14 - int(np.frexp(np.float32(mx))[1]), 126)
        s = np.float32(2.0 ** kk)
        out[r] = (xg[r] * s).astype(np.float16).astype(np.float64) / float(s)
        if gamma is not None:
            ms = np.float32(np.sum(x[r].astype(np.float64) ** 2) / x.shape[1])
            out[r] *= 1.0 / np.sqrt(np.float64(ms) + eps)
    return out


def run_tc(w, rb, x, n, k, m, gamma=None, eps=0.0, bias=None, y0=None, path=Q.PATH_TENSOR, t=O.Q4_K):
    import torch
    y = dev(y0.copy()) if y0 is not None else torch.full((m, n), float("nan"), device="cuda:0")
    Q.quant_matmul_ex(t, dev(w).data_ptr(), rb, dev(x).data_ptr(), k, y.data_ptr(), n, n, k, m,
                      dev(gamma).data_ptr() if gamma is not None else None, eps,
                      dev(bias).data_ptr() if bias is not None else None, y0 is not None, path)
    return host(y)


# (n, k, m): one tile; ragged tiles; split-K (small grid); several tiles and super-blocks
SHAPES = [(256, 256, 128), (300, 512, 77), (512, 4096, 64), (1024, 2048, 256), (4096, 4096, 128), (100, 768, 8)]


@pytest.mark.parametrize("t", [O.Q4_K, O.Q4_0, O.Q8_0])
@pytest.mark.parametrize("n,k,m", SHAPES)
def test_tc_gemm_matches_oracle_and_f16_operands(n, k, m, t):
    w = make_weights(t, n, k, seed=n + 3 * k)
    x = _x(n + k + m, m, k)
    rb = O.row_bytes(t, k)
    got = run_tc(w, rb, x, n, k, m, t=t)
    assert np.isfinite(got).all()
    ref = O.gemv(t, w, rb, x, n, k, m, order=1)
    err = rel_l2(got, ref)
    assert err < NORTH_STAR, err
    ref16 = act_f16_operand(x) @ f16_operand(t, w, n, k).T
    assert rel_l2(got, ref16) < EXACT_F16_OPERANDS


def test_tc_gemm_q40_sweep_shape_and_swiglu():
    """Q4_0 at a BASELINE sweep shape (N 11008, K 4096, M 512) and as a SwiGLU pair with a fused
    RMSNorm, against the oracle."""
    import torch
    n, k, m = 11008, 4096, 512
    w = make_weights(O.Q4_0, n, k, seed=91)
    x = _x(92, m, k)
    rb = O.row_bytes(O.Q4_0, k)
    got = run_tc(w, rb, x, n, k, m, t=O.Q4_0)
    err = rel_l2(got, O.gemv(O.Q4_0, w, rb, x, n, k, m, order=1))
    print(f"Q4_0 tensor-core GEMM 11008x4096 M=512: rel_l2 {err:.2e}")
    assert err < NORTH_STAR
    f, k2, m2 = 1024, 2048, 64
    g, u = make_weights(O.Q4_0, f, k2, seed=93), make_weights(O.Q4_0, f, k2, seed=94)
    x2 = _x(95, m2, k2)
    gamma = (1.0 + 0.1 * _x(96, 1, k2)[0]).astype(np.float32)
    act = torch.empty((m2, f), device="cuda:0")
    rb2 = O.row_bytes(O.Q4_0, k2)
    Q.quant_swiglu_ex(O.Q4_0, dev(g).data_ptr(), dev(u).data_ptr(), rb2, rb2, dev(x2).data_ptr(), k2,
                      act.data_ptr(), f, f, k2, m2, dev(gamma).data_ptr(), 1e-6)
    xn = O.rmsnorm(x2, gamma, 1e-6)
    gv = O.gemv(O.Q4_0, g, rb2, xn, f, k2, m2, order=1).astype(np.float64)
    uv = O.gemv(O.Q4_0, u, rb2, xn, f, k2, m2, order=1).astype(np.float64)
    assert rel_l2(host(act), gv / (1 + np.exp(-gv)) * uv) < NORTH_STAR
    assert Q.last_launch_count() == 2  # xprep + the tensor-core GEMM


@pytest.mark.parametrize("n,k,m", [(4096, 4096, 512), (11008, 4096, 512), (4096, 11008, 2048)])
def test_tc_gemm_q80_sweep_shapes(n, k, m):
    """Q8_0 on the tensor cores at the BASELINE sweep shapes (M 512 and 2048, routed by QL_PATH_AUTO),
    against the oracle and against the exact f16 operands."""
    w = make_weights(O.Q8_0, n, k, seed=n + k + 7)
    x = _x(m + 5, m, k)
    rb = O.row_bytes(O.Q8_0, k)
    got = run_tc(w, rb, x, n, k, m, t=O.Q8_0, path=Q.PATH_AUTO)
    assert Q.last_launch_count() == 2  # xprep + the tensor-core GEMM
    mo = 256  # the oracle on one full 256-token tile (it takes ~1 s per GMAC on the host)
    err = rel_l2(got[:mo], O.gemv(O.Q8_0, w, rb, x[:mo], n, k, mo, order=1))
    print(f"Q8_0 tensor-core GEMM {n}x{k} M={m}: rel_l2 {err:.2e} (first {mo} tokens vs the oracle)")
    assert err < NORTH_STAR
    # every token against the exact f16 operands (float64 host product); fp32 accumulation error grows
    # with K (random walk over the K products), hence twice the bar at K = 11008
    ref16 = act_f16_operand(x) @ q80_f16_operand(w, n, k).T
    assert rel_l2(got, ref16) < EXACT_F16_OPERANDS * (2 if k > 8192 else 1)


def test_tc_gemm_q80_swiglu_stacked_bias_accumulate():
    """Q8_0 SwiGLU pair with a fused RMSNorm, a stacked q/k/v-style job with bias, and an accumulating
    plain GEMM, all on the tensor cores, against the oracle."""
    import torch
    f, k, m = 1280, 2048, 96
    g, u = make_weights(O.Q8_0, f, k, seed=201), make_weights(O.Q8_0, f, k, seed=202)
    x = _x(203, m, k)
    gamma = (1.0 + 0.1 * _x(204, 1, k)[0]).astype(np.float32)
    rb = O.row_bytes(O.Q8_0, k)
    act = torch.empty((m, f), device="cuda:0")
    Q.quant_swiglu_ex(O.Q8_0, dev(g).data_ptr(), dev(u).data_ptr(), rb, rb, dev(x).data_ptr(), k,
                      act.data_ptr(), f, f, k, m, dev(gamma).data_ptr(), 1e-6)
    assert Q.last_launch_count() == 2
    xn = O.rmsnorm(x, gamma, 1e-6)
    gv = O.gemv(O.Q8_0, g, rb, xn, f, k, m, order=1).astype(np.float64)
    uv = O.gemv(O.Q8_0, u, rb, xn, f, k, m, order=1).astype(np.float64)
    assert rel_l2(host(act), gv / (1 + np.exp(-gv)) * uv) < NORTH_STAR
    n = 640
    w = make_weights(O.Q8_0, n, k, seed=205)
    bias = _x(206, 1, n)[0]
    y0 = _x(207, m, n)
    got = run_tc(w, rb, x, n, k, m, gamma=gamma, eps=1e-6, bias=bias, y0=y0, t=O.Q8_0)
    ref = y0 + O.gemv(O.Q8_0, w, rb, xn, n, k, m, order=1) + bias[None, :]
    assert rel_l2(got, ref) < NORTH_STAR


def test_tc_gemm_fused_rmsnorm_bias_accumulate():
    n, k, m, eps = 640, 3584, 40, 1e-6
    w = make_weights(O.Q4_K, n, k, seed=41)
    x = _x(42, m, k) * 3.0
    gamma = (1.0 + 0.1 * _x(43, 1, k)[0]).astype(np.float32)
    bias = _x(44, 1, n)[0]
    y0 = _x(45, m, n)
    rb = O.row_bytes(O.Q4_K, k)
    got = run_tc(w, rb, x, n, k, m, gamma=gamma, eps=eps, bias=bias, y0=y0)
    ref = y0 + O.gemv(O.Q4_K, w, rb, O.rmsnorm(x, gamma, eps), n, k, m, order=1) + bias[None, :]
    assert rel_l2(got, ref) < NORTH_STAR
    ref16 = y0 + act_f16_operand(x, gamma, eps) @ q4k_f16_operand(w, n, k).T + bias[None, :]
    assert rel_l2(got, ref16) < EXACT_F16_OPERANDS


def test_tc_gemm_row_scaling_extremes():
    """Rows far outside f16 range, tiny rows and an all-zero row keep full relative precision."""
    n, k, m = 256, 512, 6
    w = make_weights(O.Q4_K, n, k, seed=51)
    x = _x(52, m, k)
    x[0] *= 1e6
    x[1] *= 1e-7
    x[2] = 0.0
    x[3, ::7] *= 1e4  # a row with a wide dynamic range
    rb = O.row_bytes(O.Q4_K, k)
    got = run_tc(w, rb, x, n, k, m)
    ref = O.gemv(O.Q4_K, w, rb, x, n, k, m, order=1)
    assert np.all(got[2] == 0.0)
    for r in (0, 1, 3, 4, 5):
        assert rel_l2(got[r], ref[r]) < NORTH_STAR, r


def test_tc_gemm_deterministic_with_k_split():
    n, k, m = 512, 8192, 32  # 2 tiles -> K split over many CTAs
    w = dev(make_weights(O.Q4_K, n, k, seed=61))
    x = dev(_x(62, m, k))
    import torch
    outs = []
    for _ in range(3):
        y = torch.empty((m, n), device="cuda:0")
        Q.quant_matmul_ex(O.Q4_K, w.data_ptr(), O.row_bytes(O.Q4_K, k), x.data_ptr(), k, y.data_ptr(), n, n, k, m,
                          None, 0.0, None, False, Q.PATH_TENSOR)
        outs.append(host(y).view(np.uint32))
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


def test_auto_path_routes_by_token_count():
    import torch
    n, k = 384, 1024
    w = make_weights(O.Q4_K, n, k, seed=71)
    rb = O.row_bytes(O.Q4_K, k)
    for m, forced in ((16, Q.PATH_TENSOR), (3, Q.PATH_GEMV)):
        x = _x(72 + m, m, k)
        y = torch.empty((m, n), device="cuda:0")
        Q.quant_matmul(O.Q4_K, dev(w).data_ptr(), rb, dev(x).data_ptr(), y.data_ptr(), n, k, m)
        assert np.array_equal(host(y).view(np.uint32), run_tc(w, rb, x, n, k, m, path=forced).view(np.uint32))


@pytest.mark.parametrize("t,k", [(O.Q5_0, 512), (O.Q8_0, 480)])
def test_tensor_path_rejects_ineligible_shapes(t, k):
    """No tensor-core kernel for Q5_0, and none for in_dim not a multiple of 256."""
    import torch
    w = make_weights(t, 64, k, seed=81)
    x = dev(_x(82, 16, k))
    y = torch.empty((16, 64), device="cuda:0")
    with pytest.raises(Q.QLError) as e:
        Q.quant_matmul_ex(t, dev(w).data_ptr(), O.row_bytes(t, k), x.data_ptr(), k, y.data_ptr(), 64,
                          64, k, 16, None, 0.0, None, False, Q.PATH_TENSOR)
    assert e.value.status == Q.QL_EINVAL


def test_tc_gemm_prefill_shape_against_torch():
    """Full Qwen2-7B gate/up prefill shape (M 2048, N 18944, K 3584) against torch
    fp32 (TF32 off) on the same f16 operands."""
    import torch
    n, k, m = 18944, 3584, 2048
    rb = O.row_bytes(O.Q4_K, k)
    wt = torch.empty((n, rb), dtype=torch.uint8, device="cuda:0")
    Q.synth_quantized(O.Q4_K, 5, n, k, 0.02, wt.data_ptr())
    x = _x(91, m, k)
    y = torch.empty((m, n), device="cuda:0")
    xd = dev(x)
    Q.quant_matmul_ex(O.Q4_K, wt.data_ptr(), rb, xd.data_ptr(), k, y.data_ptr(), n, n, k, m, None, 0.0, None, False,
                      Q.PATH_TENSOR)
    torch.cuda.synchronize()
    w16 = torch.from_numpy(q4k_f16_operand(host(wt), n, k).astype(np.float32)).to("cuda:0")
    x16 = torch.from_numpy(act_f16_operand(x).astype(np.float32)).to("cuda:0")
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = x16 @ w16.T
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    err = float(torch.linalg.norm((y - ref).double()) / torch.linalg.norm(ref.double()))
    assert err < EXACT_F16_OPERANDS, err


@pytest.mark.parametrize("m", [40, 300])
def test_tc_swiglu_matches_oracle(m):
    """Gate/up pair in one tensor-core launch, fused RMSNorm: below 128 tokens the tokens-as-M kernel
    (128 gate + 128 up rows per tile), from 128 tokens the weights-as-M kernel (64 + 64 rows per
    tile, A in tensor memory, a ragged last token tile at 300)."""
    import torch
    f, k, eps = 640, 1024, 1e-6
    g = make_weights(O.Q4_K, f, k, seed=101)
    u = make_weights(O.Q4_K, f, k, seed=102)
    x = _x(103, m, k)
    gamma = (1.0 + 0.1 * _x(104, 1, k)[0]).astype(np.float32)
    rb = O.row_bytes(O.Q4_K, k)
    act = torch.full((m, f), float("nan"), device="cuda:0")
    Q.quant_swiglu_ex(O.Q4_K, dev(g).data_ptr(), dev(u).data_ptr(), rb, rb, dev(x).data_ptr(), k, act.data_ptr(), f,
                      f, k, m, dev(gamma).data_ptr(), eps)
    got = host(act)
    xn = O.rmsnorm(x, gamma, eps)
    gv = O.gemv(O.Q4_K, g, rb, xn, f, k, m, order=1).astype(np.float64)
    uv = O.gemv(O.Q4_K, u, rb, xn, f, k, m, order=1).astype(np.float64)
    assert rel_l2(got, gv / (1.0 + np.exp(-gv)) * uv) < NORTH_STAR
    x16 = act_f16_operand(x, gamma, eps)
    g16 = x16 @ q4k_f16_operand(g, f, k).T
    u16 = x16 @ q4k_f16_operand(u, f, k).T
    assert rel_l2(got, g16 / (1.0 + np.exp(-g16)) * u16) < EXACT_F16_OPERANDS


@pytest.mark.parametrize("rows,m", [((512, 256, 100), 24), ((3584, 512, 512), 64), ((3584, 512, 512), 300)])
def test_tc_stacked_sources_match_concatenated(rows, m):
    """Stacked q/k/v sources (each but the last a multiple of 256 rows) with bias and fused norm."""
    import torch
    k, eps = 1024, 1e-6
    ws = [make_weights(O.Q4_K, r, k, seed=110 + i) for i, r in enumerate(rows)]
    x = _x(115, m, k)
    gamma = (1.0 + 0.1 * _x(116, 1, k)[0]).astype(np.float32)
    n = sum(rows)
    bias = _x(117, 1, n)[0]
    rb = O.row_bytes(O.Q4_K, k)
    y = torch.full((m, n), float("nan"), device="cuda:0")
    Q.quant_gemv_stacked_ex(O.Q4_K, [dev(w).data_ptr() for w in ws], [rb] * 3, list(rows), dev(x).data_ptr(), k,
                            y.data_ptr(), n, k, m, dev(gamma).data_ptr(), eps, dev(bias).data_ptr())
    got = host(y)
    wcat = np.concatenate(ws, axis=0)
    ref = O.gemv(O.Q4_K, wcat, rb, O.rmsnorm(x, gamma, eps), n, k, m, order=1) + bias[None, :]
    assert rel_l2(got, ref) < NORTH_STAR
    ref16 = act_f16_operand(x, gamma, eps) @ q4k_f16_operand(wcat, n, k).T + bias[None, :]
    assert rel_l2(got, ref16) < EXACT_F16_OPERANDS
