"""Opt-in Q8_1 activation path (ql_quantize_q8_1, ql_quant_gemv_q8_1) through the C ABI.

The quantizer must produce the reference's bytes exactly: checked against the oracle's
restatement (quantize_q8_1_kernel, kernel.cu:1679-1720) and against the reference's own kernel
(oracle/_ref).  The GEMV sums each block's integer dot product in a different order than the
reference (per lane, then a warp reduction, against the reference's block order on one lane or
per-element floats), so it is held to 1e-5 relative L2 against both."""
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


def _quantize(x, raw):
    import torch
    m, k = x.shape
    out = torch.zeros((m, Q.q8_1_row_bytes(k)), dtype=torch.uint8, device="cuda:0")
    Q.quantize_q8_1(dev(x).data_ptr(), out.data_ptr(), k, m, raw)
    assert Q.last_launch_count() == 1
    return host(out)


@pytest.mark.parametrize("raw", [False, True])
@pytest.mark.parametrize("m,k", [(1, 4096), (5, 3584), (3, 100), (2, 18944)])
def test_quantize_q8_1_bytes_match_oracle_and_reference(m, k, raw):
    import torch
    rng = np.random.default_rng(m * 7 + k)
    x = (rng.standard_normal((m, k)) * rng.uniform(0.01, 10.0, (m, 1))).astype(np.float32)
    x[0, :7] = 0.0  # a partly zero block
    got = _quantize(x, raw)
    assert np.array_equal(got, O.quantize_q8_1(x, raw))
    R = O.ref_lib()
    if R is not None:
        ref = torch.zeros((m, Q.q8_1_row_bytes(k)), dtype=torch.uint8, device="cuda:0")
        R.ref_set_stream(torch.cuda.current_stream().cuda_stream)
        R.ref_quantize_q8_1(dev(x).data_ptr(), ref.data_ptr(), k, m, int(raw))
        torch.cuda.synchronize()
        assert np.array_equal(got, host(ref))


@pytest.mark.parametrize("t,n,k", [(O.Q4_K, 4096, 4096), (O.Q6_K, 1000, 2048), (O.Q5_0, 1000, 1408),
                                   (O.Q8_0, 3000, 896)])
def test_gemv_q8_1_matches_oracle_and_reference(t, n, k):
    import torch
    w = make_weights(t, n, k, seed=n + k + t)
    rb = O.row_bytes(t, k)
    x = np.random.default_rng(k).standard_normal((1, k)).astype(np.float32)
    xq = O.quantize_q8_1(x, t == O.Q4_K)[0]
    y = torch.full((n,), float("nan"), device="cuda:0")
    Q.quant_gemv_q8_1(t, dev(w).data_ptr(), rb, dev(xq).data_ptr(), y.data_ptr(), n, k)
    got = host(y)
    err = rel_l2(got, O.gemv_q8_1(t, w, rb, xq, n, k))
    exact = rel_l2(got, O.gemv(t, w, rb, x, n, k, 1, order=1)[0])
    print(f"Q8_1 GEMV type {t}: rel_l2 {err:.2e} vs the oracle's Q8_1 form, {exact:.2e} vs fp32 activations")
    assert err < TOL
    R = O.ref_lib()
    if R is not None:
        ref = torch.zeros(n, device="cuda:0")
        R.ref_set_stream(torch.cuda.current_stream().cuda_stream)
        R.ref_quant_gemv_q8_1(t, dev(w).data_ptr(), rb, dev(xq).data_ptr(), ref.data_ptr(), n, k)
        torch.cuda.synchronize()
        assert rel_l2(got, host(ref)) < TOL


@pytest.mark.parametrize("t,n,k,m", [(O.Q4_K, 1000, 2048, 100), (O.Q6_K, 300, 1024, 37), (O.Q5_0, 520, 1408, 64),
                                     (O.Q8_0, 777, 896, 16), (O.Q8_0, 64, 4096, 3)])
def test_matmul_q8_1_matches_oracle_and_reference(t, n, k, m):
    """The tensor-core Q8_1 matmul (ragged row and token tiles; Q8_0 with in_dim 4096 runs the
    per-token GEMV) against the oracle's per-token Q8_1 GEMV and the reference's matmul kernel."""
    import torch
    w = make_weights(t, n, k, seed=3 * n + k + t)
    rb = O.row_bytes(t, k)
    x = np.random.default_rng(m + k).standard_normal((m, k)).astype(np.float32)
    xq = O.quantize_q8_1(x, t == O.Q4_K)
    y = torch.full((m, n), float("nan"), device="cuda:0")
    Q.quant_matmul_q8_1(t, dev(w).data_ptr(), rb, dev(xq).data_ptr(), y.data_ptr(), n, k, m)
    got = host(y)
    want = np.stack([O.gemv_q8_1(t, w, rb, xq[i], n, k) for i in range(m)])
    err = rel_l2(got, want)
    print(f"Q8_1 matmul type {t} {n}x{k} M={m}: rel_l2 {err:.2e} (launches {Q.last_launch_count()})")
    assert err < TOL
    R = O.ref_lib()
    if R is not None:
        ref = torch.zeros((m, n), device="cuda:0")
        R.ref_set_stream(torch.cuda.current_stream().cuda_stream)
        R.ref_quant_matmul_q8_1(t, dev(w).data_ptr(), rb, dev(xq).data_ptr(), ref.data_ptr(), n, k, m)
        torch.cuda.synchronize()
        assert rel_l2(got, host(ref)) < TOL


@pytest.mark.parametrize("t,n,k,m,raw", [(O.Q4_K, 600, 2048, 40, True), (O.Q6_K, 300, 1024, 19, False)])
def test_mmq_layout_quantizer_and_matmul(t, n, k, m, raw):
    """The packed (MMQ) Q8_1 layout: quantizer bytes equal to the oracle's blocks repacked and to the
    reference's own MMQ quantizer; the matmul from that layout equal to the plain-layout matmul and
    within 1e-5 of the reference's MMQ matmul kernel."""
    import torch
    x = np.random.default_rng(n + m).standard_normal((m, k)).astype(np.float32)
    xm = torch.zeros(m * Q.q8_1_mmq_row_bytes(k), dtype=torch.uint8, device="cuda:0")
    Q.quantize_q8_1_mmq(dev(x).data_ptr(), xm.data_ptr(), k, m, raw)
    got_bytes = host(xm)
    rows = O.quantize_q8_1(x, raw)
    assert np.array_equal(got_bytes, O.q8_1_mmq_from_rows(rows, k))
    R = O.ref_lib()
    w = make_weights(t, n, k, seed=n + 5 * k)
    rb = O.row_bytes(t, k)
    y = torch.full((m, n), float("nan"), device="cuda:0")
    Q.quant_matmul_q8_1_mmq(t, dev(w).data_ptr(), rb, xm.data_ptr(), y.data_ptr(), n, k, m)
    yp = torch.full((m, n), float("nan"), device="cuda:0")
    Q.quant_matmul_q8_1(t, dev(w).data_ptr(), rb, dev(rows).data_ptr(), yp.data_ptr(), n, k, m)
    assert np.array_equal(host(y), host(yp))
    if R is not None:
        ref = torch.zeros(m * Q.q8_1_mmq_row_bytes(k), dtype=torch.uint8, device="cuda:0")
        R.ref_set_stream(torch.cuda.current_stream().cuda_stream)
        R.ref_quantize_q8_1_mmq(dev(x).data_ptr(), ref.data_ptr(), k, m, int(raw))
        yr = torch.zeros((m, n), device="cuda:0")
        R.ref_quant_matmul_q8_1_mmq(t, dev(w).data_ptr(), rb, xm.data_ptr(), yr.data_ptr(), n, k, m)
        torch.cuda.synchronize()
        assert np.array_equal(got_bytes, host(ref))
        err = rel_l2(host(y), host(yr))
        print(f"MMQ matmul type {t}: rel_l2 {err:.2e} vs the reference's MMQ kernel")
        assert err < TOL


def test_q8_1_rejects_unsupported_types():
    import torch
    x = torch.zeros(64, device="cuda:0")
    with pytest.raises(Q.QLError) as e:
        Q.quant_gemv_q8_1(O.Q4_0, x.data_ptr(), 18, x.data_ptr(), x.data_ptr(), 1, 32)
    assert e.value.status == Q.QL_EINVAL
