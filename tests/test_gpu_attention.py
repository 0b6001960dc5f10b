"""Causal gated decode attention (ql_full_attention_attend{,_batch}) against the oracle's restatement
of the reference kernel (full_attn_attend_head, kernel.cu:355-430; double-precision softmax) and
against the reference's own kernel (launch_full_attention_attend, built from its sources into
oracle/_ref), through the C ABI.  Both compute in fp32 with different summation orders and exp
implementations, so the bar is 1e-5 relative L2."""
import numpy as np
import pytest

import blog_b200 as Q
import oracle as O
from gpu_util import dev, host, rel_l2

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


def _case(seed, tokens, n_heads, kv_heads, hd, max_seq, bf16):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((tokens, n_heads * hd)).astype(np.float32)
    gate = rng.standard_normal((tokens, n_heads * hd)).astype(np.float32)
    k = (rng.standard_normal((max_seq, kv_heads * hd)) * 0.5).astype(np.float32)
    v = rng.standard_normal((max_seq, kv_heads * hd)).astype(np.float32)
    if bf16:  # bf16 bits (round to nearest even) as the cache stores them
        k, v = (np.round(a.view(np.uint32).astype(np.uint64) / 65536.0).astype(np.uint32).astype(np.uint16)
                for a in (k, v))
    return q, gate, k, v


def _run_single(q, gate, k, v, bf16, n_heads, kv_heads, hd, max_seq, pos):
    import torch
    out = torch.full((n_heads * hd,), float("nan"), device="cuda:0")
    p = dev(np.array([pos], np.int32))
    Q.full_attention_attend(dev(q).data_ptr(), dev(gate).data_ptr(), dev(k).data_ptr(), dev(v).data_ptr(), bf16,
                            out.data_ptr(), n_heads, kv_heads, hd, max_seq, p.data_ptr())
    assert Q.last_launch_count() == 2  # key splits + merge
    return host(out)


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("pos", [0, 1, 63, 64, 200, 4095])
def test_decode_attention_qwen2_7b_heads(pos, bf16):
    """Qwen2-7B attention shape (28 query heads over 4 KV heads, head_dim 128), cache of 4096."""
    nh, kvh, hd, ms = 28, 4, 128, 4096
    q, gate, k, v = _case(400 + pos, 1, nh, kvh, hd, ms, bf16)
    got = _run_single(q, gate, k, v, bf16, nh, kvh, hd, ms, pos)
    ref = O.attention_attend(q, gate, k, v, bf16, 1, nh, kvh, hd, pos)[0]
    err = rel_l2(got, ref)
    print(f"decode attention pos {pos} bf16 {bf16}: rel_l2 {err:.2e}")
    assert err < TOL


@pytest.mark.parametrize("bf16", [False, True])
def test_decode_attention_matches_reference_kernel(bf16):
    """The reference's own CUDA kernel on the same inputs (device position)."""
    import torch
    R = O.ref_lib()
    if R is None:
        pytest.skip("reference kernels not built")
    nh, kvh, hd, ms, pos = 28, 4, 128, 1024, 777
    q, gate, k, v = _case(430, 1, nh, kvh, hd, ms, bf16)
    got = _run_single(q, gate, k, v, bf16, nh, kvh, hd, ms, pos)
    out = torch.zeros(nh * hd, device="cuda:0")
    p = dev(np.array([pos], np.int32))
    R.ref_set_stream(torch.cuda.current_stream().cuda_stream)
    R.ref_full_attention_attend(dev(q).data_ptr(), dev(gate).data_ptr(), dev(k).data_ptr(), dev(v).data_ptr(),
                                int(bf16), out.data_ptr(), nh, kvh, hd, ms, p.data_ptr())
    torch.cuda.synchronize()
    assert R.ref_last_error() == 0
    err = rel_l2(got, host(out))
    print(f"decode attention vs the reference kernel (bf16 {bf16}): rel_l2 {err:.2e}")
    assert err < TOL


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("nh,kvh,hd", [(8, 8, 64), (32, 4, 256), (16, 2, 96), (13, 1, 128), (32, 2, 64)])
def test_decode_attention_batch_and_group_shapes(nh, kvh, hd, bf16):
    """Batched queries (causal: token t sees keys 0..start_pos + t), group sizes 1, 8, 8, 13 and 16
    with head_dim 64 / 256 / 96 / 128 / 64 (groups above 8 take the 16-head kernel variant, an odd
    group ends on a single-head pair; head_dim <= 128 stages tiles by cp.async, 256 through
    registers), f32 and bf16 caches, against the oracle and against the reference's batch kernel."""
    import torch
    tokens, ms, start = 5, 300, 37
    q, gate, k, v = _case(450 + hd, tokens, nh, kvh, hd, ms, bf16)
    out = torch.full((tokens, nh * hd), float("nan"), device="cuda:0")
    Q.full_attention_attend_batch(dev(q).data_ptr(), dev(gate).data_ptr(), dev(k).data_ptr(), dev(v).data_ptr(),
                                  bf16, out.data_ptr(), tokens, nh, kvh, hd, ms, start)
    got = host(out)
    ref = O.attention_attend(q, gate, k, v, bf16, tokens, nh, kvh, hd, start)
    assert rel_l2(got, ref) < TOL
    R = O.ref_lib()
    if R is not None:
        out2 = torch.zeros((tokens, nh * hd), device="cuda:0")
        R.ref_set_stream(torch.cuda.current_stream().cuda_stream)
        R.ref_full_attention_attend_batch(dev(q).data_ptr(), dev(gate).data_ptr(), dev(k).data_ptr(),
                                          dev(v).data_ptr(), int(bf16), out2.data_ptr(), tokens, nh, kvh, hd, ms,
                                          start)
        torch.cuda.synchronize()
        assert rel_l2(got, host(out2)) < TOL


def test_decode_attention_position_is_read_on_the_device():
    """One buffer holds the position; updating it between calls (as a replayed graph does) moves
    the causal window."""
    import torch
    nh, kvh, hd, ms = 28, 4, 128, 512
    q, gate, k, v = _case(470, 1, nh, kvh, hd, ms, False)
    qd, gd, kd, vd = dev(q), dev(gate), dev(k), dev(v)
    p = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    out = torch.empty(nh * hd, device="cuda:0")
    for pos in (10, 300, 511):
        p.fill_(pos)
        Q.full_attention_attend(qd.data_ptr(), gd.data_ptr(), kd.data_ptr(), vd.data_ptr(), False, out.data_ptr(),
                                nh, kvh, hd, ms, p.data_ptr())
        assert rel_l2(host(out), O.attention_attend(q, gate, k, v, False, 1, nh, kvh, hd, pos)[0]) < TOL


def test_decode_attention_replays_in_a_cuda_graph():
    """The single-token call (key splits, then the merge as a programmatic dependent launch) captured
    once in a CUDA graph and replayed with the device position moved between replays, f32 and bf16."""
    import torch
    nh, kvh, hd, ms = 28, 4, 128, 512
    for bf16 in (False, True):
        q, gate, k, v = _case(480 + int(bf16), 1, nh, kvh, hd, ms, bf16)
        qd, gd, kd, vd = dev(q), dev(gate), dev(k), dev(v)
        p = torch.zeros(1, dtype=torch.int32, device="cuda:0")
        out = torch.empty(nh * hd, device="cuda:0")

        def call():
            Q.full_attention_attend(qd.data_ptr(), gd.data_ptr(), kd.data_ptr(), vd.data_ptr(), bf16, out.data_ptr(),
                                    nh, kvh, hd, ms, p.data_ptr())
        try:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                Q.set_stream(s.cuda_stream)
                p.fill_(3)
                call()  # workspace sized outside the capture
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=s):
                    call()
                for pos in (10, 300, 511):
                    p.fill_(pos)
                    g.replay()
                    torch.cuda.synchronize()
                    err = rel_l2(host(out), O.attention_attend(q, gate, k, v, bf16, 1, nh, kvh, hd, pos)[0])
                    assert err < TOL, (bf16, pos, err)
            del g
        finally:
            Q.set_stream(torch.cuda.current_stream().cuda_stream)


def test_decode_attention_rejects_bad_shapes():
    import torch
    x = torch.zeros(64, device="cuda:0")
    with pytest.raises(Q.QLError) as e:  # n_heads not a multiple of kv_heads
        Q.full_attention_attend_batch(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), False, x.data_ptr(),
                                      1, 6, 4, 8, 8, 0)
    assert e.value.status == Q.QL_EINVAL
    with pytest.raises(Q.QLError) as e:  # past the cache
        Q.full_attention_attend_batch(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), False, x.data_ptr(),
                                      4, 4, 4, 8, 8, 6)
    assert e.value.status == Q.QL_EINVAL
