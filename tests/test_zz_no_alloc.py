"""ql_argmax_noalloc: the argmax for callers that cannot let the library
allocate device memory (HBM owned by the caller's own pool or budgeted once at
start-up, an allocation ban after start-up).  It must return what
ql_argmax returns, call after call, through the C ABI.

This file sorts last so that a run stopping at its first failure has run
every other test already; it also passes alone in a fresh process."""
import numpy as np
import pytest

import blog_b200 as Q

pytestmark = pytest.mark.gpu


def _logits(seed, n):
    v = np.random.default_rng(seed).standard_normal(n).astype(np.float32)
    if n > 16:
        v[[5, n // 3, n - 2]] = v.max() + 2.0  # a three-way tie: lowest index wins
        v[1] = np.nan
    return v


@pytest.mark.parametrize("n", [1, 1000, 152064, 1 << 22])
def test_argmax_noalloc_matches_argmax_twice(n):
    import torch
    torch.cuda.init()
    L = Q.lib()
    assert L.ql_set_stream(torch.cuda.current_stream().cuda_stream) == Q.QL_OK
    for call in range(2):  # the shared scratch keeps the previous call's contents
        x = torch.from_numpy(_logits(100 * call + n % 97, n)).cuda()
        a = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        b = torch.full((1,), -2, dtype=torch.int32, device="cuda")
        assert L.ql_argmax_noalloc(x.data_ptr(), n, a.data_ptr()) == Q.QL_OK, L.ql_last_error()
        assert L.ql_last_launch_count() == 2
        assert L.ql_argmax(x.data_ptr(), n, b.data_ptr()) == Q.QL_OK, L.ql_last_error()
        torch.cuda.synchronize()
        assert int(a.item()) == int(b.item())
        assert int(a.item()) == int(np.nanargmax(np.where(np.isnan(x.cpu().numpy()), -np.inf, x.cpu().numpy())))


def test_argmax_noalloc_rejects_oversize():
    L = Q.lib()
    assert L.ql_argmax_noalloc(1 << 40, (1 << 24) + 1, 1 << 40) == Q.QL_EINVAL
    assert b"no-allocation maximum" in L.ql_last_error()
