"""CPU-only checks of the native library: exports, argument validation and the
stream-K work plan (no kernel runs here)."""
import os
import re

import pytest

import blog_b200 as Q
from blog_b200 import build as B

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        if h.endswith(".h"):
            text = open(os.path.join(ROOT, "include", h)).read()
            names |= set(re.findall(r"^QL_API[^;(]*?\b(ql_\w+)\s*\(", text, flags=re.M))
    return names


def test_library_exports_every_declared_symbol():
    import subprocess
    if not os.path.exists(Q.LIB_PATH):
        B.build()
    out = subprocess.run(["nm", "-D", "--defined-only", Q.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (ql_\w+)", out))
    declared = declared_symbols()
    assert declared, "no declarations parsed"
    assert declared <= exported, f"declared but not exported: {sorted(declared - exported)}"
    assert set(Q.SIGNATURES) == declared, "ctypes signature table out of sync with the header"


def test_library_loads_and_binds():
    L = Q.lib()
    for name in Q.SIGNATURES:
        assert hasattr(L, name)


@pytest.mark.parametrize("t,k,rb", [(Q.Q4_K, 4096, 16 * 144), (Q.Q8_0, 896, 28 * 34), (Q.Q4_0, 29568, 924 * 18)])
def test_row_bytes(t, k, rb):
    assert Q.lib().ql_row_bytes(t, k) == rb == Q.row_bytes(t, k)
    assert Q.lib().ql_row_bytes(t, k + 1) == 0


def test_validation_rejects_without_touching_the_device():
    L = Q.lib()
    fake = 1 << 40  # never dereferenced: validation fails first
    # unsupported dtype (the reference silently no-ops here, launch.cu:57-58)
    assert L.ql_quant_gemv(3, fake, 144, fake, fake, 8, 256, 1) == Q.QL_EINVAL
    assert b"unsupported quant_type" in L.ql_last_error()
    # in_dim not a block multiple
    assert L.ql_quant_gemv(Q.Q4_K, fake, 144, fake, fake, 8, 100, 1) == Q.QL_EINVAL
    # row_bytes too small
    assert L.ql_quant_gemv(Q.Q8_0, fake, 33, fake, fake, 8, 32, 1) == Q.QL_EINVAL
    # Q4_K needs 16-byte aligned rows
    assert L.ql_quant_gemv(Q.Q4_K, fake + 8, 144, fake, fake, 8, 256, 1) == Q.QL_EINVAL
    # router limits (the reference kernel has a fixed used[64])
    assert L.ql_moe_router_topk(fake, fake, fake, 4, 65, 6, 1.0) == Q.QL_EINVAL
    assert L.ql_moe_router_topk(fake, fake, fake, 4, 64, 0, 1.0) == Q.QL_EINVAL
    # dequant element count not a block multiple
    assert L.ql_dequantize_to_f16(Q.Q4_K, fake, fake, 300) == Q.QL_EINVAL
    # null weight
    assert L.ql_quant_swiglu(Q.Q8_0, None, fake, 34, 34, fake, fake, 4, 32) == Q.QL_EINVAL
    # zero-size calls are no-ops
    assert L.ql_quant_gemv(Q.Q8_0, fake, 34, fake, fake, 0, 32, 1) == Q.QL_OK


# ---------------------------------------------------------------------------
# Python restatement of the stream-K plan (ql_common.cuh Plan, ql_gemv.cuh
# next_stage): every (group, block) tile is visited exactly once, stages obey
# the segment and route limits, and each group's parts are the CTAs found by
# plan_cta_of.
# ---------------------------------------------------------------------------
def plan_start(T, C, c):
    return c * T // C


def cta_of(T, C, t):
    return ((t + 1) * C - 1) // T


def stages(t0, t1, U, seg, upr):
    t = t0
    while t < t1:
        g, u = divmod(t, U)
        gend = min((g + 1) * U, t1)
        uend = u + (gend - t)
        ue = min(u + seg, uend)
        if upr:
            ue = min(ue, (u // upr + 1) * upr)
        yield g, u, ue, ue == uend
        t += ue - u


@pytest.mark.parametrize("G,U,C,seg,upr", [
    (112, 14, 148, 4, 0), (592, 14, 148, 4, 0), (112, 74, 148, 4, 0), (4752, 14, 148, 4, 0),
    (1, 1, 1, 16, 0), (1, 43, 148, 4, 0), (3, 7, 5, 2, 0), (64, 264, 148, 24, 44), (9, 12, 7, 16, 2),
])
def test_stream_k_plan_covers_every_tile_once(G, U, C, seg, upr):
    T = G * U
    C = min(C, T)
    seen = [0] * T
    parts = {}
    for c in range(C):
        t0, t1 = plan_start(T, C, c), plan_start(T, C, c + 1)
        assert t1 > t0
        for g, us, ue, last in stages(t0, t1, U, seg, upr):
            assert 0 < ue - us <= seg
            if upr:
                assert us // upr == (ue - 1) // upr
            for u in range(us, ue):
                seen[g * U + u] += 1
            parts.setdefault(g, set()).add(c)
    assert all(v == 1 for v in seen)
    for g, cs in parts.items():
        assert min(cs) == cta_of(T, C, g * U) and max(cs) == cta_of(T, C, (g + 1) * U - 1)
        assert cs == set(range(min(cs), max(cs) + 1))
        # partial-slot rule: slot 0 when g is the CTA's first group, else slot 1; never shared
        slots = {(c, 0 if g == plan_start(T, C, c) // U else 1) for c in cs}
        assert len(slots) == len(cs)
