"""CPU oracle for the block-quantized linear path (TEST INFRASTRUCTURE ONLY).

Wraps ``liboracle.so`` (qlinear_oracle.c, a C restatement of the reference's
CUDA arithmetic) and, when built, ``_ref/libref_local_llm.so`` (the reference's
own CUDA kernels compiled from its sources for sm_100a).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import
this package; the product library never does.

Parity status: pinned by the reference's known-answer tests
(test/LaunchAddTest.cpp), by gguf-py 0.19.0 vectors, and on a GPU bit for bit
against the reference's own kernels.  Q4_0 is pinned by gguf-py only (the
reference has no Q4_0 arithmetic).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libref_local_llm.so")

# GGML type codes (reference src/tensor/TensorCommon.h:15-33)
F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 6, 8, 12, 14
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q5_0: (32, 22), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}
NAMES = {Q4_0: "Q4_0", Q5_0: "Q5_0", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K", F16: "F16", F32: "F32"}


def row_bytes(t: int, k: int) -> int:
    be, bb = BLOCK[t]
    assert k % be == 0, (t, k)
    return k // be * bb


def build() -> None:
    """Compile liboracle.so (and _ref when the reference sources are present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P, I, I64, U64, SZ, F = C.c_void_p, C.c_int, C.c_int64, C.c_uint64, C.c_size_t, C.c_float
        sig = {
            "orc_f16_to_f32": (F, [C.c_uint16]),
            "orc_f32_to_f16": (C.c_uint16, [F]),
            "orc_dequant_rows_f32": (I, [I, P, SZ, I64, I, P]),
            "orc_dequant_f16": (I, [I, P, I64, P]),
            "orc_gemv": (I, [I, P, SZ, P, P, I, I, I, I]),
            "orc_gemv_add": (I, [I, P, SZ, P, P, I, I, I]),
            "orc_swiglu": (I, [I, P, P, SZ, SZ, P, P, I, I, I]),
            "orc_swiglu_indexed": (I, [I, P, P, SZ, SZ, SZ, SZ, P, P, P, I, I, I, I]),
            "orc_down_indexed_ordered": (I, [I, P, SZ, SZ, P, P, P, P, I, I, I, I]),
            "orc_router_topk": (I, [P, P, P, I, I, I, F]),
            "orc_attention_attend": (I, [P, P, P, P, I, P, I, I, I, I, I]),
            "orc_quantize_q8_1": (I, [P, P, I, I, I]),
            "orc_gemv_q8_1": (I, [I, P, C.c_size_t, P, P, I, I]),
            "orc_argmax": (I, [P, I]),
            "orc_rmsnorm": (None, [P, P, P, I, I, F]),
            "orc_embedding": (I, [I, P, P, P, SZ, I, I]),
            "orc_quantize_rows": (I, [I, P, I64, I, P]),
            "orc_randn": (None, [U64, U64, I64, F, P]),
            "orc_num_threads": (I, []),
            "orc_set_num_threads": (None, [I]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def _ok(rc):
    if rc != 0:
        raise ValueError(f"oracle call rejected its arguments (rc={rc})")


def randn(seed: int, n: int, std: float = 1.0, offset: int = 0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_randn(seed, offset, n, std, _p(out))
    return out


def quantize(t: int, x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    rows, k = x.shape
    out = np.empty((rows, row_bytes(t, k)), np.uint8)
    _ok(lib().orc_quantize_rows(t, _p(x), rows, k, _p(out)))
    return out


def dequant_rows(t: int, w: np.ndarray, k: int, rb: int | None = None) -> np.ndarray:
    w = _c(w, np.uint8)
    rb = rb if rb is not None else row_bytes(t, k)
    rows = w.size // rb
    out = np.empty((rows, k), np.float32)
    _ok(lib().orc_dequant_rows_f32(t, _p(w), rb, rows, k, _p(out)))
    return out


def dequant_f16(t: int, src: np.ndarray, n: int) -> np.ndarray:
    src = _c(src, np.uint8)
    out = np.empty(n, np.uint16)
    _ok(lib().orc_dequant_f16(t, _p(src), n, _p(out)))
    return out


def gemv(t, w, rb, x, n, k, m, order=0):
    w, x = _c(w, np.uint8), _c(x, np.float32)
    y = np.empty((m, n), np.float32)
    _ok(lib().orc_gemv(t, _p(w), rb, _p(x), _p(y), n, k, m, order))
    return y


def gemv_add(t, w, rb, x, y, n, k, order=0):
    w, x = _c(w, np.uint8), _c(x, np.float32)
    y = np.array(y, np.float32, copy=True)
    _ok(lib().orc_gemv_add(t, _p(w), rb, _p(x), _p(y), n, k, order))
    return y


def swiglu(t, g, u, grb, urb, x, f, k, order=0):
    g, u, x = _c(g, np.uint8), _c(u, np.uint8), _c(x, np.float32)
    act = np.empty(f, np.float32)
    _ok(lib().orc_swiglu(t, _p(g), _p(u), grb, urb, _p(x), _p(act), f, k, order))
    return act


def swiglu_indexed(t, g, u, geb, ueb, grb, urb, x, ids, k, f, kin, order=0):
    g, u, x = _c(g, np.uint8), _c(u, np.uint8), _c(x, np.float32)
    ids = _c(ids, np.int32)
    act = np.empty((k, f), np.float32)
    _ok(lib().orc_swiglu_indexed(t, _p(g), _p(u), geb, ueb, grb, urb, _p(x), _p(ids), _p(act), k, f, kin, order))
    return act


def down_indexed_ordered(t, d, deb, drb, act, ids, rw, out, k, h, f, order=0):
    d, act = _c(d, np.uint8), _c(act, np.float32)
    ids, rw = _c(ids, np.int32), _c(rw, np.float32)
    out = np.array(out, np.float32, copy=True)
    _ok(lib().orc_down_indexed_ordered(t, _p(d), deb, drb, _p(act), _p(ids), _p(rw), _p(out), k, h, f, order))
    return out


def attention_attend(q, gate, kc, vc, kv_bf16, tokens, n_heads, kv_heads, head_dim, start_pos):
    """Causal gated decode attention for `tokens` queries at positions start_pos.. (restates
    full_attn_attend_head, kernel.cu:355-430); kc / vc: [seq][kv_heads][head_dim] float32, or uint16
    bf16 bits when kv_bf16."""
    q, gate = _c(q, np.float32), _c(gate, np.float32)
    kc, vc = _c(kc, np.uint16 if kv_bf16 else np.float32), _c(vc, np.uint16 if kv_bf16 else np.float32)
    out = np.empty((tokens, n_heads * head_dim), np.float32)
    _ok(lib().orc_attention_attend(_p(q), _p(gate), _p(kc), _p(vc), int(kv_bf16), _p(out), tokens, n_heads,
                                   kv_heads, head_dim, start_pos))
    return out


def q8_1_row_bytes(k: int) -> int:
    return (k + 31) // 32 * 36


def quantize_q8_1(x, store_raw_sum=False):
    """Q8_1 blocks of each row of x [m, k] (restates quantize_q8_1_kernel, kernel.cu:1679-1720)."""
    x = _c(np.atleast_2d(x), np.float32)
    m, k = x.shape
    out = np.empty((m, q8_1_row_bytes(k)), np.uint8)
    _ok(lib().orc_quantize_q8_1(_p(x), _p(out), k, m, int(store_raw_sum)))
    return out


def q8_1_mmq_from_rows(xq_rows, k):
    """The packed (MMQ) layout of Q8_1 rows [m][q8_1_row_bytes(k)] (quantize_q8_1_mmq_kernel's
    layout, kernel.cu:1724-1765): per 128 activations a 144-byte group {4 x (d, sum), 4 x 32 int8},
    group-major; blocks past the row's last are those of zeros (d = sum = 0, q = 0)."""
    xq_rows = np.atleast_2d(xq_rows)
    m = xq_rows.shape[0]
    bpr, groups = (k + 31) // 32, (k + 127) // 128
    out = np.zeros((groups, m, 144), np.uint8)
    for b in range(bpr):
        blk = xq_rows[:, b * 36:(b + 1) * 36]
        g, sub = b // 4, b % 4
        out[g, :, 4 * sub:4 * sub + 4] = blk[:, 0:4]
        out[g, :, 16 + 32 * sub:48 + 32 * sub] = blk[:, 4:36]
    return out.reshape(-1)


def gemv_q8_1(t, w, rb, xq, n, k):
    """y[n] against one Q8_1 activation row (restates quant_gemv_q8_1_kernel, kernel.cu:1767-1865)."""
    w, xq = _c(w, np.uint8), _c(xq, np.uint8)
    y = np.empty(n, np.float32)
    _ok(lib().orc_gemv_q8_1(t, _p(w), rb, _p(xq), _p(y), n, k))
    return y


def router_topk(logits, k, scale):
    logits = _c(logits, np.float32)
    t, e = logits.shape
    idx = np.empty((t, k), np.int32)
    w = np.empty((t, k), np.float32)
    _ok(lib().orc_router_topk(_p(logits), _p(idx), _p(w), t, e, k, scale))
    return idx, w


def argmax(v) -> int:
    v = _c(v, np.float32)
    return int(lib().orc_argmax(_p(v), v.size))


def rmsnorm(x, gamma, eps):
    x = _c(x, np.float32)
    rows, h = x.reshape(-1, x.shape[-1]).shape
    y = np.empty_like(x)
    g = _c(gamma, np.float32) if gamma is not None else None
    lib().orc_rmsnorm(_p(x), _p(y), _p(g) if g is not None else None, rows, h, eps)
    return y


def embedding(t, ids, table, rb, h):
    ids, table = _c(ids, np.int32), _c(table, np.uint8)
    out = np.empty((ids.size, h), np.float32)
    _ok(lib().orc_embedding(t, _p(ids), _p(out), _p(table), rb, h, ids.size))
    return out


def num_threads() -> int:
    return int(lib().orc_num_threads())


def set_threads(n: int) -> None:
    """OpenMP threads of the oracle's loops (overrides OMP_NUM_THREADS)."""
    lib().orc_set_num_threads(int(n))


def host_cores() -> int:
    """Cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ----------------------------------------------------------------------------
# One decode token of a Qwen2-style linear stack, restated on the CPU.
#
# The reference's decode step (DeepSeek/Qwen engines: LL/src/llm/module/*) is, per
# layer, rms_norm (kernel.cu:112-147) -> q/k/v projections (+ bias) -> attention ->
# o projection + residual add (kernel.cu:80-84) -> rms_norm -> gate/up SwiGLU
# (quant_swiglu_kernel, kernel.cu:1288-1328) -> down projection + residual; then the
# final rms_norm, the LM head and the greedy argmax (kernel.cu:3531-3592, strict '>'
# as Sampler.cpp:24-50).  Attention is outside the quantized-linear path: its output
# is stood in by the q projection (which has o_proj's input width).  Each layer is a
# dict of quantized weights wq, wk, wv, wo, wg, wu, wd ([rows, row_bytes] uint8) and
# float32 ln1, ln2, bqkv.
# ----------------------------------------------------------------------------
def rope(x, pos, theta, head_dim, rows):
    """Rotary embedding of rows [0, rows) of x[..., :] (whole heads of head_dim), restating the
    reference's rotation (kernel.cu:186-260): for i < head_dim/2, inv_freq = 1 / powf(theta,
    2i / head_dim) and angle = pos * inv_freq in fp32, then (x1, x2) -> (x1 c - x2 s, x2 c + x1 s)
    for x1 = row i and x2 = row i + head_dim/2 of each head.  x: [tokens, n]; pos: one per token."""
    x = np.array(x, np.float64, copy=True)
    half = head_dim // 2
    i = np.arange(half, dtype=np.float32)
    inv = np.float32(1.0) / np.power(np.float32(theta), (np.float32(2) * i) / np.float32(head_dim))
    for tk, p in enumerate(np.atleast_1d(pos)):
        ang = (np.float32(p) * inv).astype(np.float64)
        c, s = np.cos(ang), np.sin(ang)
        for h0 in range(0, rows, head_dim):
            x1, x2 = x[tk, h0:h0 + half].copy(), x[tk, h0 + half:h0 + head_dim].copy()
            x[tk, h0:h0 + half] = x1 * c - x2 * s
            x[tk, h0 + half:h0 + head_dim] = x2 * c + x1 * s
    return x


def linear_stack_token(layers, lm, lnf, h, t=Q4_K, eps=1e-6, order=1, with_logits=True, rope_args=None):
    """h (float32 [hidden]) -> (h after the stack, logits or None, greedy token).  rope_args
    (pos, theta, head_dim, rows): RoPE on the first `rows` q/k/v outputs, as the chain's fused
    epilogue does."""
    h = np.array(h, np.float32, copy=True).reshape(1, -1)
    H = h.shape[1]
    for L in layers:
        xn = rmsnorm(h, L["ln1"], eps)
        parts = [gemv(t, L[n], L[n].shape[1], xn, L[n].shape[0], H, 1, order) for n in ("wq", "wk", "wv")]
        qkv = np.concatenate(parts, axis=1) + np.asarray(L["bqkv"], np.float32)[None, :]
        if rope_args is not None:
            qkv = rope(qkv, *rope_args).astype(np.float32)
        qw = L["wq"].shape[0]
        h = gemv_add(t, L["wo"], L["wo"].shape[1], qkv[:, :qw], h[0], H, qw, order).reshape(1, -1)
        xn = rmsnorm(h, L["ln2"], eps)
        f = L["wg"].shape[0]
        act = swiglu(t, L["wg"], L["wu"], L["wg"].shape[1], L["wu"].shape[1], xn, f, H, order)
        h = gemv_add(t, L["wd"], L["wd"].shape[1], act, h[0], H, f, order).reshape(1, -1)
    xn = rmsnorm(h, lnf, eps)
    logits = gemv(t, lm, lm.shape[1], xn, lm.shape[0], H, 1, order)[0]
    return h[0], (logits if with_logits else None), argmax(logits)


def _dq(t, w, k, chunk=16384):
    """Exact dequantized rows (float64), in row chunks to bound memory."""
    rb = w.shape[1]
    out = np.empty((w.shape[0], k), np.float64)
    for r0 in range(0, w.shape[0], chunk):
        out[r0:r0 + chunk] = dequant_rows(t, w[r0:r0 + chunk], k, rb)
    return out


def linear_stack_batch(layers, lm, lnf, h, t=Q4_K, eps=1e-6, rope_args=None):
    """linear_stack_token for a batch of tokens (h: [M, hidden]): the same steps with the exact
    dequantized weights and float64 accumulation (numpy matmul).  Returns (h, logits [M, vocab]).
    rope_args (positions [M], theta, head_dim, rows) as linear_stack_token."""
    h = np.array(h, np.float64, copy=True)
    H = h.shape[1]

    def norm(x, g):
        return x / np.sqrt(np.mean(x * x, axis=1, keepdims=True) + eps) * np.asarray(g, np.float64)
    for L in layers:
        xn = norm(h, L["ln1"])
        qkv = np.concatenate([xn @ _dq(t, L[n], H).T for n in ("wq", "wk", "wv")], axis=1) + L["bqkv"]
        if rope_args is not None:
            qkv = rope(qkv, *rope_args)
        qw = L["wq"].shape[0]
        h = h + qkv[:, :qw] @ _dq(t, L["wo"], qw).T
        xn = norm(h, L["ln2"])
        gv, uv = xn @ _dq(t, L["wg"], H).T, xn @ _dq(t, L["wu"], H).T
        h = h + (gv / (1 + np.exp(-gv)) * uv) @ _dq(t, L["wd"], L["wg"].shape[0]).T
    xn = norm(h, lnf)
    logits = np.concatenate([xn @ _dq(t, lm[r0:r0 + 16384], H).T for r0 in range(0, lm.shape[0], 16384)], axis=1)
    return h, logits


def greedy_decode(layers, lm, lnf, table, first_token, steps, t=Q4_K, emb_type=Q4_K, eps=1e-6, order=1,
                  rope=None):
    """Greedy loop: token -> quantized embedding row (quant_embedding_kernel, kernel.cu:2677-2693)
    -> linear stack -> argmax -> next token.  rope (theta, head_dim, rows): RoPE at position = step
    index.  Returns (tokens, per-step (best, runner-up) logit margins)."""
    H = lm.shape[1] // BLOCK[t][1] * BLOCK[t][0]
    tok, toks, margins = int(first_token), [], []
    for step in range(steps):
        h = embedding(emb_type, np.array([tok], np.int32), table, table.shape[1], H)[0]
        ra = None if rope is None else (step, *rope)
        _, logits, tok = linear_stack_token(layers, lm, lnf, h, t, eps, order, rope_args=ra)
        top2 = np.partition(logits, -2)[-2:]
        toks.append(tok)
        margins.append(float(top2[1] - top2[0]))
    return toks, margins


def f16_bits_to_f32(bits) -> np.ndarray:
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float32)


# ----------------------------------------------------------------------------
# The reference's own CUDA kernels (GPU only; built into _ref/ from the
# reference sources).  Arguments are raw device pointers (ints).
# ----------------------------------------------------------------------------
_ref = None


def ref_lib():
    global _ref
    if _ref is None:
        if not os.path.exists(REF_LIB_PATH):
            return None
        L = C.CDLL(REF_LIB_PATH)
        P, I, I64, SZ, F = C.c_void_p, C.c_int, C.c_int64, C.c_size_t, C.c_float
        sig = {
            "ref_set_stream": (I, [P]),
            "ref_last_error": (I, []),
            "ref_quant_gemv": (None, [I, P, SZ, P, P, I, I, I]),
            "ref_quant_gemv_add": (None, [I, P, SZ, P, P, I, I]),
            "ref_quant_matmul": (None, [I, P, SZ, P, P, I, I, I]),
            "ref_quant_swiglu": (None, [I, P, P, SZ, SZ, P, P, I, I]),
            "ref_quant_swiglu_indexed": (None, [I, P, P, SZ, SZ, SZ, SZ, P, P, P, I, I, I]),
            "ref_quant_down_ordered": (None, [I, P, SZ, SZ, P, P, P, P, I, I, I]),
            "ref_moe_router_topk": (None, [P, P, P, I, I, I, F]),
            "ref_quant_embedding": (None, [I, P, P, P, SZ, I, I]),
            "ref_argmax": (None, [P, I, P]),
            "ref_dequantize_q4k": (None, [P, P, I64]),
            "ref_dequantize_q80": (None, [P, P, I64]),
            "ref_dequantize_q50": (None, [P, P, I64]),
            "ref_dequantize_q6k": (None, [P, P, I64]),
            "ref_full_attention_attend": (None, [P, P, P, P, I, P, I, I, I, I, P]),
            "ref_full_attention_attend_batch": (None, [P, P, P, P, I, P, I, I, I, I, I, I]),
            "ref_quantize_q8_1": (None, [P, P, I, I, I]),
            "ref_quant_gemv_q8_1": (None, [I, P, SZ, P, P, I, I]),
            "ref_quant_matmul_q8_1": (None, [I, P, SZ, P, P, I, I, I]),
            "ref_quantize_q8_1_mmq": (None, [P, P, I, I, I]),
            "ref_quant_matmul_q8_1_mmq": (None, [I, P, SZ, P, P, I, I, I]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _ref = L
    return _ref
