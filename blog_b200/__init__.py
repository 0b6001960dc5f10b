"""blog_b200 -- B200-native block-quantized linear path of the local-llm engine.

The product is the native library ``lib/libqlinear_b200.so`` (CUDA, sm_100a)
with the C ABI declared in ``include/qlinear_b200.h``.  This module binds that
ABI through ctypes for Python callers (tests, benchmarks).  It mirrors the
reference's launch layer (AI/codes/local-llm/src/backend/cuda/ops/kernel.cuh):
same function names without the ``launch_`` prefix, same argument order and
meaning, device pointers passed as integers (e.g. ``tensor.data_ptr()``).

There is no CPU fallback: if the library is missing the import of ``lib()``
raises, and every call returns the library's status, raised as ``QLError``.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libqlinear_b200.so")
HEADER = os.path.join(os.path.dirname(PKG), "include", "qlinear_b200.h")

# GGML type codes (reference src/tensor/TensorCommon.h:15-33)
F32, F16, Q4_0, Q5_0, Q8_0, Q4_K, Q6_K = 0, 1, 2, 6, 8, 12, 14
BLOCK = {Q4_0: (32, 18), Q5_0: (32, 22), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}
QL_OK, QL_EINVAL, QL_ECUDA, QL_EDEVICE = 0, 1, 2, 3
PATH_AUTO, PATH_GEMV, PATH_TENSOR = 0, 1, 2


class QLError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"qlinear status {status}: {msg}")
        self.status = status


def row_bytes(t: int, k: int) -> int:
    be, bb = BLOCK[t]
    if k % be:
        raise ValueError(f"in_dim {k} is not a multiple of {be}")
    return k // be * bb


P, I, I32, I64, U64, SZ, F = C.c_void_p, C.c_int, C.c_int32, C.c_int64, C.c_uint64, C.c_size_t, C.c_float
SIGNATURES = {
    "ql_set_stream": (I, [P]),
    "ql_get_stream": (P, []),
    "ql_init": (I, [I]),
    "ql_last_error": (C.c_char_p, []),
    "ql_check_device": (I, []),
    "ql_quant_gemv": (I, [I32, P, SZ, P, P, I, I, I]),
    "ql_quant_gemv_add": (I, [I32, P, SZ, P, P, I, I]),
    "ql_quant_matmul": (I, [I32, P, SZ, P, P, I, I, I]),
    "ql_quant_swiglu": (I, [I32, P, P, SZ, SZ, P, P, I, I]),
    "ql_quant_swiglu_indexed": (I, [I32, P, P, SZ, SZ, SZ, SZ, P, P, P, I, I, I]),
    "ql_quant_down_f32_indexed_accum_ordered": (I, [I32, P, SZ, SZ, P, P, P, P, I, I, I]),
    "ql_moe_router_topk": (I, [P, P, P, I, I, I, F]),
    "ql_full_attention_attend": (I, [P, P, P, P, I, P, I, I, I, I, P]),
    "ql_q8_1_row_bytes": (SZ, [I]),
    "ql_quantize_q8_1": (I, [P, P, I, I, I]),
    "ql_quant_gemv_q8_1": (I, [I32, P, SZ, P, P, I, I]),
    "ql_quant_matmul_q8_1": (I, [I32, P, SZ, P, P, I, I, I]),
    "ql_q8_1_mmq_row_bytes": (SZ, [I]),
    "ql_quantize_q8_1_mmq": (I, [P, P, I, I, I]),
    "ql_quant_matmul_q8_1_mmq": (I, [I32, P, SZ, P, P, I, I, I]),
    "ql_full_attention_attend_batch": (I, [P, P, P, P, I, P, I, I, I, I, I, I]),
    "ql_moe_swiglu_grouped": (I, [I32, P, P, SZ, SZ, SZ, SZ, P, I64, P, I, I, P, I, I, I, I]),
    "ql_moe_down_grouped_accum_ordered": (I, [I32, P, SZ, SZ, P, P, I, I, P, P, I64, I, I, I, I]),
    "ql_quant_embedding": (I, [I32, P, P, P, SZ, I, I]),
    "ql_dequantize_to_f16": (I, [I32, P, P, I64]),
    "ql_dequantize_q4k_to_f16": (I, [P, P, I64]),
    "ql_dequantize_q80_to_f16": (I, [P, P, I64]),
    "ql_dequantize_q50_to_f16": (I, [P, P, I64]),
    "ql_dequantize_q6k_to_f16": (I, [P, P, I64]),
    "ql_dequantize_q40_to_f16": (I, [P, P, I64]),
    "ql_argmax": (I, [P, I, P]),
    "ql_argmax_noalloc": (I, [P, I, P]),
    "ql_quant_gemv_ex": (I, [I32, P, SZ, P, I64, P, I64, I, I, I, P, F, P, I]),
    "ql_quant_swiglu_ex": (I, [I32, P, P, SZ, SZ, P, I64, P, I64, I, I, I, P, F]),
    "ql_quant_gemv_stacked_ex": (I, [I32, I, P, P, P, P, I64, P, I64, I, I, P, F, P]),
    "ql_quant_matmul_ex": (I, [I32, P, SZ, P, I64, P, I64, I, I, I, P, F, P, I, I]),
    "ql_reserve_prefill": (I, [I, I]),
    "ql_quant_gemv_argmax_ex": (I, [I32, P, SZ, P, I64, P, I64, I, I, I, P, F, I, P, P]),
    "ql_gemv_chain_create": (I, [P, I, C.POINTER(C.c_void_p)]),
    "ql_gemv_chain_exchange_bytes": (SZ, [P, I, I]),
    "ql_gemv_chain_create_tp": (I, [P, I, I, I, P, C.POINTER(C.c_void_p)]),
    "ql_gemv_chain_create_batch": (I, [P, I, I, C.POINTER(C.c_void_p)]),
    "ql_ipc_alloc": (I, [SZ, C.POINTER(C.c_void_p), C.c_char_p]),
    "ql_ipc_free": (I, [P]),
    "ql_ipc_open": (I, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "ql_ipc_close": (I, [P]),
    "ql_gemv_chain_run": (I, [P]),
    "ql_gemv_chain_destroy": (I, [P]),
    "ql_comm_bytes": (SZ, [I, I, I]),
    "ql_comm_alloc": (I, [I, I, I, C.POINTER(C.c_void_p), C.c_char_p]),
    "ql_comm_create": (I, [I, I, I, I, P, C.c_char_p, C.POINTER(C.c_void_p)]),
    "ql_comm_destroy": (I, [P]),
    "ql_allreduce_f32": (I, [P, P, I, I]),
    "ql_comm_step": (I, [P]),
    "ql_rms_norm_f32": (I, [P, P, P, I, I, F]),
    "ql_synth_quantized": (I, [I32, U64, I64, I, F, P]),
    "ql_gguf_open": (I, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "ql_gguf_close": (I, [P]),
    "ql_gguf_version": (I, [P]),
    "ql_gguf_tensor_count": (I64, [P]),
    "ql_gguf_find_tensor": (I64, [P, C.c_char_p]),
    "ql_gguf_tensor_info": (I, [P, I64, C.POINTER(C.c_char_p), C.POINTER(C.c_int32), C.POINTER(C.c_int32), P,
                                C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)]),
    "ql_gguf_metadata_type": (I, [P, C.c_char_p]),
    "ql_gguf_metadata_int": (I, [P, C.c_char_p, C.POINTER(C.c_int64)]),
    "ql_gguf_metadata_float": (I, [P, C.c_char_p, C.POINTER(C.c_double)]),
    "ql_gguf_metadata_string": (I, [P, C.c_char_p, C.POINTER(C.c_char_p)]),
    "ql_gguf_metadata_array_len": (I64, [P, C.c_char_p]),
    "ql_gguf_metadata_array_int": (I, [P, C.c_char_p, I64, C.POINTER(C.c_int64)]),
    "ql_gguf_metadata_array_float": (I, [P, C.c_char_p, I64, C.POINTER(C.c_double)]),
    "ql_gguf_metadata_array_string": (I, [P, C.c_char_p, I64, C.POINTER(C.c_char_p)]),
    "ql_gguf_validate": (I, [P]),
    "ql_weight_upload": (I, [P, SZ, I64, I64, SZ, SZ, P]),
    "ql_row_bytes": (SZ, [I32, I]),
    "ql_last_launch_count": (I, []),
}

_lib = None


def lib() -> C.CDLL:
    """The loaded native library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m blog_b200.build` (there is no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _check(status: int) -> None:
    if status != QL_OK:
        raise QLError(status, lib().ql_last_error().decode(errors="replace"))


def _call(name: str, *args) -> None:
    _check(getattr(lib(), name)(*args))


# ---- thin wrappers, names follow the reference's launch_* functions ----------
def set_stream(stream_handle: int | None) -> None:
    _call("ql_set_stream", stream_handle or None)


def init(device: int = 0) -> None:
    _call("ql_init", device)


def check_device() -> None:
    _call("ql_check_device")


def quant_gemv(t, weight, rb, x, y, out_dim, in_dim, m):
    _call("ql_quant_gemv", t, weight, rb, x, y, out_dim, in_dim, m)


def quant_gemv_add(t, weight, rb, x, y, out_dim, in_dim):
    _call("ql_quant_gemv_add", t, weight, rb, x, y, out_dim, in_dim)


def quant_matmul(t, weight, rb, x, y, out_dim, in_dim, m):
    _call("ql_quant_matmul", t, weight, rb, x, y, out_dim, in_dim, m)


def quant_matmul_ex(t, w, rb, x, x_stride, y, y_stride, out_dim, in_dim, m, gamma=None, eps=0.0, bias=None,
                    accumulate=False, path=PATH_AUTO):
    """Prefill GEMM; path PATH_TENSOR forces the tcgen05 kernel, PATH_GEMV the streaming engine."""
    _call("ql_quant_matmul_ex", t, w, rb, x, x_stride, y, y_stride, out_dim, in_dim, m, gamma, eps, bias,
          1 if accumulate else 0, path)


IPC_HANDLE_BYTES = 64


class Comm:
    """Peer-memory all-reduce communicator of one rank (see include/qlinear_b200.h).

    `exchange_handles(own_handle) -> list of handles in rank order` is supplied by the
    caller (e.g. torch.distributed.all_gather_object); the library stays host-agnostic."""

    def __init__(self, rank, world, max_floats, slots, exchange_handles):
        ptr = C.c_void_p()
        hbuf = C.create_string_buffer(IPC_HANDLE_BYTES)
        _call("ql_comm_alloc", world, max_floats, slots, C.byref(ptr), hbuf)
        handles = exchange_handles(bytes(hbuf.raw))
        if len(handles) != world or any(len(h) != IPC_HANDLE_BYTES for h in handles):
            raise ValueError("exchange_handles must return one 64-byte handle per rank")
        comm = C.c_void_p()
        _call("ql_comm_create", rank, world, max_floats, slots, ptr, b"".join(handles), C.byref(comm))
        self.handle, self.max_floats, self.slots = comm, max_floats, slots

    def allreduce(self, buf_ptr, n, slot):
        _call("ql_allreduce_f32", self.handle, buf_ptr, n, slot)

    def step(self):
        _call("ql_comm_step", self.handle)

    def close(self):
        if self.handle:
            _call("ql_comm_destroy", self.handle)
            self.handle = None


def quant_gemv_argmax_ex(t, w, rb, x, x_stride, logits, logits_stride, out_dim, in_dim, m, gamma=None, eps=0.0,
                         index_offset=0, out_idx=None, out_key=None):
    """Fused LM head + greedy argmax (see include/qlinear_b200.h)."""
    _call("ql_quant_gemv_argmax_ex", t, w, rb, x, x_stride, logits, logits_stride, out_dim, in_dim, m, gamma, eps,
          index_offset, out_idx, out_key)


OP_STORE, OP_ADD, OP_SWIGLU, OP_MLP = 0, 1, 2, 3


class ChainOp(C.Structure):
    """ql_chain_op (include/qlinear_b200.h)."""
    _fields_ = [("kind", C.c_int32), ("quant_type", C.c_int32), ("nsrc", C.c_int32),
                ("w", C.c_void_p * 3), ("row_bytes", C.c_size_t * 3), ("rows", C.c_int32 * 3),
                ("in_dim", C.c_int32), ("x", C.c_void_p), ("gamma", C.c_void_p), ("eps", C.c_float),
                ("bias", C.c_void_p), ("y", C.c_void_p), ("argmax_idx", C.c_void_p), ("argmax_offset", C.c_int32),
                ("reduce", C.c_int32), ("x_stride", C.c_int64), ("y_stride", C.c_int64),
                ("rope_pos", C.c_void_p), ("rope_theta", C.c_float), ("rope_rows", C.c_int32),
                ("head_dim", C.c_int32)]


def chain_op(kind, weights, row_bytes, rows, in_dim, x, y, gamma=None, eps=0.0, bias=None, argmax_idx=None,
             argmax_offset=0, quant_type=Q4_K, reduce=False, x_stride=0, y_stride=0, rope_pos=None, rope_theta=0.0,
             rope_rows=0, head_dim=0):
    op = ChainOp()
    op.kind, op.quant_type, op.nsrc, op.in_dim = kind, quant_type, len(weights), in_dim
    for i, (w, rb, r) in enumerate(zip(weights, row_bytes, rows)):
        op.w[i], op.row_bytes[i], op.rows[i] = w, rb, r
    op.x, op.y, op.gamma, op.eps, op.bias = x, y, gamma, eps, bias
    op.argmax_idx, op.argmax_offset, op.reduce = argmax_idx, argmax_offset, 1 if reduce else 0
    op.x_stride, op.y_stride = x_stride, y_stride
    op.rope_pos, op.rope_theta, op.rope_rows, op.head_dim = rope_pos, rope_theta, rope_rows, head_dim
    return op


class GemvChain:
    """A list of single-token GEMV ops run as one persistent launch (ql_gemv_chain_*).

    Tensor parallel: pass rank, world and `exchange_handles(own_handle) -> handles in rank
    order` (any host channel, e.g. torch.distributed.all_gather_object); ops with reduce=True
    then sum their partials over ranks inside the kernel through peer memory."""

    def __init__(self, ops, rank=0, world=1, exchange_handles=None, tokens=None):
        """tokens=None: the one-token chain; tokens=M (1..32): the batched chain over M tokens."""
        arr = (ChainOp * len(ops))(*ops)
        h = C.c_void_p()
        self.own, self.mapped = None, []
        if tokens is not None:
            _call("ql_gemv_chain_create_batch", C.cast(arr, C.c_void_p), len(ops), tokens, C.byref(h))
        elif world == 1:
            _call("ql_gemv_chain_create", C.cast(arr, C.c_void_p), len(ops), C.byref(h))
        else:
            nbytes = lib().ql_gemv_chain_exchange_bytes(C.cast(arr, C.c_void_p), len(ops), world)
            own = C.c_void_p()
            hb = C.create_string_buffer(IPC_HANDLE_BYTES)
            _call("ql_ipc_alloc", max(nbytes, 256), C.byref(own), hb)
            self.own = own
            handles = exchange_handles(bytes(hb.raw))
            ptrs = (C.c_void_p * world)()
            for r, hr in enumerate(handles):
                if r == rank:
                    ptrs[r] = own.value
                else:
                    m = C.c_void_p()
                    _call("ql_ipc_open", hr, C.byref(m))
                    self.mapped.append(m)
                    ptrs[r] = m.value
            _call("ql_gemv_chain_create_tp", C.cast(arr, C.c_void_p), len(ops), rank, world, C.cast(ptrs, C.c_void_p),
                  C.byref(h))
        self.handle = h

    def run(self):
        _call("ql_gemv_chain_run", self.handle)

    def close(self):
        """Release the chain; with world > 1 call it on every rank after a host barrier."""
        if self.handle:
            _call("ql_gemv_chain_destroy", self.handle)
            self.handle = None
        for m in self.mapped:
            _call("ql_ipc_close", m)
        self.mapped = []
        if self.own is not None:
            _call("ql_ipc_free", self.own)
            self.own = None


def reserve_prefill(max_tokens, max_in_dim):
    _call("ql_reserve_prefill", max_tokens, max_in_dim)


def quant_swiglu(t, gw, uw, grb, urb, x, act, ffn_dim, in_dim):
    _call("ql_quant_swiglu", t, gw, uw, grb, urb, x, act, ffn_dim, in_dim)


def quant_swiglu_indexed(t, gw, uw, geb, ueb, grb, urb, x, ids, act, k, ffn_dim, in_dim):
    _call("ql_quant_swiglu_indexed", t, gw, uw, geb, ueb, grb, urb, x, ids, act, k, ffn_dim, in_dim)


def quant_down_f32_indexed_accum_ordered(t, dw, deb, drb, act, ids, rw, out, k, hidden, ffn_dim):
    _call("ql_quant_down_f32_indexed_accum_ordered", t, dw, deb, drb, act, ids, rw, out, k, hidden, ffn_dim)


def moe_router_topk(logits, idx, w, tokens, n_experts, k, scale):
    _call("ql_moe_router_topk", logits, idx, w, tokens, n_experts, k, scale)


def q8_1_row_bytes(in_dim):
    return lib().ql_q8_1_row_bytes(in_dim)


def quantize_q8_1(x, xq, in_dim, m, store_raw_sum=False):
    _call("ql_quantize_q8_1", x, xq, in_dim, m, int(store_raw_sum))


def quant_gemv_q8_1(t, w, rb, xq, y, out_dim, in_dim):
    _call("ql_quant_gemv_q8_1", t, w, rb, xq, y, out_dim, in_dim)


def quant_matmul_q8_1(t, w, rb, xq, y, out_dim, in_dim, m):
    _call("ql_quant_matmul_q8_1", t, w, rb, xq, y, out_dim, in_dim, m)


def q8_1_mmq_row_bytes(in_dim):
    return lib().ql_q8_1_mmq_row_bytes(in_dim)


def quantize_q8_1_mmq(x, xq, in_dim, m, store_raw_sum=False):
    _call("ql_quantize_q8_1_mmq", x, xq, in_dim, m, int(store_raw_sum))


def quant_matmul_q8_1_mmq(t, w, rb, xq, y, out_dim, in_dim, m):
    _call("ql_quant_matmul_q8_1_mmq", t, w, rb, xq, y, out_dim, in_dim, m)


def full_attention_attend(q, gate, kc, vc, kv_bf16, attn, n_heads, kv_heads, head_dim, max_seq_len, pos_dev):
    _call("ql_full_attention_attend", q, gate, kc, vc, int(kv_bf16), attn, n_heads, kv_heads, head_dim, max_seq_len,
          pos_dev)


def full_attention_attend_batch(q, gate, kc, vc, kv_bf16, attn, tokens, n_heads, kv_heads, head_dim, max_seq_len,
                                start_pos):
    _call("ql_full_attention_attend_batch", q, gate, kc, vc, int(kv_bf16), attn, tokens, n_heads, kv_heads, head_dim,
          max_seq_len, start_pos)


def moe_swiglu_grouped(t, gw, uw, geb, ueb, grb, urb, x, x_stride, ids, expert_begin, n_experts, act, tokens, k,
                       ffn_dim, in_dim):
    _call("ql_moe_swiglu_grouped", t, gw, uw, geb, ueb, grb, urb, x, x_stride, ids, expert_begin, n_experts, act,
          tokens, k, ffn_dim, in_dim)


def moe_down_grouped_accum_ordered(t, dw, deb, drb, act, ids, expert_begin, n_experts, rw, out, out_stride, tokens,
                                   k, hidden, ffn_dim):
    _call("ql_moe_down_grouped_accum_ordered", t, dw, deb, drb, act, ids, expert_begin, n_experts, rw, out,
          out_stride, tokens, k, hidden, ffn_dim)


def quant_embedding(t, ids, out, table, rb, hidden, n):
    _call("ql_quant_embedding", t, ids, out, table, rb, hidden, n)


def dequantize_to_f16(t, src, out, n):
    _call("ql_dequantize_to_f16", t, src, out, n)


def argmax(logits, n, out_idx):
    _call("ql_argmax", logits, n, out_idx)


def argmax_noalloc(logits, n, out_idx):
    """ql_argmax without device allocation (fixed in-library scratch; see the header)."""
    _call("ql_argmax_noalloc", logits, n, out_idx)


def quant_gemv_ex(t, w, rb, x, x_stride, y, y_stride, out_dim, in_dim, m, gamma=None, eps=0.0, bias=None,
                  accumulate=False):
    _call("ql_quant_gemv_ex", t, w, rb, x, x_stride, y, y_stride, out_dim, in_dim, m, gamma, eps, bias,
          1 if accumulate else 0)


def quant_gemv_stacked_ex(t, weights, row_bytes_list, rows, x, x_stride, y, y_stride, in_dim, m, gamma=None,
                          eps=0.0, bias=None):
    """Stacked projections (e.g. fused q/k/v): weights, row_bytes_list, rows are Python sequences (<= 3)."""
    n = len(weights)
    W = (C.c_void_p * n)(*weights)
    RB = (C.c_size_t * n)(*row_bytes_list)
    R = (C.c_int * n)(*rows)
    _call("ql_quant_gemv_stacked_ex", t, n, C.cast(W, C.c_void_p), C.cast(RB, C.c_void_p), C.cast(R, C.c_void_p), x,
          x_stride, y, y_stride, in_dim, m, gamma, eps, bias)


def quant_swiglu_ex(t, gw, uw, grb, urb, x, x_stride, act, act_stride, ffn_dim, in_dim, m, gamma=None, eps=0.0):
    _call("ql_quant_swiglu_ex", t, gw, uw, grb, urb, x, x_stride, act, act_stride, ffn_dim, in_dim, m, gamma, eps)


def rms_norm_f32(x, y, gamma, rows, hidden, eps):
    _call("ql_rms_norm_f32", x, y, gamma, rows, hidden, eps)


def synth_quantized(t, seed, rows, in_dim, std, dst):
    _call("ql_synth_quantized", t, seed, rows, in_dim, std, dst)


def weight_upload(host_ptr, row_bytes, row0, nrows, byte0, nbytes_per_row, dst):
    """Host GGUF rows (a matrix or a tensor-parallel shard of it) to device memory (ql_weight_upload)."""
    _call("ql_weight_upload", host_ptr, row_bytes, row0, nrows, byte0, nbytes_per_row, dst)


def last_launch_count() -> int:
    return int(lib().ql_last_launch_count())
