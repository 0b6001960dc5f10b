"""GGUF end to end: a synthetic Qwen2-architecture model written to a GGUF v3 file (llama.cpp
tensor names, Q4_K matrices, F32 norms and biases), opened and validated by the library's loader,
uploaded with ql_weight_upload, then decoded greedily by the one-token chain (embedding -> q/k/v
with RMSNorm, bias and RoPE -> o + residual -> fused MLP -> LM head + argmax).  The oracle decodes
from the same file's bytes (read by the third-party gguf-py reader, so the loader is checked too):
token ids must match for 8 steps."""
import numpy as np
import pytest

import blog_b200 as Q
import blog_b200.gguf as G
import oracle as O

pytestmark = pytest.mark.gpu
gguf = pytest.importorskip("gguf")
H, NH, NKV, HD, F, V, LAYERS, EPS, THETA = 2048, 16, 2, 128, 4096, 6000, 2, 1e-6, 1e6


def _write_model(path):
    rng = np.random.default_rng(3)
    q = lambda r, k, s: O.quantize(O.Q4_K, O.randn(s, r * k, 0.02).reshape(r, k))
    ts = [("token_embd.weight", 12, (V, H), q(V, H, 1)), ("output.weight", 12, (V, H), q(V, H, 2)),
          ("output_norm.weight", 0, (H,), (1 + 0.1 * rng.standard_normal(H)).astype(np.float32))]
    for l in range(LAYERS):
        p = f"blk.{l}."
        ts += [(p + "attn_q.weight", 12, (NH * HD, H), q(NH * HD, H, 10 * l + 3)),
               (p + "attn_k.weight", 12, (NKV * HD, H), q(NKV * HD, H, 10 * l + 4)),
               (p + "attn_v.weight", 12, (NKV * HD, H), q(NKV * HD, H, 10 * l + 5)),
               (p + "attn_output.weight", 12, (H, NH * HD), q(H, NH * HD, 10 * l + 6)),
               (p + "ffn_gate.weight", 12, (F, H), q(F, H, 10 * l + 7)),
               (p + "ffn_up.weight", 12, (F, H), q(F, H, 10 * l + 8)),
               (p + "ffn_down.weight", 12, (H, F), q(H, F, 10 * l + 9))]
        for n, size in (("attn_q.bias", NH * HD), ("attn_k.bias", NKV * HD), ("attn_v.bias", NKV * HD)):
            ts.append((p + n, 0, (size,), (0.01 * rng.standard_normal(size)).astype(np.float32)))
        for n in ("attn_norm.weight", "ffn_norm.weight"):
            ts.append((p + n, 0, (H,), (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)))
    meta = {"general.architecture": "qwen2", "qwen2.block_count": LAYERS, "qwen2.embedding_length": H,
            "qwen2.feed_forward_length": F, "qwen2.attention.head_count": NH, "qwen2.attention.head_count_kv": NKV,
            "qwen2.rope.freq_base": THETA, "qwen2.attention.layer_norm_rms_epsilon": EPS}
    G.write_gguf(path, meta, ts)


def test_gguf_model_loads_and_decodes_like_the_oracle(tmp_path):
    import torch
    torch.cuda.init()
    Q.init(0)
    Q.set_stream(torch.cuda.current_stream().cuda_stream)
    path = str(tmp_path / "qwen2-synthetic.gguf")
    _write_model(path)
    f = G.GgufFile(path)
    f.validate()
    assert f.metadata("general.architecture") == "qwen2" and f.metadata("qwen2.block_count") == LAYERS
    hd = f.metadata("qwen2.embedding_length") // f.metadata("qwen2.attention.head_count")
    theta, eps = f.metadata("qwen2.rope.freq_base"), f.metadata("qwen2.attention.layer_norm_rms_epsilon")
    up = lambda n: G.upload_tensor(f, n, torch)
    vec = lambda n: up(n).view(torch.float32).reshape(-1)
    rb = lambda k: Q.row_bytes(Q.Q4_K, k)
    D = []
    for l in range(LAYERS):
        p = f"blk.{l}."
        D.append({"wq": up(p + "attn_q.weight"), "wk": up(p + "attn_k.weight"), "wv": up(p + "attn_v.weight"),
                  "wo": up(p + "attn_output.weight"), "wg": up(p + "ffn_gate.weight"), "wu": up(p + "ffn_up.weight"),
                  "wd": up(p + "ffn_down.weight"), "ln1": vec(p + "attn_norm.weight"), "ln2": vec(p + "ffn_norm.weight"),
                  "b": torch.cat([vec(p + "attn_q.bias"), vec(p + "attn_k.bias"), vec(p + "attn_v.bias")])})
    table, lm, lnf = up("token_embd.weight"), up("output.weight"), vec("output_norm.weight")
    qw, kv = NH * hd, NKV * hd
    b = {"h": torch.zeros(H, device="cuda"), "qkv": torch.zeros(qw + 2 * kv, device="cuda"),
         "logits": torch.zeros(V, device="cuda"), "tok": torch.zeros(1, dtype=torch.int32, device="cuda"),
         "pos": torch.zeros(1, dtype=torch.int32, device="cuda")}
    hp, ops = b["h"].data_ptr(), []
    for L in D:
        ops.append(Q.chain_op(Q.OP_STORE, [L["wq"].data_ptr(), L["wk"].data_ptr(), L["wv"].data_ptr()], [rb(H)] * 3,
                              [qw, kv, kv], H, hp, b["qkv"].data_ptr(), L["ln1"].data_ptr(), eps, L["b"].data_ptr(),
                              rope_pos=b["pos"].data_ptr(), rope_theta=theta, rope_rows=qw + kv, head_dim=hd))
        ops.append(Q.chain_op(Q.OP_ADD, [L["wo"].data_ptr()], [rb(qw)], [H], qw, b["qkv"].data_ptr(), hp))
        ops.append(Q.chain_op(Q.OP_MLP, [L["wg"].data_ptr(), L["wu"].data_ptr(), L["wd"].data_ptr()],
                              [rb(H), rb(H), rb(F)], [F, F, H], H, hp, hp, L["ln2"].data_ptr(), eps))
    ops.append(Q.chain_op(Q.OP_STORE, [lm.data_ptr()], [rb(H)], [V], H, hp, b["logits"].data_ptr(), lnf.data_ptr(),
                          eps, argmax_idx=b["tok"].data_ptr()))
    chain = Q.GemvChain(ops)
    steps, first = 8, 123
    hist = torch.zeros(steps, dtype=torch.int32, device="cuda")
    b["tok"].fill_(first)
    try:
        for i in range(steps):
            b["pos"].fill_(i)
            Q.quant_embedding(Q.Q4_K, b["tok"].data_ptr(), hp, table.data_ptr(), rb(H), H, 1)
            chain.run()
            hist[i:i + 1].copy_(b["tok"])
        torch.cuda.synchronize()
        got = [int(x) for x in hist.cpu()]
        Q.check_device()
    finally:
        chain.close()
        f.close()
    # the oracle reads the same file through gguf-py
    r = gguf.GGUFReader(path)
    T = {t.name: np.asarray(t.data) for t in r.tensors}
    mat = lambda n: T[n].view(np.uint8).reshape(T[n].shape[0], -1)
    layers = [{"wq": mat(f"blk.{l}.attn_q.weight"), "wk": mat(f"blk.{l}.attn_k.weight"),
               "wv": mat(f"blk.{l}.attn_v.weight"), "wo": mat(f"blk.{l}.attn_output.weight"),
               "wg": mat(f"blk.{l}.ffn_gate.weight"), "wu": mat(f"blk.{l}.ffn_up.weight"),
               "wd": mat(f"blk.{l}.ffn_down.weight"), "ln1": T[f"blk.{l}.attn_norm.weight"],
               "ln2": T[f"blk.{l}.ffn_norm.weight"],
               "bqkv": np.concatenate([T[f"blk.{l}.attn_q.bias"], T[f"blk.{l}.attn_k.bias"],
                                       T[f"blk.{l}.attn_v.bias"]])} for l in range(LAYERS)]
    want, margins = O.greedy_decode(layers, mat("output.weight"), T["output_norm.weight"], mat("token_embd.weight"),
                                    first, steps, eps=eps, rope=(theta, hd, qw + kv))
    print(f"GGUF model greedy tokens {got} (oracle {want}), smallest margin {min(margins):.3e}")
    assert got == want
