"""CPU: the GGUF loader (ql_gguf_* over the native library) and the synthetic-model writer
(blog_b200.gguf), cross-checked in both directions against the third-party gguf-py package
(0.19.0, present in this environment; the reference's own parser, GgufFile.cpp:152-250, needs
its engine's build and a model file, which are not available here).

Covered: header/metadata/tensor-table parsing, dims reversed to outermost-first, data offsets
after alignment (default 32 and general.alignment), block-trait byte sizes, every metadata
value type incl. arrays, MF::validate's container rules with Q4_0 admitted, and malformed
files rejected with QL_EINVAL instead of a crash."""
import os
import struct

import numpy as np
import pytest

import blog_b200 as Q
import blog_b200.gguf as G
import oracle as O

gguf = pytest.importorskip("gguf")


def _tensors():
    rng = np.random.default_rng(0)
    q4k = O.quantize(O.Q4_K, O.randn(1, 64 * 512, 0.02).reshape(64, 512))
    q40 = O.quantize(O.Q4_0, O.randn(2, 48 * 96, 0.02).reshape(48, 96))
    q80 = O.quantize(O.Q8_0, O.randn(3, 8 * 64, 0.02).reshape(8, 64))
    f32 = rng.standard_normal(96).astype(np.float32)
    return [("blk.0.attn_q.weight", 12, (64, 512), q4k), ("blk.0.ffn_down.weight", 2, (48, 96), q40),
            ("token_embd.weight", 8, (8, 64), q80), ("output_norm.weight", 0, (96,), f32)]


def test_writer_read_back_by_library_and_gguf_py(tmp_path):
    p = str(tmp_path / "m.gguf")
    meta = {"general.architecture": "qwen2", "qwen2.block_count": 2, "qwen2.rope.freq_base": 1e6,
            "tokenizer.ggml.tokens": ["<a>", "b", "c"], "qwen2.ints": [3, -1, 7], "flag": True,
            "neg": (G.I32, -5), "big": (G.U64, 2 ** 40), "f64": (G.F64, 0.125)}
    ts = _tensors()
    G.write_gguf(p, meta, ts)
    with G.GgufFile(p) as f:
        assert f.version == 3 and len(f) == len(ts)
        f.validate()  # Q4_0 admitted
        for name, t, shape, data in ts:
            n, tt, sh, buf = f.tensor(name)
            assert (n, tt, sh) == (name, t, shape)
            assert np.array_equal(buf, np.ascontiguousarray(data).view(np.uint8).ravel())
        assert f.metadata("general.architecture") == "qwen2"
        assert f.metadata("qwen2.block_count") == 2
        assert f.metadata("qwen2.rope.freq_base") == pytest.approx(1e6)
        assert f.metadata("tokenizer.ggml.tokens") == ["<a>", "b", "c"]
        assert f.metadata("qwen2.ints") == [3, -1, 7]
        assert f.metadata("flag") is True and f.metadata("neg") == -5 and f.metadata("big") == 2 ** 40
        assert f.metadata("f64") == 0.125 and f.metadata("missing") is None
        assert f.find("nope") == -1
    r = gguf.GGUFReader(p)  # the third-party reader agrees
    by = {t.name: t for t in r.tensors}
    for name, t, shape, data in ts:
        rt = by[name]
        assert int(rt.tensor_type) == t
        assert list(rt.shape) == list(reversed(shape))  # gguf-py reports dims innermost-first
        assert np.array_equal(np.asarray(rt.data).view(np.uint8).ravel(), np.ascontiguousarray(data).view(np.uint8).ravel())
    assert bytes(r.fields["general.architecture"].parts[-1]).decode() == "qwen2"


def test_library_reads_gguf_py_file(tmp_path):
    p = str(tmp_path / "w.gguf")
    w = gguf.GGUFWriter(p, "qwen2")
    w.add_block_count(3)
    w.add_string("custom.s", "hello")
    ts = _tensors()
    for name, t, shape, data in ts:
        raw = np.ascontiguousarray(data)
        if t == 0:
            w.add_tensor(name, raw)
        else:
            # gguf-py takes quantized tensors as their byte matrix [rows, row bytes]
            w.add_tensor(name, raw.view(np.uint8), raw_shape=raw.shape, raw_dtype=gguf.GGMLQuantizationType(t))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with G.GgufFile(p) as f:
        assert f.metadata("general.architecture") == "qwen2" and f.metadata("qwen2.block_count") == 3
        assert f.metadata("custom.s") == "hello"
        for name, t, shape, data in ts:
            n, tt, sh, buf = f.tensor(name)
            assert (tt, sh) == (t, shape)
            assert np.array_equal(buf, np.ascontiguousarray(data).view(np.uint8).ravel())
        f.validate()


def test_alignment_metadata_moves_the_data_section(tmp_path):
    p = str(tmp_path / "a.gguf")
    ts = _tensors()
    G.write_gguf(p, {"general.architecture": "x"}, ts, alignment=64)
    with G.GgufFile(p) as f:
        assert f.metadata("general.alignment") == 64
        for name, t, shape, data in ts:
            assert np.array_equal(f.tensor(name)[3], np.ascontiguousarray(data).view(np.uint8).ravel())


def _raw_file(path, tensors, version=3, magic=0x46554747):
    """A GGUF file with arbitrary tensor-table entries (name, dims innermost-first, type, offset)."""
    head = struct.pack("<IIQQ", magic, version, len(tensors), 0)
    table = b"".join(G._str(n) + struct.pack("<I", len(d)) + b"".join(struct.pack("<Q", x) for x in d) +
                     struct.pack("<IQ", t, off) for n, d, t, off in tensors)
    body = head + table
    body += b"\0" * ((-len(body)) % 32) + b"\x11" * 4096
    open(path, "wb").write(body)


@pytest.mark.parametrize("case,needle", [
    ("dup", "duplicate"), ("empty_name", "empty name"), ("zero_dim", "non-positive"), ("q5k", "unsupported"),
    ("none", "no tensors")])
def test_validate_rejects(tmp_path, case, needle):
    p = str(tmp_path / "v.gguf")
    t = {"dup": [("a", [32], 8, 0), ("a", [32], 8, 64)], "empty_name": [("", [32], 8, 0)],
         "zero_dim": [("a", [32, 0], 8, 0)], "q5k": [("a", [256], 13, 0)], "none": []}[case]
    _raw_file(p, t)
    with G.GgufFile(p) as f:
        with pytest.raises(Q.QLError) as e:
            f.validate()
        assert needle in str(e.value)


@pytest.mark.parametrize("case", ["magic", "version", "truncated", "past_end", "block", "tiny"])
def test_malformed_files_rejected(tmp_path, case):
    p = str(tmp_path / "bad.gguf")
    if case == "magic":
        _raw_file(p, [("a", [32], 8, 0)], magic=0x12345678)
    elif case == "version":
        _raw_file(p, [("a", [32], 8, 0)], version=1)
    elif case == "past_end":
        _raw_file(p, [("a", [32 * 1000], 8, 0)])  # 34 KB of data in a 4 KB section
    elif case == "block":
        _raw_file(p, [("a", [33], 8, 0)])  # not a multiple of the Q8_0 block
    elif case == "tiny":
        open(p, "wb").write(b"GGUF")
    else:
        G.write_gguf(p, {"general.architecture": "x"}, _tensors())
        data = open(p, "rb").read()
        open(p, "wb").write(data[:100])
    with pytest.raises(Q.QLError):
        G.GgufFile(p)
