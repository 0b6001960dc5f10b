"""GGUF files for the quantized linear path: a v3 writer for synthetic models and a reader
over the library's native loader (ql_gguf_* in include/qlinear_b200.h).

The reference engine consumes GGUF files through GgufFile (AI/codes/local-llm/src/format/
gguf/GgufFile.cpp:152-250).  The writer produces the container that loader (and this
library's) reads: header {magic "GGUF", version 3, tensor count, metadata count}, the
metadata key/value table, the tensor table {name, dims innermost-first, ggml type, offset
relative to the data section}, padding to general.alignment (32), then each tensor's bytes
at an aligned offset.  Quantized tensors are passed as their raw block bytes.
"""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np

from . import QLError, lib

# GGUF metadata value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?", U64: "<Q",
           I64: "<q", F64: "<d"}
# ggml block traits: type -> (elements, bytes) per block
BLOCK = {0: (1, 4), 1: (1, 2), 30: (1, 2), 2: (32, 18), 6: (32, 22), 8: (32, 34), 12: (256, 144), 14: (256, 210)}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype == STRING:
        return _str(v)
    if vtype == ARRAY:
        etype, items = v
        out = struct.pack("<IQ", etype, len(items))
        return out + b"".join(_value(etype, x) for x in items)
    return struct.pack(_SCALAR[vtype], v)


def _guess(v):
    if isinstance(v, tuple) and len(v) == 2 and isinstance(v[0], int) and v[0] in _SCALAR.keys() | {STRING}:
        return v  # explicit (type, value)
    if isinstance(v, bool):
        return BOOL, v
    if isinstance(v, int):
        return (I64 if v < 0 else U32 if v < 2 ** 32 else U64), v
    if isinstance(v, float):
        return F32, v
    if isinstance(v, str):
        return STRING, v
    if isinstance(v, (list, tuple)):
        if all(isinstance(x, str) for x in v):
            return ARRAY, (STRING, list(v))
        if all(isinstance(x, float) for x in v):
            return ARRAY, (F32, list(v))
        return ARRAY, (I32, [int(x) for x in v])
    raise TypeError(f"cannot encode metadata value {v!r}")


def write_gguf(path: str, metadata: dict, tensors, alignment: int = 32) -> None:
    """Write a GGUF v3 file.  metadata: key -> value (int, float, bool, str, list, or an explicit
    (gguf_type, value)); tensors: iterable of (name, ggml_type, shape outermost-first, raw bytes)."""
    tensors = list(tensors)
    meta = dict(metadata)
    if alignment != 32:
        meta.setdefault("general.alignment", (U32, alignment))
    head = struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(meta))
    kv = b"".join(_str(k) + struct.pack("<I", _guess(v)[0]) + _value(*_guess(v)) for k, v in meta.items())
    table, blobs, off = [], [], 0
    for name, t, shape, data in tensors:
        data = np.ascontiguousarray(data).view(np.uint8).tobytes()
        be, bb = BLOCK[t]
        n = int(np.prod(shape))
        if n % be or n // be * bb != len(data):
            raise ValueError(f"{name}: {len(data)} bytes do not hold {shape} of ggml type {t}")
        dims = list(reversed([int(d) for d in shape]))
        table.append(_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) +
                     struct.pack("<IQ", t, off))
        blobs.append(data)
        off += len(data)
        off += (-off) % alignment
    header = head + kv + b"".join(table)
    with open(path, "wb") as f:
        f.write(header)
        f.write(b"\0" * ((-len(header)) % alignment))
        for blob in blobs:
            f.write(blob)
            f.write(b"\0" * ((-len(blob)) % alignment))


class GgufFile:
    """A GGUF file opened by the library's loader (read-only mapping)."""

    def __init__(self, path: str):
        h = C.c_void_p()
        st = lib().ql_gguf_open(path.encode(), C.byref(h))
        if st != 0:
            raise QLError(st, lib().ql_last_error().decode(errors="replace"))
        self.h = h

    def close(self):
        if self.h:
            lib().ql_gguf_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def version(self) -> int:
        return int(lib().ql_gguf_version(self.h))

    def __len__(self):
        return int(lib().ql_gguf_tensor_count(self.h))

    def find(self, name: str) -> int:
        return int(lib().ql_gguf_find_tensor(self.h, name.encode()))

    def tensor(self, i_or_name):
        """(name, ggml type, shape outermost-first, uint8 array viewing the mapped bytes)."""
        i = self.find(i_or_name) if isinstance(i_or_name, str) else int(i_or_name)
        name, t, nd = C.c_char_p(), C.c_int32(), C.c_int32()
        shape = (C.c_int64 * 8)()
        data, nbytes = C.c_void_p(), C.c_size_t()
        st = lib().ql_gguf_tensor_info(self.h, i, C.byref(name), C.byref(t), C.byref(nd), shape, C.byref(data),
                                       C.byref(nbytes))
        if st != 0:
            raise QLError(st, lib().ql_last_error().decode(errors="replace"))
        buf = (C.c_uint8 * nbytes.value).from_address(data.value) if nbytes.value else (C.c_uint8 * 0)()
        return name.value.decode(), t.value, tuple(shape[d] for d in range(nd.value)), np.frombuffer(buf, np.uint8)

    def metadata(self, key: str):
        """The value of a metadata key (None when absent)."""
        L, k = lib(), key.encode()
        vt = L.ql_gguf_metadata_type(self.h, k)
        if vt < 0:
            return None
        if vt == STRING:
            out = C.c_char_p()
            L.ql_gguf_metadata_string(self.h, k, C.byref(out))
            return out.value.decode()
        if vt == ARRAY:
            n = L.ql_gguf_metadata_array_len(self.h, k)
            vals = []
            for i in range(n):
                s, iv, fv = C.c_char_p(), C.c_int64(), C.c_double()
                if L.ql_gguf_metadata_array_string(self.h, k, i, C.byref(s)) == 0:
                    vals.append(s.value.decode())
                elif L.ql_gguf_metadata_array_int(self.h, k, i, C.byref(iv)) == 0:
                    vals.append(iv.value)
                elif L.ql_gguf_metadata_array_float(self.h, k, i, C.byref(fv)) == 0:
                    vals.append(fv.value)
            return vals
        if vt in (F32, F64):
            out = C.c_double()
            L.ql_gguf_metadata_float(self.h, k, C.byref(out))
            return out.value
        out = C.c_int64()
        L.ql_gguf_metadata_int(self.h, k, C.byref(out))
        return bool(out.value) if vt == BOOL else out.value

    def validate(self) -> None:
        st = lib().ql_gguf_validate(self.h)
        if st != 0:
            raise QLError(st, lib().ql_last_error().decode(errors="replace"))


def upload_tensor(f: GgufFile, name: str, torch, device="cuda", rows=None, byte_range=None):
    """A tensor's raw bytes on the device through ql_weight_upload: the whole matrix, a row range
    (column-parallel shard) or a byte range of every row (row-parallel shard, whole blocks).
    Returns a uint8 tensor [rows, bytes per row] (1-D tensors: [1, nbytes])."""
    _, t, shape, buf = f.tensor(name)
    nrows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
    rb = len(buf) // nrows
    r0, r1 = rows if rows is not None else (0, nrows)
    b0, b1 = byte_range if byte_range is not None else (0, rb)
    dst = torch.empty((r1 - r0, b1 - b0), dtype=torch.uint8, device=device)
    host = np.ascontiguousarray(buf)  # the mapped file (pageable): the copy is synchronous
    from . import weight_upload
    weight_upload(host.ctypes.data, rb, r0, r1 - r0, b0, b1 - b0, dst.data_ptr())
    torch.cuda.synchronize()
    return dst
