"""Minimal GGUF v2/v3 writer for the tests (test infrastructure only).

Layout (little-endian), as the reference reader parses it
(Qwen35Sharp.Gguf/GgufFile.cs:110-172): magic "GGUF", u32 version, u64 tensor
count, u64 metadata count; per metadata entry a string key (u64 length +
bytes), an i32 value type and the value (arrays: i32 element type, u64
count, elements); per tensor a string name, u32 dim count, i64 dims (dim 0
innermost), i32 ggml type, u64 offset into the data section; the data
section starts at the next multiple of general.alignment (default 32).
"""

from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
        I64: "<q", F64: "<d"}
F32_TYPE = 0  # ggml type id of an f32 tensor


def gstr(s: str | bytes) -> bytes:
    b = s.encode() if isinstance(s, str) else s
    return struct.pack("<Q", len(b)) + b


def scalar(t: int, v) -> bytes:
    if t == STRING:
        return gstr(v)
    return struct.pack(_FMT[t], v)


def value(t: int, v, elem: int | None = None) -> bytes:
    """Type tag + value; arrays take the element type and a list."""
    if t == ARRAY:
        return struct.pack("<iiQ", ARRAY, elem, len(v)) + b"".join(scalar(elem, e) for e in v)
    return struct.pack("<i", t) + scalar(t, v)


def build(kv: list, tensors: list, version: int = 3, alignment: int | None = None,
          pad_data: bool = True) -> bytes:
    """kv: [(key, type, value[, elem])]; tensors: [(name, ggml_type, dims, bytes)].
    Tensors are laid out in order, each at an aligned offset."""
    al = 32 if alignment is None else alignment
    kv = list(kv)
    if alignment is not None:
        kv.append(("general.alignment", U32, alignment))
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kv))
    for entry in kv:
        key, t, v = entry[0], entry[1], entry[2]
        head += gstr(key) + value(t, v, entry[3] if len(entry) > 3 else None)
    offsets, off = [], 0
    for name, ty, dims, data in tensors:
        offsets.append(off)
        off += len(data)
        off = (off + al - 1) // al * al
    for (name, ty, dims, data), o in zip(tensors, offsets):
        head += gstr(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<q", d) for d in dims)
        head += struct.pack("<iQ", ty, o)
    if tensors:
        head += b"\0" * ((-len(head)) % al)
    body = bytearray()
    for (name, ty, dims, data), o in zip(tensors, offsets):
        body += b"\0" * (o - len(body))
        body += bytes(data)
    if pad_data:
        body += b"\0" * ((-len(body)) % al)
    return head + bytes(body)


def kquant_tensor(name: str, qtype: int, blocks: np.ndarray, n_in: int, n_out: int):
    return (name, qtype, [n_in, n_out], np.ascontiguousarray(blocks, dtype=np.uint8).tobytes())
