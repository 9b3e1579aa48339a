"""Writes GGUF v3 files from the published layout (magic "GGUF", u32
version, u64 tensor and key-value counts, typed key-value pairs, tensor
descriptors, padding to the alignment, then tensor payloads each padded to
the alignment), for synthetic checkpoints in the benchmark and the tests.
Keyword overrides write malformed files on purpose (reader tests)."""
from __future__ import annotations

import struct
from pathlib import Path

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
        I64: "<q", F64: "<d"}
# ggml type -> (values per block, bytes per block) for the types the reader accepts.
GEOMETRY = {0: (1, 4), 8: (32, 34), 11: (256, 110), 12: (256, 144), 14: (256, 210), 18: (256, 98), 20: (32, 18),
            21: (256, 110), 22: (256, 82), 23: (256, 136), 30: (1, 2), 39: (32, 17)}


def text(s) -> bytes:
    b = s.encode() if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


def value(vtype: int, v) -> bytes:
    if vtype == STRING:
        return text(v)
    if vtype == ARRAY:
        elem, items = v
        out = struct.pack("<IQ", elem, len(items))
        return out + b"".join(value(elem, x) for x in items)
    return struct.pack(_FMT.get(vtype, "<B"), v)  # unknown types: one byte, for malformed files


def payload_bytes(ne, ggml_type: int) -> int:
    values, width = GEOMETRY.get(ggml_type, (1, 2))
    rows = 1
    for d in ne[1:]:
        rows *= d
    return ne[0] // values * width * rows


def pad(n: int, a: int) -> int:
    return (n + a - 1) // a * a


def build(kvs, tensors, *, alignment: int = 32, magic: bytes = b"GGUF", version: int = 3, tensor_count=None,
          kv_count=None, offsets=None, data_pad: bool = True, truncate=None, extra=b""):
    """kvs: [(key, type, value)] (ARRAY value = (element type, [items])).
    tensors: [(name, ne, ggml_type, payload bytes or None for a pattern)].
    Returns (file bytes, {name: payload})."""
    head = magic + struct.pack("<I", version)
    head += struct.pack("<QQ", len(tensors) if tensor_count is None else tensor_count,
                        len(kvs) if kv_count is None else kv_count)
    for key, vtype, v in kvs:
        head += text(key) + struct.pack("<I", vtype) + value(vtype, v)
    payloads, running = {}, 0
    infos = b""
    for i, (name, ne, gtype, data) in enumerate(tensors):
        n = payload_bytes(ne, gtype)
        if data is None:
            data = bytes((7 * i + 13 * k) & 0xFF for k in range(n))
        payloads[name] = data
        off = running if offsets is None else offsets[i]
        infos += text(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", d) for d in ne)
        infos += struct.pack("<IQ", gtype, off)
        running += pad(len(data), alignment)
    head += infos
    body = bytearray(head)
    if tensors and data_pad:
        body += b"\0" * (pad(len(body), alignment) - len(body))
    start = len(body)
    for name, ne, gtype, _ in tensors:
        data = payloads[name]
        body += data
        body += b"\0" * (pad(len(body) - start, alignment) - (len(body) - start))
    body += extra
    if truncate is not None:
        body = body[:truncate]
    return bytes(body), payloads


def write(path: Path, kvs, tensors, **kw):
    data, payloads = build(kvs, tensors, **kw)
    Path(path).write_bytes(data)
    return payloads


def write_arrays(path: Path, kvs, tensors, alignment: int = 32) -> dict:
    """A well-formed file from large payloads, streamed to disk.
    tensors: [(name, ne, ggml_type, array or bytes)]. Returns {name: absolute
    payload offset}."""
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kvs))
    for key, vtype, v in kvs:
        head += text(key) + struct.pack("<I", vtype) + value(vtype, v)
    running, offsets = 0, {}
    for name, ne, gtype, data in tensors:
        n = memoryview(data).nbytes
        if n != payload_bytes(ne, gtype):
            raise ValueError(f"{name}: {n} payload bytes for shape {ne} of type {gtype}")
        head += text(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", d) for d in ne)
        head += struct.pack("<IQ", gtype, running)
        offsets[name] = running
        running += pad(n, alignment)
    start = pad(len(head), alignment) if tensors else len(head)
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (start - len(head)))
        for name, ne, gtype, data in tensors:
            mv = memoryview(data).cast("B")
            f.write(mv)
            f.write(b"\0" * (pad(mv.nbytes, alignment) - mv.nbytes))
    return {k: start + v for k, v in offsets.items()}
