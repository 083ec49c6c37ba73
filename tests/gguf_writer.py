"""A small GGUF v3 writer for the tests (test infrastructure): builds files
with chosen metadata and tensors so that the reader's checks can be driven
file by file."""
import struct

import numpy as np

_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B", 10: "<Q", 11: "<q", 12: "<d"}


def _string(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(kind, v):
    if kind == 8:
        return _string(v)
    if kind == 9:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    if kind not in _SCALAR:  # an unknown type id: 4 payload bytes, for the reader to reject
        return struct.pack("<I", v)
    return struct.pack(_SCALAR[kind], v)


def gguf_bytes(metadata=(), tensors=(), alignment=32, version=3, offsets=None):
    """metadata: (key, type, value); tensors: (name, dims, type_id, bytes).
    Tensor data follows the header at the alignment, in order, each padded
    to the alignment (offsets overrides the relative offsets)."""
    out = bytearray(b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(metadata)))
    for key, kind, v in metadata:
        out += _string(key) + struct.pack("<I", kind) + _value(kind, v)
    rel, pos = [], 0
    for _, _, _, data in tensors:
        rel.append(pos)
        pos = (pos + len(data) + alignment - 1) // alignment * alignment
    if offsets is not None:
        rel = list(offsets)
    for (name, dims, tid, _), off in zip(tensors, rel):
        out += _string(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", tid, off)
    out += b"\0" * ((-len(out)) % alignment)
    base = len(out)
    for (_, _, _, data), off in zip(tensors, rel):
        need = base + off + len(data)
        if len(out) < need:
            out += b"\0" * (base + off - len(out)) if len(out) < base + off else b""
            out[base + off:base + off + len(data)] = data
    return bytes(out)


def f32(a):
    return np.asarray(a, dtype=np.float32).tobytes()
