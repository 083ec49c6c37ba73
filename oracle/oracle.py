"""ctypes bindings of the C oracle (test infrastructure only).

Every function mirrors one reference routine of hy-mt-rs src/quant.rs; the
C file cites the exact lines.  Arrays are numpy; the library is built on first
use by oracle/build.py.
"""
import ctypes as C
import os

import numpy as np

from . import build as _build

_LIB = None

_f32p = C.POINTER(C.c_float)
_u8p = C.POINTER(C.c_uint8)
_i8p = C.POINTER(C.c_int8)


def lib():
    global _LIB
    if _LIB is None:
        path = _build.build()
        L = C.CDLL(path)
        L.hyo_block_len.argtypes = [C.c_int]
        L.hyo_block_bytes.argtypes = [C.c_int]
        L.hyo_dtype_from_id.argtypes = [C.c_uint32, C.c_int]
        L.hyo_half.argtypes = [C.c_uint16]
        L.hyo_half.restype = C.c_float
        L.hyo_decode.argtypes = [C.c_int, _u8p, C.c_size_t, _f32p, C.c_size_t]
        L.hyo_dot.argtypes = [_f32p, _f32p, C.c_size_t]
        L.hyo_dot.restype = C.c_float
        L.hyo_dot_scalar.argtypes = [_f32p, _f32p, C.c_size_t]
        L.hyo_dot_scalar.restype = C.c_float
        L.hyo_row_dot_f32.argtypes = [C.c_int, _u8p, _f32p, C.c_int64]
        L.hyo_row_dot_f32.restype = C.c_float
        L.hyo_matmul.argtypes = [C.c_int, _u8p, C.c_int64, C.c_int64, _f32p, C.c_int64, _f32p, C.c_int]
        L.hyo_matmul.restype = None
        L.hyo_gate_up_silu.argtypes = [C.c_int, _u8p, _u8p, C.c_int64, C.c_int64, _f32p, _f32p, C.c_int]
        L.hyo_gate_up_silu.restype = None
        L.hyo_q8_quantize.argtypes = [_f32p, C.c_int64, _i8p, _f32p, _i8p]
        L.hyo_q8_quantize.restype = None
        L.hyo_row_dot_q8.argtypes = [C.c_int, _u8p, C.c_int64, _i8p, _f32p, _i8p]
        L.hyo_row_dot_q8.restype = C.c_float
        L.hyo_gemv_q8.argtypes = [C.c_int, _u8p, C.c_int64, C.c_int64, _i8p, _f32p, _i8p, _f32p, C.c_int]
        L.hyo_rms_norm.argtypes = [_f32p, _f32p, C.c_int64, C.c_float, _f32p]
        L.hyo_rms_norm.restype = None
        L.hyo_rms_norm_rows.argtypes = [_f32p, C.c_int64, _f32p, C.c_int64, C.c_float]
        L.hyo_rms_norm_rows.restype = None
        L.hyo_rope_table.argtypes = [C.c_int64, C.c_int, C.c_float, _f32p, _f32p]
        L.hyo_rope_table.restype = None
        L.hyo_rope.argtypes = [_f32p, C.c_int64, C.c_int64, _f32p, _f32p]
        L.hyo_rope.restype = None
        L.hyo_attention.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_int, C.c_int64, _f32p]
        L.hyo_attention.restype = None
        L.hyo_gemv_q8.restype = None
        L.hyo_gate_up_silu_q8.argtypes = [C.c_int, _u8p, _u8p, C.c_int64, C.c_int64, _i8p, _f32p, _i8p,
                                          _f32p, C.c_int]
        L.hyo_gate_up_silu_q8.restype = None
        L.hyo_decode_rows.argtypes = [C.c_int, _u8p, C.c_int64, C.c_int64, _f32p, C.c_int]
        L.hyo_decode_rows.restype = None
        L.hyo_max_threads.argtypes = []
        L.hyo_moe_route.argtypes = [_f32p, C.c_int, _f32p, C.c_int, C.c_int, C.c_float, C.POINTER(C.c_int32), _f32p]
        L.hyo_moe_route.restype = None
        _LIB = L
    return _LIB


def _p(a, t):
    return a.ctypes.data_as(t)


def _u8(a):
    a = np.ascontiguousarray(a, dtype=np.uint8)
    return a


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def block_len(t):
    return lib().hyo_block_len(int(t))


def block_bytes(t):
    return lib().hyo_block_bytes(int(t))


def dtype_from_id(type_id, profile):
    return lib().hyo_dtype_from_id(type_id, profile)


def half(bits):
    return lib().hyo_half(bits)


def decode(t, data, n_out):
    """decode (quant.rs:1066).  Raises ValueError where the reference bails."""
    data = _u8(data)
    out = np.empty(n_out, dtype=np.float32)
    rc = lib().hyo_decode(int(t), _p(data, _u8p), data.size, _p(out, _f32p), n_out)
    if rc != 0:
        raise ValueError("decode: shape/byte-count mismatch")
    return out


def dot(a, b):
    a, b = _f32(a), _f32(b)
    assert a.size == b.size
    return lib().hyo_dot(_p(a, _f32p), _p(b, _f32p), a.size)


def dot_scalar(a, b):
    a, b = _f32(a), _f32(b)
    return lib().hyo_dot_scalar(_p(a, _f32p), _p(b, _f32p), a.size)


def row_dot_f32(t, row, x):
    row, x = _u8(row), _f32(x)
    return lib().hyo_row_dot_f32(int(t), _p(row, _u8p), _p(x, _f32p), x.size)


def matmul(t, w, K, N, x, batch, threads=0):
    """Weight::matmul, output [batch, N]."""
    w, x = _u8(w), _f32(x)
    assert x.size == batch * K
    y = np.empty(batch * N, dtype=np.float32)
    lib().hyo_matmul(int(t), _p(w, _u8p), K, N, _p(x, _f32p), batch, _p(y, _f32p), threads)
    return y.reshape(batch, N)


def decode_rows(t, w, K, N, threads=0):
    """Rows of a packed [K, N] weight decoded to f32 [N, K], in parallel (the
    decode half of quant.rs:280-296)."""
    w = _u8(w)
    out = np.empty((N, K), dtype=np.float32)
    lib().hyo_decode_rows(int(t), _p(w, _u8p), K, N, _p(out, _f32p), threads)
    return out


def gate_up_silu(t, gate, up, K, N, x, threads=0):
    gate, up, x = _u8(gate), _u8(up), _f32(x)
    y = np.empty(N, dtype=np.float32)
    lib().hyo_gate_up_silu(int(t), _p(gate, _u8p), _p(up, _u8p), K, N, _p(x, _f32p), _p(y, _f32p), threads)
    return y


def q8_quantize(x):
    """Q8::quantize -> (values int8, scales f32, values_q2c int8)."""
    x = _f32(x)
    n = x.size
    values = np.empty(n, dtype=np.int8)
    q2c = np.empty(n, dtype=np.int8)
    scales = np.empty((n + 255) // 256, dtype=np.float32)
    lib().hyo_q8_quantize(_p(x, _f32p), n, _p(values, _i8p), _p(scales, _f32p), _p(q2c, _i8p))
    return values, scales, q2c


def row_dot_q8(t, row, K, values, scales, q2c):
    row = _u8(row)
    values = np.ascontiguousarray(values, dtype=np.int8)
    q2c = np.ascontiguousarray(q2c, dtype=np.int8)
    scales = _f32(scales)
    return lib().hyo_row_dot_q8(int(t), _p(row, _u8p), K, _p(values, _i8p), _p(scales, _f32p), _p(q2c, _i8p))


def gemv_q8(t, w, K, N, values, scales, q2c, threads=0):
    w = _u8(w)
    values = np.ascontiguousarray(values, dtype=np.int8)
    q2c = np.ascontiguousarray(q2c, dtype=np.int8)
    scales = _f32(scales)
    y = np.empty(N, dtype=np.float32)
    lib().hyo_gemv_q8(int(t), _p(w, _u8p), K, N, _p(values, _i8p), _p(scales, _f32p), _p(q2c, _i8p),
                      _p(y, _f32p), threads)
    return y


def gate_up_silu_q8(t, gate, up, K, N, values, scales, q2c, threads=0):
    gate, up = _u8(gate), _u8(up)
    values = np.ascontiguousarray(values, dtype=np.int8)
    q2c = np.ascontiguousarray(q2c, dtype=np.int8)
    scales = _f32(scales)
    y = np.empty(N, dtype=np.float32)
    lib().hyo_gate_up_silu_q8(int(t), _p(gate, _u8p), _p(up, _u8p), K, N, _p(values, _i8p), _p(scales, _f32p),
                              _p(q2c, _i8p), _p(y, _f32p), threads)
    return y


def max_threads():
    return lib().hyo_max_threads()


def host_cores():
    return os.cpu_count() or 1


# ---------------------------------------------------------------- model step
def rms_norm(x, w, eps):
    """rms_norm_into (model.rs:785-830)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty_like(x)
    lib().hyo_rms_norm(_p(x, _f32p), _p(np.ascontiguousarray(w, dtype=np.float32), _f32p), x.size, eps,
                       _p(out, _f32p))
    return out


def rms_norm_rows(v, w, eps):
    """rms_norm per row of len(w) (model.rs:832-872); returns a new array."""
    v = np.array(v, dtype=np.float32, copy=True)
    w = np.ascontiguousarray(w, dtype=np.float32)
    lib().hyo_rms_norm_rows(_p(v, _f32p), v.size // w.size, _p(w, _f32p), w.size, eps)
    return v


def rope_table(pos, head_dim, base):
    """cos, sin for one position (model.rs:266-272, 378-391)."""
    c = np.empty(head_dim // 2, dtype=np.float32)
    s = np.empty(head_dim // 2, dtype=np.float32)
    lib().hyo_rope_table(pos, head_dim, base, _p(c, _f32p), _p(s, _f32p))
    return c, s


def rope(v, heads, dim, cos, sin):
    """rope_with_cache (model.rs:874-913); returns a new array."""
    v = np.array(v, dtype=np.float32, copy=True)
    lib().hyo_rope(_p(v, _f32p), heads, dim, _p(cos, _f32p), _p(sin, _f32p))
    return v


def attention(q, keys, values, heads, kv_heads, dim, past):
    """attention_into for one token (model.rs:949-1021)."""
    out = np.empty(heads * dim, dtype=np.float32)
    lib().hyo_attention(_p(np.ascontiguousarray(q, dtype=np.float32), _f32p),
                        _p(np.ascontiguousarray(keys, dtype=np.float32), _f32p),
                        _p(np.ascontiguousarray(values, dtype=np.float32), _f32p), heads, kv_heads, dim, past,
                        _p(out, _f32p))
    return out


def moe_route(logits, bias, used, normalize, scale):
    """route (model.rs:728-767) per token of logits [tokens, experts]:
    (indices [tokens, used] int32, weights [tokens, used] f32)."""
    logits = np.ascontiguousarray(np.atleast_2d(logits), dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    T, E = logits.shape
    idx = np.empty((T, used), dtype=np.int32)
    w = np.empty((T, used), dtype=np.float32)
    for t in range(T):
        lib().hyo_moe_route(_p(logits[t], _f32p), E, _p(bias, _f32p), used, 1 if normalize else 0, scale,
                            idx[t].ctypes.data_as(C.POINTER(C.c_int32)), _p(w[t], _f32p))
    return idx, w
