"""CPU checks of the C ABI: the library loads, exports every entry point that
include/hyq.h declares, and rejects bad arguments on the host (no GPU work)."""
import ctypes as C
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "hyq.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hyq_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from hy_mt_rs_b200 import _native

    names = declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(_native.lib, n)]
    assert not missing, missing
    # the Python binding covers the whole header
    assert set(_native.exported_symbols()) == set(names)


def test_geometry_and_profiles():
    from hy_mt_rs_b200.quant import DType, HyqError, Profile

    assert [DType(t).block_len() for t in range(7)] == [1, 1, 256, 256, 32, 512, 256]
    assert [DType(t).block_bytes() for t in range(7)] == [4, 2, 144, 210, 34, 130, 42]
    assert DType.from_id(42, Profile.TENCENT_STQ1) == DType.STQ1_0
    assert DType.from_id(40, Profile.TENCENT_Q2_0C) == DType.Q2_0C
    with pytest.raises(HyqError):
        DType.from_id(40, Profile.STANDARD)
    with pytest.raises(HyqError):
        DType.from_id(42, Profile.TENCENT_Q2_0C)


def _wrap(dtype, dims, nbytes, ptr=0x10000):
    from hy_mt_rs_b200 import _native

    d = (C.c_int64 * 3)(*dims, *([0] * (3 - len(dims))))
    h = C.c_void_p()
    rc = _native.lib.hyq_weight_wrap(C.c_void_p(ptr), nbytes, dtype, len(dims), d, C.byref(h))
    return rc, h


def test_weight_handle_validation():
    from hy_mt_rs_b200 import _native

    L = _native.lib
    rc, h = _wrap(2, [2048, 6144], 6144 * 1152)
    assert rc == 0 and h.value
    dims = (C.c_int64 * 3)()
    t = C.c_int()
    nd = C.c_int()
    nb = C.c_size_t()
    assert L.hyq_weight_info(h, C.byref(t), C.byref(nd), dims, C.byref(nb), None) == 0
    assert (t.value, nd.value, list(dims), nb.value) == (2, 2, [2048, 6144, 0], 6144 * 1152)
    L.hyq_free(h)
    # byte count / block multiple / dtype checks
    assert _wrap(2, [2048, 6144], 6144 * 1152 - 1)[0] == -2
    assert _wrap(2, [2000, 10], 10 * 1152)[0] == -2
    assert _wrap(9, [2048, 10], 10)[0] == -1
    assert "unsupported tensor type" in _native.last_error()
    # experts: Weight::expert (quant.rs:144-154)
    rc, h3 = _wrap(2, [2048, 1024, 64], 64 * 1024 * 1152)
    assert rc == 0
    e = C.c_void_p()
    assert L.hyq_weight_expert(h3, 5, C.byref(e)) == 0
    ptr = C.c_void_p()
    assert L.hyq_weight_info(e, None, C.byref(nd), dims, C.byref(nb), C.byref(ptr)) == 0
    assert nd.value == 2 and nb.value == 1024 * 1152 and ptr.value == 0x10000 + 5 * 1024 * 1152
    assert L.hyq_weight_expert(h3, 64, C.byref(e)) == -2
    rc, h2 = _wrap(2, [2048, 6144], 6144 * 1152)
    assert L.hyq_weight_expert(h2, 0, C.byref(e)) == -2  # a matrix has no experts
    L.hyq_free(e)
    L.hyq_free(h2)
    L.hyq_free(h3)


def test_weight_shard_validation():
    """hyq_weight_shard: row shards are views at the right byte offset; the
    K split must fall on block boundaries (checked before any allocation)."""
    from hy_mt_rs_b200 import _native

    L = _native.lib
    rc, h = _wrap(2, [4096, 14336], 14336 * 2304)  # Q4_K 14336x4096 (7B gate)
    assert rc == 0
    s = C.c_void_p()
    dims = (C.c_int64 * 3)()
    nb = C.c_size_t()
    ptr = C.c_void_p()
    assert L.hyq_weight_shard(h, 0, 3, 8, None, C.byref(s)) == 0
    assert L.hyq_weight_info(s, None, None, dims, C.byref(nb), C.byref(ptr)) == 0
    assert list(dims)[:2] == [4096, 1792] and nb.value == 1792 * 2304
    assert ptr.value == 0x10000 + 3 * 1792 * 2304
    L.hyq_free(s)
    assert L.hyq_weight_shard(h, 0, 8, 8, None, C.byref(s)) == -1       # part out of range
    assert L.hyq_weight_shard(h, 2, 0, 2, None, C.byref(s)) == -1       # no such axis
    assert L.hyq_weight_shard(h, 0, 0, 5, None, C.byref(s)) == -2       # 14336 rows / 5
    assert L.hyq_weight_shard(h, 1, 0, 32, None, C.byref(s)) == -2      # 4096/32 = 128 < one block
    L.hyq_free(h)
    rc, h = _wrap(5, [6144, 2048], 2048 * 12 * 130)  # Q2_0C down, K = 12 blocks of 512
    assert L.hyq_weight_shard(h, 1, 0, 8, None, C.byref(s)) == -2       # 768 is not whole blocks
    assert "whole 512-weight blocks" in _native.last_error()
    L.hyq_free(h)


def test_entry_points_reject_bad_shapes_before_launch():
    from hy_mt_rs_b200 import _native

    L = _native.lib
    # decode: partial block / wrong byte count (quant.rs:1067-1076)
    assert L.hyq_decode(2, C.c_void_p(0x10000), 144, C.c_void_p(0x20000), 255, None) == -2
    assert L.hyq_decode(2, C.c_void_p(0x10000), 143, C.c_void_p(0x20000), 256, None) == -2
    assert L.hyq_decode(2, None, 0, None, 0, None) == 0
    rc, h = _wrap(5, [2048, 512], 512 * 520)
    rc3, h3 = _wrap(5, [2048, 8, 2], 16 * 520)
    # matmul: not a matrix / bad batch (quant.rs:160-166)
    assert L.hyq_matmul(h3, C.c_void_p(0x30000), 1, C.c_void_p(0x40000), None) == -2
    assert L.hyq_matmul(h, C.c_void_p(0x30000), 0, C.c_void_p(0x40000), None) == -2
    # qkv: widths must match (quant.rs:664-671)
    rc2, hk = _wrap(5, [1024, 512], 512 * 260)
    assert L.hyq_gemv_qkv(h, hk, h, C.c_void_p(0x30000), C.c_void_p(0x40000), C.c_void_p(0x50000),
                          C.c_void_p(0x60000), None) == -2
    # gate/up shape mismatch (quant.rs:726)
    assert L.hyq_matmul_gate_up_silu(h, hk, C.c_void_p(0x30000), C.c_void_p(0x40000), None) == -2
    # misaligned f32 input
    assert L.hyq_matmul(h, C.c_void_p(0x30002), 1, C.c_void_p(0x40000), None) == -3
    # null pointers
    assert L.hyq_matmul(None, C.c_void_p(0x30000), 1, C.c_void_p(0x40000), None) == -1
    assert L.hyq_q8_quantize(None, 16, None, None, None, None) == -1
    for x in (h, h3, hk):
        L.hyq_free(x)
