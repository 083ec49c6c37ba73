"""The GGUF v3 reader (hyq_gguf_*, gguf.rs:50-210) on files built by
tests/gguf_writer.py: the reference's own tests (gguf.rs:339-399: a
little-endian F32 tensor, every truncation rejected, huge header counts
rejected before allocation) and the other checks of gguf.rs (metadata
types, alignment, split files, Tencent legacy profiles, partial blocks,
truncated and overlapping tensors).  Host code only: no GPU needed."""
import struct

import numpy as np
import pytest

from gguf_writer import f32, gguf_bytes


def _open(tmp_path, b, profile=0):
    from hy_mt_rs_b200.gguf import Gguf
    p = tmp_path / "m.gguf"
    p.write_bytes(b)
    return Gguf(p, profile)


def _tiny():
    return gguf_bytes(tensors=[("weight", [2], 0, f32([1.0, -2.0]))])


def test_reads_little_endian_tensor(tmp_path):
    g = _open(tmp_path, _tiny())
    assert g.tensors["weight"].dims == (2,) and g.tensors["weight"].dtype == 0
    np.testing.assert_array_equal(g.floats("weight"), [1.0, -2.0])
    assert g.profile == 1  # Standard


def test_every_truncation_is_an_error(tmp_path):
    from hy_mt_rs_b200._native import HyqError
    b = _tiny()
    for n in range(len(b)):
        with pytest.raises(HyqError):
            _open(tmp_path, b[:n])


def test_excessive_header_counts_fail(tmp_path):
    from hy_mt_rs_b200._native import HyqError
    b = bytearray(_tiny())
    b[8:16] = struct.pack("<Q", 2 ** 64 - 1)
    with pytest.raises(HyqError):
        _open(tmp_path, bytes(b))


def test_metadata_types(tmp_path):
    md = [("a.u8", 0, 7), ("a.i8", 1, -3), ("a.u16", 2, 600), ("a.i16", 3, -600), ("a.u32", 4, 70000),
          ("a.i32", 5, -70000), ("a.f32", 6, 1.5), ("a.bool", 7, 1), ("a.str", 8, "hunyuan-dense"),
          ("a.arr", 9, (8, ["x", "yy", "zzz"])), ("a.u64", 10, 2 ** 40), ("a.i64", 11, -(2 ** 40)),
          ("a.f64", 12, 0.25)]
    g = _open(tmp_path, gguf_bytes(metadata=md, tensors=[("w", [2], 0, f32([0, 0]))]))
    m = g.metadata
    assert (m["a.u8"], m["a.i8"], m["a.u16"], m["a.i16"], m["a.u32"], m["a.i32"]) == (7, -3, 600, -600, 70000, -70000)
    assert m["a.f32"] == 1.5 and m["a.bool"] is True and m["a.str"] == "hunyuan-dense"
    assert m["a.arr"].length == 3 and m["a.u64"] == 2 ** 40 and m["a.i64"] == -(2 ** 40) and m["a.f64"] == 0.25
    assert list(m) == [k for k, _, _ in md]  # file order


@pytest.mark.parametrize("bad", [
    [("k", 6, float("nan"))],                 # non-finite float
    [("k", 7, 2)],                            # invalid boolean
    [("k", 4, 1), ("k", 4, 2)],               # duplicate key
    [("general.alignment", 4, 3)],            # not a power of two
    [("general.alignment", 4, 131072)],       # above 65536
    [("split.count", 4, 2)],                  # split file
    [("k", 13, 0)],                           # unknown type
])
def test_bad_metadata_rejected(tmp_path, bad):
    from hy_mt_rs_b200._native import HyqError
    with pytest.raises(HyqError):
        _open(tmp_path, gguf_bytes(metadata=bad, tensors=[("w", [2], 0, f32([0, 0]))]))


def test_alignment_and_offsets(tmp_path):
    from hy_mt_rs_b200._native import HyqError
    md = [("general.alignment", 4, 64)]
    g = _open(tmp_path, gguf_bytes(metadata=md, alignment=64,
                                   tensors=[("a", [3], 0, f32([1, 2, 3])), ("b", [2], 0, f32([4, 5]))]))
    assert g.tensors["a"].offset % 64 == 0 and g.tensors["b"].offset - g.tensors["a"].offset == 64
    np.testing.assert_array_equal(g.floats("b"), [4, 5])
    with pytest.raises(HyqError):   # an offset off the alignment
        _open(tmp_path, gguf_bytes(metadata=md, alignment=64, tensors=[("a", [2], 0, f32([1, 2]))], offsets=[8]))


def test_tensor_checks(tmp_path):
    from hy_mt_rs_b200._native import HyqError
    with pytest.raises(HyqError):   # overlapping
        _open(tmp_path, gguf_bytes(tensors=[("a", [8], 0, f32(range(8))), ("b", [8], 0, f32(range(8)))],
                                   offsets=[0, 16]))
    with pytest.raises(HyqError):   # a partial Q4_K block in a row
        _open(tmp_path, gguf_bytes(tensors=[("q", [100, 1], 12, bytes(144))]))
    with pytest.raises(HyqError):   # truncated data
        _open(tmp_path, gguf_bytes(tensors=[("a", [8], 0, f32(range(8)))])[:-4])
    with pytest.raises(HyqError):   # zero dimension
        _open(tmp_path, gguf_bytes(tensors=[("a", [0], 0, b"")]))
    with pytest.raises(HyqError):   # rank 5
        _open(tmp_path, gguf_bytes(tensors=[("a", [1, 1, 1, 1, 1], 0, f32([1]))]))
    with pytest.raises(HyqError):   # unsupported type id
        _open(tmp_path, gguf_bytes(tensors=[("a", [32], 2, bytes(18))]))
    with pytest.raises(HyqError):   # version 2
        _open(tmp_path, gguf_bytes(tensors=[("a", [1], 0, f32([1]))], version=2))


def test_tencent_legacy_profiles(tmp_path):
    from hy_mt_rs_b200._native import HyqError
    from hy_mt_rs_b200.gguf import TENCENT_Q2_0C, TENCENT_STQ1
    q2 = ("blk.0.attn_q.weight", [512, 1], 40, bytes(130))
    ok_md = [("general.architecture", 8, "hunyuan-dense"), ("general.file_type", 4, 39)]
    b = gguf_bytes(metadata=ok_md, tensors=[q2, ("n", [4], 0, f32([1, 2, 3, 4]))])
    with pytest.raises(HyqError):   # legacy id under Auto in an unrecognised file
        _open(tmp_path, b)
    g = _open(tmp_path, b, TENCENT_Q2_0C)
    assert g.profile == TENCENT_Q2_0C and g.tensors["blk.0.attn_q.weight"].dtype == 5
    with pytest.raises(HyqError):   # the other profile
        _open(tmp_path, b, TENCENT_STQ1)
    with pytest.raises(HyqError):   # not hunyuan-dense
        _open(tmp_path, gguf_bytes(metadata=[("general.architecture", 8, "llama"), ("general.file_type", 4, 39)],
                                   tensors=[q2]), TENCENT_Q2_0C)
    with pytest.raises(HyqError):   # wrong file type
        _open(tmp_path, gguf_bytes(metadata=[ok_md[0], ("general.file_type", 4, 41)], tensors=[q2]), TENCENT_Q2_0C)
    with pytest.raises(HyqError):   # a Q4_K tensor in a Tencent export
        _open(tmp_path, gguf_bytes(metadata=ok_md, tensors=[q2, ("k", [256, 1], 12, bytes(144))]), TENCENT_Q2_0C)


def test_legacy_file_digest_is_sha256(tmp_path):
    """The unrecognised-file error names the file's SHA-256 (gguf.rs:113-126),
    computed by the library's own SHA-256: it equals hashlib's."""
    import hashlib
    from hy_mt_rs_b200._native import HyqError
    for extra in (0, 55, 56, 64, 119):   # padding boundaries of the last block
        b = gguf_bytes(metadata=[("general.architecture", 8, "hunyuan-dense"), ("pad", 8, "x" * extra)],
                       tensors=[("q", [512, 1], 40, bytes(130))])
        with pytest.raises(HyqError) as e:
            _open(tmp_path, b)
        assert hashlib.sha256(b).hexdigest() in str(e.value)
