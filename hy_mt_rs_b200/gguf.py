"""GGUF v3 model files (hy-mt-rs src/gguf.rs:50-210) through libhyq's reader:
the file is memory-mapped and checked as the reference does, tensors go to
the device unchanged.

    g = Gguf("model.gguf")                  # profile AUTO, STANDARD, TENCENT_Q2_0C, TENCENT_STQ1
    g.metadata["general.architecture"]      # typed scalars; arrays as their length
    g.tensors["token_embd.weight"]          # TensorInfo(dtype, type_id, dims, offset, byte_len)
    w = g.tensor("blk.0.attn_q.weight")     # quant.Weight on the device
"""
import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import quant
from ._native import check, lib

AUTO, STANDARD, TENCENT_Q2_0C, TENCENT_STQ1 = 0, 1, 2, 3


@dataclass
class TensorInfo:
    name: str
    dtype: int
    type_id: int
    dims: tuple
    offset: int
    byte_len: int


@dataclass
class ArrayValue:
    """A metadata array (the reader keeps its length)."""
    length: int


class Gguf:
    def __init__(self, path, profile=AUTO):
        h = C.c_void_p()
        check(lib.hyq_gguf_open(str(path).encode(), int(profile), C.byref(h)))
        self._h = h
        self.path = str(path)
        self.profile = lib.hyq_gguf_profile(h)
        self.metadata = self._read_metadata()
        self.tensors = self._read_tensors()

    def _read_metadata(self):
        md = {}
        n = lib.hyq_gguf_meta_count(self._h)
        for i in range(n):
            key, kind = C.c_char_p(), C.c_int()
            check(lib.hyq_gguf_meta_key(self._h, i, C.byref(key), C.byref(kind)))
            k = key.value.decode()
            t = kind.value
            if t == 8:
                s, ln = C.c_char_p(), C.c_size_t()
                check(lib.hyq_gguf_meta_str(self._h, key.value, C.byref(s), C.byref(ln)))
                md[k] = C.string_at(s, ln.value).decode("utf-8", errors="replace")
            elif t == 7:
                b = C.c_int()
                check(lib.hyq_gguf_meta_bool(self._h, key.value, C.byref(b)))
                md[k] = bool(b.value)
            elif t == 9:
                ln = C.c_int64()
                check(lib.hyq_gguf_meta_array_len(self._h, key.value, C.byref(ln)))
                md[k] = ArrayValue(ln.value)
            elif t in (6, 12):
                f = C.c_double()
                check(lib.hyq_gguf_meta_f64(self._h, key.value, C.byref(f)))
                md[k] = f.value
            else:
                u = C.c_uint64()
                if lib.hyq_gguf_meta_u64(self._h, key.value, C.byref(u)) == 0:
                    md[k] = int(u.value)
                else:  # a negative signed integer
                    f = C.c_double()
                    check(lib.hyq_gguf_meta_f64(self._h, key.value, C.byref(f)))
                    md[k] = int(f.value)
        return md

    def _read_tensors(self):
        out = {}
        for i in range(lib.hyq_gguf_tensor_count(self._h)):
            name = C.c_char_p()
            check(lib.hyq_gguf_tensor_name(self._h, i, C.byref(name)))
            dtype, tid, nd = C.c_int(), C.c_uint32(), C.c_int()
            dims = (C.c_int64 * 4)()
            off, ln = C.c_uint64(), C.c_uint64()
            check(lib.hyq_gguf_tensor_info(self._h, name.value, C.byref(dtype), C.byref(tid), C.byref(nd), dims,
                                           C.byref(off), C.byref(ln)))
            n = name.value.decode()
            out[n] = TensorInfo(n, dtype.value, tid.value, tuple(dims[:nd.value]), off.value, ln.value)
        return out

    def data(self, name):
        """The tensor's packed bytes in the mapped file (read-only numpy view,
        valid while the file is open)."""
        p, n = C.c_void_p(), C.c_size_t()
        check(lib.hyq_gguf_tensor_data(self._h, name.encode(), C.byref(p), C.byref(n)))
        buf = (C.c_uint8 * n.value).from_address(p.value)
        arr = np.frombuffer(buf, dtype=np.uint8)
        arr.flags.writeable = False
        return arr

    def tensor(self, name):
        """Gguf::tensor (gguf.rs:214-220): the tensor as a device weight."""
        info = self.tensors.get(name)
        if info is None:
            raise KeyError(f"missing tensor {name}")
        h = C.c_void_p()
        check(lib.hyq_gguf_upload(self._h, name.encode(), C.byref(h)))
        return quant.Weight(None, info.dtype, info.dims, name, _handle=h)

    def floats(self, name):
        """An F32 or F16 tensor (norms, router bias) as a float32 numpy array."""
        info = self.tensors[name]
        b = self.data(name)
        if info.dtype == quant.DType.F32:
            return b.view(np.float32).copy()
        if info.dtype == quant.DType.F16:
            return b.view(np.float16).astype(np.float32)
        raise ValueError(f"{name} is not an F32/F16 tensor")

    def close(self):
        h = getattr(self, "_h", None)
        if h is not None:
            lib.hyq_gguf_close(h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
