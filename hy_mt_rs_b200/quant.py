"""Host-side mirror of hy-mt-rs `quant` (src/quant.rs) over the libhyq C ABI.

Same type enum, same entry points, same argument meaning and error behaviour
as the reference, with packed GGUF blocks resident in device memory:

    reference (quant.rs)                     here
    DType / from_id / block_len / bytes      DType (same values and rules)
    Weight (:65-154)                         Weight (device bytes, GGUF shape)
    Weight::matmul (:159)                    Weight.matmul
    Weight::gemv_qkv (:658)                  Weight.gemv_qkv
    Weight::matmul_gate_up_silu (:724)       Weight.matmul_gate_up_silu
    Q8::quantize(_into) (:904-928)           Q8.quantize / Q8.quantize_into
    gemv_q8_fast (:354)                      Weight.gemv_q8_fast
    gemv_qkv_fast (:442)                     Weight.gemv_qkv_fast
    matmul_gate_up_silu_fast (:541)          Weight.matmul_gate_up_silu_fast
    decode (:1066), dot (:2500)              decode, dot

Tensors are torch CUDA tensors used as device buffers; every call runs on the
current torch CUDA stream.  Shape errors raise HyqError where the reference
returns an anyhow error.
"""
import ctypes as C
import enum

import torch

from . import _native
from ._native import HyqError, check, lib

__all__ = ["DType", "Profile", "Weight", "Q8", "decode", "dot", "device_status", "set_launch_overlap",
           "HyqError"]


class Profile(enum.IntEnum):
    """GGUF tensor-type profiles (gguf.rs:17-27; Auto is resolved by the loader)."""

    STANDARD = 1
    TENCENT_Q2_0C = 2
    TENCENT_STQ1 = 3


class DType(enum.IntEnum):
    """Packed tensor types, quant.rs:19-27."""

    F32 = 0
    F16 = 1
    Q4_K = 2
    Q6_K = 3
    Q8_0 = 4
    Q2_0C = 5
    STQ1_0 = 6

    @staticmethod
    def from_id(type_id, profile):
        out = C.c_int()
        check(lib.hyq_dtype_from_id(type_id, int(profile), C.byref(out)))
        return DType(out.value)

    def block_len(self):
        return lib.hyq_block_len(int(self))

    def block_bytes(self):
        return lib.hyq_block_bytes(int(self))


def _stream(device=None):
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _need_cuda(t, name, dtype=None):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise HyqError(-1, f"{name}: expected a CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise HyqError(-1, f"{name}: expected {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise HyqError(-1, f"{name}: expected a contiguous tensor")


class Weight:
    """A packed GGUF tensor in device memory (quant.rs:65-154).

    `shape` is in GGUF order: shape[0] is the contiguous input width K,
    shape[1] the number of output rows N, shape[2] (optional) experts.
    """

    def __init__(self, packed, dtype, shape, name="weight", _handle=None, _owner=None):
        self.dtype = DType(dtype)
        self._shape = tuple(int(d) for d in shape)
        self.name = name
        self._owner = _owner
        if _handle is not None:
            self._h = _handle
            self.packed = packed
            return
        _need_cuda(packed, name, torch.uint8)
        self.packed = packed
        dims = (C.c_int64 * 3)(*self._shape, *([0] * (3 - len(self._shape))))
        h = C.c_void_p()
        check(lib.hyq_weight_wrap(_ptr(packed), packed.numel(), int(self.dtype), len(self._shape), dims,
                                  C.byref(h)))
        self._h = h

    @classmethod
    def upload(cls, packed_host, dtype, shape, name="weight"):
        """Copy host bytes (numpy/bytes/CPU tensor) to a library-owned buffer."""
        import numpy as np

        arr = np.ascontiguousarray(np.frombuffer(bytes(packed_host), dtype=np.uint8)
                                   if isinstance(packed_host, (bytes, bytearray)) else
                                   np.asarray(packed_host, dtype=np.uint8))
        shape = tuple(int(d) for d in shape)
        dims = (C.c_int64 * 3)(*shape, *([0] * (3 - len(shape))))
        h = C.c_void_p()
        check(lib.hyq_upload(arr.ctypes.data_as(C.c_void_p), arr.size, int(dtype), len(shape), dims, C.byref(h)))
        w = cls(None, dtype, shape, name, _handle=h)
        return w

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                lib.hyq_free(h)
            except Exception:
                pass
            self._h = None

    @property
    def handle(self):
        return self._h

    def shape(self):
        return self._shape

    @property
    def cols(self):
        return self._shape[0]

    @property
    def rows(self):
        return self._shape[1]

    @property
    def row_bytes(self):
        return self._shape[0] // self.dtype.block_len() * self.dtype.block_bytes()

    def expect_shape(self, shape):
        if tuple(shape) != self._shape:
            raise HyqError(-2, f"{self.name}: expected GGUF shape {list(shape)}, got {list(self._shape)}")

    def device(self):
        if self.packed is not None:
            return self.packed.device
        return torch.device("cuda", torch.cuda.current_device())

    # --------------------------------------------------------------- views
    def expert(self, index):
        """Weight::expert (quant.rs:144-154)."""
        h = C.c_void_p()
        check(lib.hyq_weight_expert(self._h, int(index), C.byref(h)))
        return Weight(self.packed, self.dtype, self._shape[:2], f"{self.name}[{index}]", _handle=h, _owner=self)

    def shard(self, axis, part, parts):
        """Tensor-parallel shard (hyq_weight_shard): axis 0 = output rows
        (column-parallel, a view), axis 1 = input columns on block
        boundaries (row-parallel, a gathered copy)."""
        h = C.c_void_p()
        check(lib.hyq_weight_shard(self._h, int(axis), int(part), int(parts), _stream(self.device()), C.byref(h)))
        shape = ((self._shape[0], self._shape[1] // parts) if axis == 0 else
                 (self._shape[0] // parts, self._shape[1]))
        return Weight(self.packed if axis == 0 else None, self.dtype, shape,
                      f"{self.name}[{axis}:{part}/{parts}]", _handle=h, _owner=self if axis == 0 else None)

    def row(self, row):
        """Weight::row (quant.rs:106-121)."""
        out = torch.empty(self._shape[0], dtype=torch.float32, device=self.device())
        check(lib.hyq_weight_row_into(self._h, int(row), _ptr(out), out.numel(), _stream(out.device)))
        return out

    def row_into(self, row, out):
        """Weight::row_into (quant.rs:123-142)."""
        _need_cuda(out, "row_into", torch.float32)
        check(lib.hyq_weight_row_into(self._h, int(row), _ptr(out), out.numel(), _stream(out.device)))

    def to_vec(self):
        """Weight::to_vec (quant.rs:99-104)."""
        n = self.packed.numel() // self.dtype.block_bytes() * self.dtype.block_len()
        out = torch.empty(n, dtype=torch.float32, device=self.device())
        decode(self.dtype, self.packed, out)
        return out

    # ------------------------------------------------------- f32 products
    def matmul(self, input, batch, out=None):
        """Weight::matmul (quant.rs:159-344): [batch, K] x W^T -> [batch, N]
        (into `out`, batch * N float32 values, when given)."""
        if len(self._shape) != 2:
            raise HyqError(-2, f"{self.name} is not a matrix")
        _need_cuda(input, "matmul input", torch.float32)
        if batch <= 0 or input.numel() != batch * self._shape[0]:
            raise HyqError(-2, f"{self.name}: invalid activation shape")
        if out is None:
            out = torch.empty((batch, self._shape[1]), dtype=torch.float32, device=input.device)
        elif out.numel() != batch * self._shape[1] or out.dtype != torch.float32:
            raise HyqError(-2, f"{self.name}: invalid output buffer")
        check(lib.hyq_matmul(self._h, _ptr(input), int(batch), _ptr(out), _stream(input.device)))
        return out

    @staticmethod
    def gemv_qkv(q, k, v, input):
        """Weight::gemv_qkv (quant.rs:658-721)."""
        cols = q._shape[0]
        if any(len(w._shape) != 2 for w in (q, k, v)) or k._shape[0] != cols or v._shape[0] != cols:
            raise HyqError(-2, "query, key and value must be matrices that share an input width")
        _need_cuda(input, "qkv input", torch.float32)
        if input.numel() != cols:
            raise HyqError(-2, "invalid activation shape for qkv")
        dev = input.device
        qo = torch.empty(q._shape[1], dtype=torch.float32, device=dev)
        ko = torch.empty(k._shape[1], dtype=torch.float32, device=dev)
        vo = torch.empty(v._shape[1], dtype=torch.float32, device=dev)
        check(lib.hyq_gemv_qkv(q._h, k._h, v._h, _ptr(input), _ptr(qo), _ptr(ko), _ptr(vo), _stream(dev)))
        return qo, ko, vo

    @staticmethod
    def matmul_qkv(q, k, v, input, batch):
        """Batched gemv_qkv (hyq_matmul_qkv): three [batch, N] outputs from
        one [batch, K] input, one tensor-core launch from 16 tokens up."""
        _need_cuda(input, "matmul_qkv input", torch.float32)
        if batch <= 0 or input.numel() != batch * q._shape[0]:
            raise HyqError(-2, "matmul_qkv: invalid activation shape")
        outs = [torch.empty((batch, w._shape[1]), dtype=torch.float32, device=input.device) for w in (q, k, v)]
        check(lib.hyq_matmul_qkv(q._h, k._h, v._h, _ptr(input), int(batch), *(_ptr(o) for o in outs),
                                 _stream(input.device)))
        return tuple(outs)

    def matmul_gate_up_silu_batch(self, up, input, batch):
        """Batched matmul_gate_up_silu (hyq_matmul_gate_up_silu_batch):
        silu(x gate^T) * (x up^T) for [batch, K] inputs."""
        _need_cuda(input, "gate_up_silu_batch input", torch.float32)
        if batch <= 0 or input.numel() != batch * self._shape[0]:
            raise HyqError(-2, "gate_up_silu_batch: invalid activation shape")
        out = torch.empty((batch, self._shape[1]), dtype=torch.float32, device=input.device)
        check(lib.hyq_matmul_gate_up_silu_batch(self._h, up._h, _ptr(input), int(batch), _ptr(out),
                                                _stream(input.device)))
        return out

    def matmul_gate_up_silu(self, up, input):
        """Weight::matmul_gate_up_silu (quant.rs:724-841): silu(gate x) * (up x)."""
        if up._shape != self._shape:
            raise HyqError(-2, "gate and up shape mismatch")
        _need_cuda(input, "gate_up_silu input", torch.float32)
        if input.numel() != self._shape[0]:
            raise HyqError(-2, "invalid activation shape for gate_up_silu")
        out = torch.empty(self._shape[1], dtype=torch.float32, device=input.device)
        check(lib.hyq_matmul_gate_up_silu(self._h, up._h, _ptr(input), _ptr(out), _stream(input.device)))
        return out

    # ------------------------------------------------------ int8 products
    def gemv_int8(self, input, out=None):
        """Batch-1 product through Q8 activations quantized in the kernel: the
        aarch64 path of Weight::matmul (quant.rs:169-178, gemv_q8 :346-351)."""
        _need_cuda(input, "gemv_int8 input", torch.float32)
        if input.numel() != self._shape[0]:
            raise HyqError(-2, f"{self.name}: invalid activation shape")
        if out is None:
            out = torch.empty(self._shape[1], dtype=torch.float32, device=input.device)
        check(lib.hyq_gemv_int8(self._h, _ptr(input), _ptr(out), _stream(input.device)))
        return out

    @staticmethod
    def gemv_qkv_int8(q, k, v, input):
        """Weight::gemv_qkv through int8 activations (quant.rs:673-714)."""
        _need_cuda(input, "qkv input", torch.float32)
        if input.numel() != q._shape[0]:
            raise HyqError(-2, "invalid activation shape for qkv")
        dev = input.device
        qo = torch.empty(q._shape[1], dtype=torch.float32, device=dev)
        ko = torch.empty(k._shape[1], dtype=torch.float32, device=dev)
        vo = torch.empty(v._shape[1], dtype=torch.float32, device=dev)
        check(lib.hyq_gemv_qkv_int8(q._h, k._h, v._h, _ptr(input), _ptr(qo), _ptr(ko), _ptr(vo), _stream(dev)))
        return qo, ko, vo

    def matmul_gate_up_silu_int8(self, up, input):
        """Weight::matmul_gate_up_silu through int8 activations (quant.rs:735-766)."""
        if up._shape != self._shape:
            raise HyqError(-2, "gate and up shape mismatch")
        _need_cuda(input, "gate_up_silu input", torch.float32)
        if input.numel() != self._shape[0]:
            raise HyqError(-2, "invalid activation shape for gate_up_silu")
        out = torch.empty(self._shape[1], dtype=torch.float32, device=input.device)
        check(lib.hyq_matmul_gate_up_silu_int8(self._h, up._h, _ptr(input), _ptr(out), _stream(input.device)))
        return out

    def gemv_q8_fast(self, q8, out=None):
        """gemv_q8_fast (quant.rs:353-357)."""
        if out is None:
            out = torch.empty(self._shape[1], dtype=torch.float32, device=q8.values.device)
        _need_cuda(out, "gemv_q8 out", torch.float32)
        if q8.len != self._shape[0] or out.numel() != self._shape[1]:
            raise HyqError(-2, f"{self.name}: invalid activation shape")
        check(lib.hyq_gemv_q8(self._h, _ptr(q8.values), _ptr(q8.scales), _ptr(q8.values_q2c), _ptr(out),
                              _stream(out.device)))
        return out

    @staticmethod
    def gemv_qkv_fast(q, k, v, q8, q_out=None, k_out=None, v_out=None):
        """gemv_qkv_fast (quant.rs:441-538)."""
        dev = q8.values.device
        q_out = torch.empty(q._shape[1], dtype=torch.float32, device=dev) if q_out is None else q_out
        k_out = torch.empty(k._shape[1], dtype=torch.float32, device=dev) if k_out is None else k_out
        v_out = torch.empty(v._shape[1], dtype=torch.float32, device=dev) if v_out is None else v_out
        if q8.len != q._shape[0]:
            raise HyqError(-2, "invalid activation shape for qkv")
        check(lib.hyq_gemv_qkv_q8(q._h, k._h, v._h, _ptr(q8.values), _ptr(q8.scales), _ptr(q8.values_q2c),
                                  _ptr(q_out), _ptr(k_out), _ptr(v_out), _stream(dev)))
        return q_out, k_out, v_out

    def matmul_gate_up_silu_fast(self, up, q8, out=None):
        """matmul_gate_up_silu_fast (quant.rs:540-651)."""
        if out is None:
            out = torch.empty(self._shape[1], dtype=torch.float32, device=q8.values.device)
        if up._shape != self._shape:
            raise HyqError(-2, "gate and up shape mismatch")
        if q8.len != self._shape[0]:
            raise HyqError(-2, "invalid activation shape for gate_up_silu")
        check(lib.hyq_matmul_gate_up_silu_q8(self._h, up._h, _ptr(q8.values), _ptr(q8.scales),
                                             _ptr(q8.values_q2c), _ptr(out), _stream(out.device)))
        return out


class Q8:
    """int8 activations with one f32 scale per 256 values (quant.rs:854-941)."""

    GROUP = 256

    def __init__(self, length, device=None):
        device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.len = int(length)
        self.values = torch.zeros(self.len, dtype=torch.int8, device=device)
        self.scales = torch.zeros((self.len + self.GROUP - 1) // self.GROUP, dtype=torch.float32, device=device)
        self.values_q2c = torch.zeros(self.len, dtype=torch.int8, device=device)

    def quantize_into(self, input):
        _need_cuda(input, "q8 input", torch.float32)
        if input.numel() != self.len:
            raise HyqError(-2, "q8: length mismatch")
        check(lib.hyq_q8_quantize(_ptr(input), self.len, _ptr(self.values), _ptr(self.scales),
                                  _ptr(self.values_q2c), _stream(input.device)))
        return self

    @classmethod
    def quantize(cls, input):
        return cls(input.numel(), input.device).quantize_into(input)


def decode(dtype, packed, out):
    """decode (quant.rs:1066-1079), bit-exact."""
    _need_cuda(packed, "decode input", torch.uint8)
    _need_cuda(out, "decode output", torch.float32)
    check(lib.hyq_decode(int(dtype), _ptr(packed), packed.numel(), _ptr(out), out.numel(), _stream(out.device)))
    return out


def dot(a, b):
    """dot (quant.rs:2500); returns a 0-d CUDA tensor."""
    _need_cuda(a, "dot a", torch.float32)
    _need_cuda(b, "dot b", torch.float32)
    if a.numel() != b.numel():
        raise HyqError(-2, "dot: length mismatch")
    out = torch.empty((), dtype=torch.float32, device=a.device)
    check(lib.hyq_dot(_ptr(a), _ptr(b), a.numel(), _ptr(out), _stream(a.device)))
    return out


def set_launch_overlap(enable):
    """hyq_set_launch_overlap: let batch-1 products start streaming their
    weights while the preceding kernel in the stream still runs (launch-latency
    hiding in decode chains).  Only for weights that no kernel in flight
    writes: build or upload them, synchronize, then enable."""
    check(lib.hyq_set_launch_overlap(1 if enable else 0))


GEMM_FP16, GEMM_F32 = 0, 1
_gemm_precision = GEMM_FP16  # the value last set through this module


def set_gemm_precision(precision):
    """hyq_set_gemm_precision: GEMM_FP16 (default) or GEMM_F32, the
    split-operand tensor-core products that agree with an f32 GEMM (three
    MMAs per K chunk).  Process-wide; captured graphs keep the precision they
    were captured with."""
    global _gemm_precision
    check(lib.hyq_set_gemm_precision(int(precision)))
    _gemm_precision = int(precision)


class gemm_precision:
    """Context manager: batched products issued inside run at `precision`;
    the previous setting comes back on exit."""

    def __init__(self, precision):
        self.precision = precision

    def __enter__(self):
        self._prev = _gemm_precision
        set_gemm_precision(self.precision)
        return self

    def __exit__(self, *exc):
        set_gemm_precision(self._prev)
        return False


def device_status(device=None):
    """Synchronize, then read and clear the device status word (0 = ok)."""
    v = C.c_uint32()
    rc = lib.hyq_device_status(_stream(device), C.byref(v))
    if rc not in (0, -5):
        check(rc)
    return v.value


del _native


# K columns of one packed block column of the tensor-core GEMM (hyq_gemm.cu wcol_for)
GEMM_BLOCK_COLUMN = {DType.Q8_0: 128, DType.Q2_0C: 512, DType.Q4_K: 256, DType.Q6_K: 256, DType.STQ1_0: 256}


def _token_tile(M, split=False):
    """hyq_gemm.cu token_tile / job_token_tile: 64 / 128 / 256 tokens by
    batch size, at most 128 with split operands."""
    bn = 256 if M >= 256 else 128 if M > 64 else 64
    return min(bn, 128) if split else bn


def gemm_splits(row_tiles, K, M, dtype, sms=148, split=False):
    """Split-K slices the tensor-core product takes (hyq_gemm.cu
    choose_splits): a grid of row tiles x token tiles smaller than the SM
    count is split into whole block columns, within one wave of CTAs, at
    most 16 ways."""
    tiles = row_tiles * -(-M // _token_tile(M, split))
    nwb = K // GEMM_BLOCK_COLUMN[dtype]
    if tiles >= sms:
        return 1
    z = max(1, min(sms // tiles, nwb, 16))
    per = -(-nwb // z)
    return -(-nwb // per)


def gemm_tail_slices(row_tiles, K, M, dtype, sms=148, split=False, pair=False):
    """K-slices of each tile of the thin last wave (hyq_gemm.cu tail_plan),
    1 when the product takes no tail split: fp16 operands on the 1-SM
    kernel, a grid of at least one wave whose tiles past the last full wave
    fill at most half the SMs, cut into whole block columns, at most 16."""
    if split or pair:
        return 1
    tiles = row_tiles * -(-M // _token_tile(M))
    nwb = K // GEMM_BLOCK_COLUMN[dtype]
    if tiles < sms or nwb < 2:
        return 1
    rem = tiles % sms
    if rem == 0 or 2 * rem > sms:
        return 1
    z = min(sms // rem, nwb, 16)
    per = -(-nwb // z)
    z = -(-nwb // per)
    return z if z >= 2 else 1


def gemm_launches(row_tiles, K, M, dtype, sms=148, split=False, pair=False):
    """Kernel launches of one tensor-core product (batch >= 16): the fp16
    activation copy, the GEMM, and the split-K or tail reduction when it
    takes one (`split`: split operands; `pair`: the product runs on the 2-SM
    kernel, which takes no tail split)."""
    return (2 + (1 if gemm_splits(row_tiles, K, M, dtype, sms, split) > 1 else 0)
            + (1 if gemm_tail_slices(row_tiles, K, M, dtype, sms, split, pair) > 1 else 0))
