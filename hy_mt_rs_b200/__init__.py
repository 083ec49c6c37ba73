"""B200-native block-quantized GEMV/GEMM for hy-mt-rs packed GGUF weights.

The compute path is libhyq.so (CUDA C++, sm_100a) behind the C ABI in
include/hyq.h; `quant` mirrors the reference's quant API on top of it.
"""
from .quant import DType, HyqError, Profile, Q8, Weight, decode, device_status, dot  # noqa: F401

__all__ = ["DType", "Profile", "Weight", "Q8", "decode", "dot", "device_status", "HyqError"]
