"""B200-native block-quantized GEMV/GEMM for hy-mt-rs packed GGUF weights.

The compute path is libhyq.so (CUDA C++, sm_100a) behind the C ABI in
include/hyq.h; `quant` mirrors the reference's quant API on top of it.
Importing `quant` (or any name below) loads the library and raises if it is
missing; importing the package alone, or `synth`, does not load it, so CPU-only
tools (the reference benchmark arm, fixture scripts) stay free of it.
"""

__all__ = ["DType", "Profile", "Weight", "Q8", "decode", "dot", "device_status", "HyqError"]


def __getattr__(name):
    if name in __all__:
        from . import quant

        return getattr(quant, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
