"""ctypes binding of libhyq.so (the C ABI declared in include/hyq.h).

The library is the only compute path: if it is missing or fails to load,
importing this module raises.  There is no CPU fallback.
"""
import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libhyq.so")

HYQ_OK = 0
ERRORS = {
    -1: "HYQ_E_INVALID",
    -2: "HYQ_E_SHAPE",
    -3: "HYQ_E_ALIGN",
    -4: "HYQ_E_CUDA",
    -5: "HYQ_E_DEVICE",
    -6: "HYQ_E_UNSUPPORTED",
    -7: "HYQ_E_NOMEM",
}


class HyqError(RuntimeError):
    """A libhyq call returned a negative status."""

    def __init__(self, code, message):
        super().__init__(f"{ERRORS.get(code, code)}: {message}")
        self.code = code


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libhyq.so not built ({LIB_PATH}); run `python -m hy_mt_rs_b200.build`")
    return C.CDLL(LIB_PATH)


lib = _load()

_vp = C.c_void_p
_i64 = C.c_int64
_i64p = C.POINTER(C.c_int64)
_wp = C.c_void_p  # hyq_weight*

_SIGS = {
    "hyq_last_error": ([], C.c_char_p),
    "hyq_block_len": ([C.c_int], C.c_int),
    "hyq_block_bytes": ([C.c_int], C.c_int),
    "hyq_dtype_from_id": ([C.c_uint32, C.c_int, C.POINTER(C.c_int)], C.c_int),
    "hyq_upload": ([_vp, C.c_size_t, C.c_int, C.c_int, _i64p, C.POINTER(_wp)], C.c_int),
    "hyq_weight_wrap": ([_vp, C.c_size_t, C.c_int, C.c_int, _i64p, C.POINTER(_wp)], C.c_int),
    "hyq_weight_expert": ([_wp, _i64, C.POINTER(_wp)], C.c_int),
    "hyq_weight_shard": ([_wp, C.c_int, _i64, _i64, _vp, C.POINTER(_wp)], C.c_int),
    "hyq_weight_info": ([_wp, C.POINTER(C.c_int), C.POINTER(C.c_int), _i64p, C.POINTER(C.c_size_t),
                         C.POINTER(_vp)], C.c_int),
    "hyq_free": ([_wp], None),
    "hyq_decode": ([C.c_int, _vp, C.c_size_t, _vp, C.c_size_t, _vp], C.c_int),
    "hyq_weight_row_into": ([_wp, _i64, _vp, _i64, _vp], C.c_int),
    "hyq_dot": ([_vp, _vp, C.c_size_t, _vp, _vp], C.c_int),
    "hyq_matmul": ([_wp, _vp, _i64, _vp, _vp], C.c_int),
    "hyq_gemv_qkv": ([_wp, _wp, _wp, _vp, _vp, _vp, _vp, _vp], C.c_int),
    "hyq_matmul_gate_up_silu": ([_wp, _wp, _vp, _vp, _vp], C.c_int),
    "hyq_gemv_qkv_norm": ([_wp, _wp, _wp, _vp, _vp, C.c_float, C.c_int, _vp, _vp, _vp, _vp], C.c_int),
    "hyq_gemv_gate_up_silu_norm": ([_wp, _wp, _vp, _vp, C.c_float, C.c_int, _vp, _vp], C.c_int),
    "hyq_gemv_norm": ([_wp, _vp, _vp, C.c_float, C.c_int, _vp, _vp], C.c_int),
    "hyq_gemv_residual": ([_wp, _vp, C.c_int, _vp, _vp], C.c_int),
    "hyq_gemv_fusable": ([_wp, C.POINTER(C.c_int)], C.c_int),
    "hyq_matmul_qkv_norm": ([_wp, _wp, _wp, _vp, _vp, _vp, C.c_float, _i64, _vp, _vp, _vp, _vp], C.c_int),
    "hyq_matmul_gate_up_silu_norm": ([_wp, _wp, _vp, _vp, _vp, C.c_float, _i64, _vp, _vp], C.c_int),
    "hyq_matmul_norm": ([_wp, _vp, _vp, _vp, C.c_float, _i64, _vp, _vp], C.c_int),
    "hyq_matmul_qkv": ([_wp, _wp, _wp, _vp, _i64, _vp, _vp, _vp, _vp], C.c_int),
    "hyq_matmul_gate_up_silu_batch": ([_wp, _wp, _vp, _i64, _vp, _vp], C.c_int),
    "hyq_q8_quantize": ([_vp, _i64, _vp, _vp, _vp, _vp], C.c_int),
    "hyq_gemv_q8": ([_wp, _vp, _vp, _vp, _vp, _vp], C.c_int),
    "hyq_gemv_qkv_q8": ([_wp, _wp, _wp, _vp, _vp, _vp, _vp, _vp, _vp, _vp], C.c_int),
    "hyq_matmul_gate_up_silu_q8": ([_wp, _wp, _vp, _vp, _vp, _vp, _vp], C.c_int),
    "hyq_gemv_int8": ([_wp, _vp, _vp, _vp], C.c_int),
    "hyq_gemv_qkv_int8": ([_wp, _wp, _wp, _vp, _vp, _vp, _vp, _vp], C.c_int),
    "hyq_matmul_gate_up_silu_int8": ([_wp, _wp, _vp, _vp, _vp], C.c_int),
    "hyq_matmul_noalloc": ([_wp, _vp, _i64, _vp, _vp], C.c_int),
    "hyq_set_launch_overlap": ([C.c_int], C.c_int),
    "hyq_set_gemm_precision": ([C.c_int], C.c_int),
    "hyq_set_peer_timeout_ms": ([C.c_int], C.c_int),
    "hyq_rope_table": ([_i64, C.c_int, C.c_float, _vp, _vp], C.c_int),
    "hyq_rms_norm": ([_vp, _vp, _i64, _i64, C.c_float, _vp, _vp], C.c_int),
    "hyq_embed": ([_wp, _vp, _i64, _vp, _vp], C.c_int),
    "hyq_rope_qk": ([_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _i64, _vp, _i64, _vp, _vp, C.c_float, C.c_int,
                     _vp, _vp, _vp], C.c_int),
    "hyq_attention_workspace_bytes": ([C.c_int, C.c_int, _i64, _i64, C.POINTER(C.c_size_t)], C.c_int),
    "hyq_attention": ([_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _i64, _vp, _i64, _vp, _vp, _vp], C.c_int),
    "hyq_add": ([_vp, _vp, _i64, _vp], C.c_int),
    "hyq_rope_qk_seqs": ([_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _i64, _vp, _i64, _vp, _vp, C.c_float,
                          C.c_int, _vp, _vp, _i64, _vp], C.c_int),
    "hyq_rope_attention": ([_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _i64, _vp, _vp, _vp, C.c_float,
                            C.c_int, _vp, _vp, _vp, _vp, _vp], C.c_int),
    "hyq_rope_attention_seqs": ([_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _i64, _vp, _i64, _vp, _vp,
                                 C.c_float, C.c_int, _vp, _vp, _i64, _vp, _vp, _vp], C.c_int),
    "hyq_attention_seqs": ([_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _i64, _vp, _i64, _i64, _vp, _vp, _vp],
                           C.c_int),
    "hyq_argmax_rows": ([_vp, _i64, _i64, _vp, _vp, _vp], C.c_int),
    "hyq_rope_qk_kv16": ([_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _i64, _vp, _i64, _vp, _vp, C.c_float,
                          C.c_int, _vp, _vp, _vp], C.c_int),
    "hyq_rope_qk_seqs_kv16": ([_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _i64, _vp, _i64, _vp, _vp,
                               C.c_float, C.c_int, _vp, _vp, _i64, _vp], C.c_int),
    "hyq_attention_kv16": ([_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _i64, _vp, _i64, _vp, _vp, _vp], C.c_int),
    "hyq_attention_seqs_kv16": ([_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _i64, _vp, _i64, _i64, _vp, _vp, _vp],
                                C.c_int),
    "hyq_gguf_open": ([C.c_char_p, C.c_int, C.POINTER(C.c_void_p)], C.c_int),
    "hyq_gguf_close": ([_vp], None),
    "hyq_gguf_profile": ([_vp], C.c_int),
    "hyq_gguf_tensor_count": ([_vp], _i64),
    "hyq_gguf_tensor_name": ([_vp, _i64, C.POINTER(C.c_char_p)], C.c_int),
    "hyq_gguf_tensor_info": ([_vp, C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_uint32), C.POINTER(C.c_int),
                              C.POINTER(C.c_int64), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)], C.c_int),
    "hyq_gguf_tensor_data": ([_vp, C.c_char_p, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t)], C.c_int),
    "hyq_gguf_upload": ([_vp, C.c_char_p, C.POINTER(C.c_void_p)], C.c_int),
    "hyq_gguf_meta_count": ([_vp], _i64),
    "hyq_gguf_meta_key": ([_vp, _i64, C.POINTER(C.c_char_p), C.POINTER(C.c_int)], C.c_int),
    "hyq_gguf_meta_u64": ([_vp, C.c_char_p, C.POINTER(C.c_uint64)], C.c_int),
    "hyq_gguf_meta_f64": ([_vp, C.c_char_p, C.POINTER(C.c_double)], C.c_int),
    "hyq_gguf_meta_bool": ([_vp, C.c_char_p, C.POINTER(C.c_int)], C.c_int),
    "hyq_gguf_meta_str": ([_vp, C.c_char_p, C.POINTER(C.c_char_p), C.POINTER(C.c_size_t)], C.c_int),
    "hyq_gguf_meta_array_len": ([_vp, C.c_char_p, C.POINTER(C.c_int64)], C.c_int),
    "hyq_dense_step_create": ([_vp, C.POINTER(C.c_void_p)], C.c_int),
    "hyq_dense_step_enqueue": ([_vp, _vp], C.c_int),
    "hyq_dense_step_free": ([_vp], None),
    "hyq_moe_router": ([_vp, _vp, _i64, _vp, _vp], C.c_int),
    "hyq_moe_route": ([_vp, _i64, C.c_int, _vp, C.c_int, C.c_int, C.c_float, _vp, _vp, _vp], C.c_int),
    "hyq_moe_group": ([_vp, _vp, _i64, C.c_int, C.c_int, _vp, _vp, _vp, _vp, _vp], C.c_int),
    "hyq_matmul_experts_gate_up_silu": ([_vp, _vp, _vp, _vp, _i64, _vp, _i64, _vp, _vp], C.c_int),
    "hyq_matmul_experts": ([_vp, _vp, _vp, _i64, _vp, _i64, _vp, _vp], C.c_int),
    "hyq_moe_combine": ([_vp, _vp, _i64, _i64, _vp, _vp, _vp, C.c_int, _vp, _vp], C.c_int),
    "hyq_add_rms_norm": ([_vp, _vp, _vp, _i64, _i64, C.c_float, _vp, _vp], C.c_int),
    "hyq_argmax": ([_vp, _i64, _vp, _vp, C.c_int, _vp, _vp], C.c_int),
    "hyq_peer_alloc": ([C.c_size_t, C.POINTER(_vp), _vp], C.c_int),
    "hyq_peer_open": ([_vp, C.POINTER(_vp)], C.c_int),
    "hyq_peer_close": ([_vp], C.c_int),
    "hyq_peer_free": ([_vp], C.c_int),
    "hyq_peer_allreduce": ([C.POINTER(C.c_uint64), C.c_int, C.c_int, _i64, _vp, _vp], C.c_int),
    "hyq_peer_exchange": ([C.POINTER(C.c_uint64), C.c_int, C.c_int, C.c_size_t, _vp, C.c_int, C.c_int, _vp, C.c_int,
                           _i64, _vp], C.c_int),
    "hyq_moe_ep_dispatch": ([C.POINTER(C.c_uint64), C.c_int, C.c_int, C.c_size_t, _i64, _vp, C.c_int, C.c_int, _vp,
                             _vp, C.c_int, C.c_int, _vp], C.c_int),
    "hyq_moe_ep_plan": ([C.POINTER(C.c_uint64), C.c_int, C.c_int, C.c_size_t, _i64, C.c_int, C.c_int, C.c_int, _vp,
                         _vp, _vp, _vp, _vp], C.c_int),
    "hyq_moe_ep_return": ([C.POINTER(C.c_uint64), C.c_int, C.c_int, C.c_size_t, _i64, _vp, C.c_int, _vp, _vp,
                           C.c_int, _vp], C.c_int),
    "hyq_moe_ep_home": ([C.POINTER(C.c_uint64), C.c_int, C.c_int, C.c_size_t, _i64, C.c_int, _vp, C.c_int, C.c_int,
                         _vp, _vp], C.c_int),
    "hyq_device_status": ([_vp, C.POINTER(C.c_uint32)], C.c_int),
}

for _name, (_args, _res) in _SIGS.items():
    _f = getattr(lib, _name)
    _f.argtypes = _args
    _f.restype = _res


def exported_symbols():
    """Names this binding requires from the library."""
    return sorted(_SIGS)


def last_error():
    return lib.hyq_last_error().decode(errors="replace")


def check(rc):
    if rc != HYQ_OK:
        raise HyqError(rc, last_error())
    return rc
