"""ctypes binding of libtinybrain_cuda.so (declared in include/tinybrain_cuda.h).

The library is built in-tree (tinybrain_b200/libtinybrain_cuda.so).  There is
no fallback: if the shared object is missing or a call fails, a TinyBrainError
is raised.
"""
import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
# TB_LIBRARY: load another in-tree build of the library (experiments)
LIB_PATH = os.environ.get("TB_LIBRARY") or os.path.join(_HERE, "libtinybrain_cuda.so")

TB_OK = 0
STATUS_NAMES = {
    0: "TB_OK", 1: "TB_ERR_INVALID_ARGUMENT", 2: "TB_ERR_CUDA", 3: "TB_ERR_OUT_OF_MEMORY",
    4: "TB_ERR_UNSUPPORTED", 5: "TB_ERR_PAGE_POOL_EXHAUSTED", 6: "TB_ERR_FORMAT",
    7: "TB_ERR_NO_DEVICE", 8: "TB_ERR_DEVICE_TIMEOUT", 9: "TB_ERR_STATE", 10: "TB_ERR_DEVICE_FAULT",
}


class TinyBrainError(RuntimeError):
    def __init__(self, status, message):
        self.status = status
        self.status_name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{self.status_name}: {message}")


class QTensorDesc(C.Structure):
    _fields_ = [
        ("precision", C.c_int32),
        ("in_features", C.c_int64),
        ("out_features", C.c_int64),
        ("group_size", C.c_int64),
        ("data", C.c_void_p),
        ("data_bytes", C.c_int64),
        ("scales", C.c_void_p),
        ("num_scales", C.c_int64),
        ("zero_points", C.c_void_p),
        ("num_zero_points", C.c_int64),
    ]


class ModelConfigC(C.Structure):
    _fields_ = [
        ("num_layers", C.c_int32), ("hidden_dim", C.c_int32), ("num_heads", C.c_int32),
        ("num_kv_heads", C.c_int32), ("vocab_size", C.c_int32), ("max_seq_len", C.c_int32),
        ("intermediate_dim", C.c_int32), ("architecture", C.c_int32), ("rms_eps", C.c_float),
    ]


class SamplerConfigC(C.Structure):
    _fields_ = [
        ("temperature", C.c_float), ("top_k", C.c_int32), ("has_top_p", C.c_int32), ("top_p", C.c_float),
        ("repetition_penalty", C.c_float), ("has_seed", C.c_int32), ("seed", C.c_uint64),
    ]


TOKEN_CALLBACK = C.CFUNCTYPE(C.c_int32, C.c_void_p, C.c_int32, C.c_int32, C.c_int32)

_P = C.c_void_p
_I32, _I64, _F = C.c_int32, C.c_int64, C.c_float
_PI32, _PI64, _PF, _PU64 = C.POINTER(C.c_int32), C.POINTER(C.c_int64), C.POINTER(C.c_float), C.POINTER(C.c_uint64)

# name -> argtypes (every function returns tb_status unless listed in _RESTYPES)
SIGNATURES = {
    "tb_abi_version": [],
    "tb_last_error": [],
    "tb_status_string": [C.c_int],
    "tb_device_count": [_PI32],
    "tb_rng_seed_state": [C.c_uint64, _PU64],
    "tb_rng_fill_normal": [_PU64, _F, _F, _I64, _P],
    "tb_context_create": [_I32, C.POINTER(_P)],
    "tb_context_destroy": [_P],
    "tb_context_synchronize": [_P],
    "tb_context_stream": [_P],
    "tb_context_check_device": [_P],
    "tb_debug_expire_wait": [_P, _I32],
    "tb_quantize_int8_per_channel": [_P, _P, _I64, _I64, _P, _P],
    "tb_quantize_int4_group": [_P, _P, _I64, _I64, _P, _P, _P],
    "tb_quantize_int8_per_channel_dev": [_P, _P, _I64, _I64, _P, _P],
    "tb_quantize_int4_group_dev": [_P, _P, _I64, _I64, _P, _P, _P],
    "tb_qweight_upload": [_P, C.POINTER(QTensorDesc), C.POINTER(_P)],
    "tb_qweight_free": [_P],
    "tb_matmul_quantized": [_P, _P, _I64, _P, _P],
    "tb_matmul_quantized_dev": [_P, _P, _I64, _P, _P],
    "tb_qgemv_stream_time": [_P, _P, _I32, _P, _I64, _P, _I32, _I32, _PF],
    "tb_attention_decode": [_P, _P, _P, _P, _I64, _I32, _I32, _I32, _P],
    "tb_paged_attention_dev": [_P, _P, _I32, _P, _P, _I32, _P, _I32, _I32, _I32, _I32, _I32, _I32, _P],
    "tb_paged_attention_dev_noalloc": [_P, _P, _I32, _P, _P, _I32, _P, _I32, _I32, _I32, _I32, _I32, _I32, _P],
    "tb_paged_attention_noalloc_status": [_P, _I32],
    "tb_model_create": [_P, C.POINTER(ModelConfigC), C.POINTER(_P)],
    "tb_model_free": [_P],
    "tb_tp_unique_id": [_P],
    "tb_context_init_tp": [_P, _P, _I32, _I32],
    "tb_model_set_tensor_parallel": [_P, _I32, _I32],
    "tb_runner_trace_launches": [_P, _P, _P, _P],
    "tb_runner_tp_handle": [_P, _P],
    "tb_runner_tp_connect": [_P, _P],
    "tb_model_set_embedding": [_P, _P],
    "tb_model_set_final_norm": [_P, _P],
    "tb_model_set_layer_norms": [_P, _I32, _P, _P],
    "tb_model_set_projection": [_P, _I32, _I32, C.POINTER(QTensorDesc), _P],
    "tb_model_set_output": [_P, C.POINTER(QTensorDesc), _P],
    "tb_model_finalize": [_P],
    "tb_model_weight_bytes": [_P, _PI64],
    "tb_runner_create": [_P, _I32, _I32, C.POINTER(_P)],
    "tb_runner_free": [_P],
    "tb_runner_reset": [_P],
    "tb_runner_step": [_P, _I32, _P, _PI32],
    "tb_runner_step_observed": [_P, _I32, _P, _PI32, _P, _P, _I64, _P],
    "tb_runner_position": [_P, _I32, _PI64],
    "tb_runner_kv_length": [_P, _I32, _PI64],
    "tb_runner_page_status": [_P, _I32, _P, _I64],
    "tb_runner_max_pages": [_P, _PI64],
    "tb_runner_generate": [_P, _P, _P, _I32, _I32, _P, _I32, _P, _P, TOKEN_CALLBACK, _P],
    "tb_runner_prefill_device": [_P, _P, _P, _I32, _I32],
    "tb_runner_decode_device": [_P, _I32, _PF],
    "tb_runner_read_tokens": [_P, _P, _P],
    "tb_runner_profile_step": [_P, _P, _P, _P, _PI32],
    "tb_runner_io_bytes": [_P, _PI64, _PI64, _I32],
    "tb_runner_set_persistent": [_P, _I32],
    "tb_runner_get_persistent": [_P, _PI32],
    "tb_runner_set_chunked_prefill": [_P, _I32],
    "tb_runner_set_sampler": [_P, _P],
    "tb_runner_perplexity": [_P, _P, _P, _I32, _P, _P],
    "tb_dequantize": [_P, _P, _P],
    "tb_requantize_int4": [_P, _P, _I64, _P, _P, _P],
    "tb_sample_detailed": [_P, _P, _I32, _P, _P, _I32, _PU64, _PI32, _PF, _PF],
    "tb_runner_token_stats": [_P, _I32, _I32, _P, _P],
    "tb_runner_set_step_history": [_P, _P, _I32],
    "tb_runner_step_stats": [_P, _PF, _PF],
    "tb_runner_debug_read": [_P, _I32, _P, _I64],
    "tb_runner_trace_step": [_P, _P, _I64, _PI32, _PI32],
}
_RESTYPES = {
    "tb_abi_version": C.c_int32,
    "tb_last_error": C.c_char_p,
    "tb_status_string": C.c_char_p,
    "tb_context_stream": C.c_void_p,
}

_lib = None


def load():
    """Load (once) and return the ctypes handle; raises if the library is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m tinybrain_b200.build` "
            "(there is no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _RESTYPES.get(name, C.c_int)
    _lib = lib
    return lib


def last_error():
    return load().tb_last_error().decode(errors="replace")


def check(status):
    if status != TB_OK:
        raise TinyBrainError(status, last_error())
    return status


def call(name, *args):
    return check(getattr(load(), name)(*args))


def exported_symbols():
    return list(SIGNATURES)
