"""ctypes binding of libbeacon_cuda.so (declared in include/beacon_cuda.h).

This is the binding a host program would write against the C ABI; the Rust
`beacon-cuda` crate would bind the same symbols through bindgen. Loading
fails loudly when the library has not been built: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import re

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG, "lib", "libbeacon_cuda.so")
HEADER = os.path.join(os.path.dirname(_PKG), "include", "beacon_cuda.h")

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_OUT_OF_MEMORY = 2
ERR_SHAPE_MISMATCH = 3
ERR_UNSUPPORTED_DTYPE = 4
ERR_KERNEL_LAUNCH = 5
ERR_CUDA = 6
ERR_CONTEXT_OVERFLOW = 7
ERR_COMM = 8
ERR_DEVICE_TIMEOUT = 9
ERR_UNKNOWN = 99

DTYPE_F32, DTYPE_F16, DTYPE_BF16, DTYPE_I32, DTYPE_I8 = 0, 1, 2, 3, 4
DTYPE_Q4_0, DTYPE_Q4_K, DTYPE_Q5_K, DTYPE_Q6_K, DTYPE_Q8_0 = 100, 101, 102, 103, 104
DTYPE_Q4_1, DTYPE_Q5_0, DTYPE_Q5_1, DTYPE_Q2_K, DTYPE_Q3_K, DTYPE_Q8_K = 105, 106, 107, 108, 109, 110

NIBBLE_REF_INTERLEAVED, NIBBLE_GGUF_SPLIT = 0, 1
NUMERICS_FAST, NUMERICS_EXACT, NUMERICS_REF_RTZ = 0, 1, 2

W_EMBED, W_FINAL_NORM, W_LM_HEAD = 0, 1, 2
W_ATTN_NORM, W_Q, W_K, W_V, W_O, W_FFN_NORM, W_GATE, W_UP, W_DOWN = 10, 11, 12, 13, 14, 15, 16, 17, 18


class SamplingParams(ctypes.Structure):
    """BeaconCudaSamplingParams: GenerationParams' sampling fields (params.rs:6-31)."""
    _fields_ = [("temperature", ctypes.c_float), ("has_top_k", ctypes.c_int32), ("top_k", ctypes.c_int32),
                ("has_top_p", ctypes.c_int32), ("top_p", ctypes.c_float), ("has_min_p", ctypes.c_int32),
                ("min_p", ctypes.c_float), ("repeat_penalty", ctypes.c_float)]


def sampling_params(temperature=0.0, top_k=None, top_p=None, min_p=None, repeat_penalty=1.0) -> SamplingParams:
    """None means the Option field is None."""
    return SamplingParams(temperature, top_k is not None, top_k or 0, top_p is not None,
                          0.0 if top_p is None else top_p, min_p is not None, 0.0 if min_p is None else min_p,
                          repeat_penalty)


class BeaconCudaError(RuntimeError):
    """A non-OK status from the C ABI, with beacon_cuda_last_error_message()."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[status {status}] {message}")
        self.status = status


class ModelConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "vocab_size", "hidden_size", "num_layers", "num_heads", "num_kv_heads", "head_dim",
        "intermediate_size", "max_context", "max_batch")] + [
        ("rope_theta", ctypes.c_float), ("rms_norm_eps", ctypes.c_float)] + [
        (n, ctypes.c_int32) for n in (
            "numerics", "kv_dtype", "kv_persist", "causal_prefill", "tp_size", "tp_rank")]


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_PP = ctypes.POINTER(ctypes.c_void_p)

SIGNATURES = {
    "beacon_cuda_context_create": (_I32, [_I32, _PP]),
    "beacon_cuda_context_destroy": (None, [_P]),
    "beacon_cuda_context_set_numerics": (_I32, [_P, _I32]),
    "beacon_cuda_context_set_wait_limit": (_I32, [_P, _I64]),
    "beacon_cuda_stream_create": (_I32, [_P, _PP]),
    "beacon_cuda_stream_wrap": (_I32, [_P, _P, _PP]),
    "beacon_cuda_stream_destroy": (None, [_P]),
    "beacon_cuda_stream_synchronize": (_I32, [_P]),
    "beacon_cuda_tensor_upload": (_I32, [_P, _P, _P, _SZ, _I32, _I32, _PP]),
    "beacon_cuda_tensor_from_device_blocks": (_I32, [_P, _P, _P, _SZ, _I32, _I32, _PP]),
    "beacon_cuda_tensor_zeros": (_I32, [_P, _P, _SZ, _I32, _PP]),
    "beacon_cuda_tensor_wrap_device": (_I32, [_P, _P, _P, _SZ, _I32, _PP]),
    "beacon_cuda_tensor_destroy": (None, [_P]),
    "beacon_cuda_tensor_shape": (_I32, [_P, _P, ctypes.POINTER(_SZ)]),
    "beacon_cuda_tensor_dtype": (_I32, [_P, ctypes.POINTER(_I32)]),
    "beacon_cuda_tensor_device_ptr": (_I32, [_P, _PP]),
    "beacon_cuda_tensor_eval": (_I32, [_P, _P]),
    "beacon_cuda_tensor_read_f32": (_I32, [_P, _P, _SZ]),
    "beacon_cuda_tensor_read_raw": (_I32, [_P, _P, _SZ]),
    "beacon_cuda_op_matmul": (_I32, [_P, _P, _P, _P, _PP]),
    "beacon_cuda_op_quantized_matmul": (_I32, [_P, _P, _P, _P, _P, _P, _I32, _I32, _PP]),
    "beacon_cuda_op_rms_norm": (_I32, [_P, _P, _P, _P, ctypes.c_float, _PP]),
    "beacon_cuda_op_rope": (_I32, [_P, _P, _P, _I32, ctypes.c_float, _I32, _P, _PP]),
    "beacon_cuda_op_silu": (_I32, [_P, _P, _P, _PP]),
    "beacon_cuda_op_softmax": (_I32, [_P, _P, _P, _I32, _PP]),
    "beacon_cuda_op_attention": (_I32, [_P, _P, _P, _P, _P, _P, ctypes.c_float, _I32, _PP]),
    "beacon_cuda_op_add": (_I32, [_P, _P, _P, _P, _PP]),
    "beacon_cuda_op_elementwise_mul": (_I32, [_P, _P, _P, _P, _PP]),
    "beacon_cuda_op_kv_cache_update": (_I32, [_P, _P, _P, _P, _P, _P, _I64, _PP, _PP]),
    "beacon_cuda_op_reshape": (_I32, [_P, _P, _P, _P, _SZ, _PP]),
    "beacon_cuda_op_transpose": (_I32, [_P, _P, _P, _PP]),
    "beacon_cuda_op_swapaxes": (_I32, [_P, _P, _P, _I32, _I32, _PP]),
    "beacon_cuda_op_embedding": (_I32, [_P, _P, _P, _P, _PP]),
    "beacon_cuda_create_token_tensor": (_I32, [_P, _P, _SZ, _PP]),
    "beacon_cuda_op_argmax": (_I32, [_P, _P, _P, _PP]),
    "beacon_cuda_profile_quantized_matmul": (_I32, [_P, _P, _PP, _I32, _P, _I32, ctypes.POINTER(ctypes.c_float),
                                                    ctypes.POINTER(ctypes.c_uint64)]),
    "beacon_cuda_op_sample": (_I32, [_P, _P, _P, _P, _P, _P, _PP]),
    "beacon_cuda_op_dequantize_to_f16": (_I32, [_P, _P, _P, _PP]),
    "beacon_cuda_op_quantize": (_I32, [_P, _P, _P, _I32, _I32, _PP]),
    "beacon_cuda_quantize_blocks": (_I32, [_P, _P, _P, _I64, _I64, _I32, _I32, _P]),
    "beacon_cuda_quantized_matvec_noalloc": (_I32, [_P, _P, _P, _I32, _I32, _P]),
    "beacon_cuda_model_create": (_I32, [_P, _P, _PP]),
    "beacon_cuda_model_destroy": (None, [_P]),
    "beacon_cuda_model_set_weight": (_I32, [_P, _I32, _I32, _P, _I32, _I32, _I32]),
    "beacon_cuda_model_reset": (_I32, [_P]),
    "beacon_cuda_model_forward": (_I32, [_P, _P, _P, _I32, _I32, _P]),
    "beacon_cuda_model_decode_step": (_I32, [_P, _P, _P, _I32, _I32, _P, _P]),
    "beacon_cuda_model_decode_step_sampled": (_I32, [_P, _P, _P, _I32, _I32, _P, _P, _P, _I32, _P]),
    "beacon_cuda_model_decode_step_device": (_I32, [_P, _P, _P, _I32, _I32, _P, _P]),
    "beacon_cuda_model_synchronize": (_I32, [_P, _P]),
    "beacon_cuda_model_profile_linear": (_I32, [_P, _P, _I32, _I32, _I32, ctypes.POINTER(ctypes.c_float),
                                                ctypes.POINTER(ctypes.c_uint64)]),
    "beacon_cuda_model_fill_kv_random": (_I32, [_P, _I32, ctypes.c_uint64]),
    "beacon_cuda_model_launches_per_step": (_I32, [_P, _I32, _I32, ctypes.POINTER(_I32)]),
    "beacon_cuda_stream_handle": (_I32, [_P, _PP]),
    "beacon_cuda_model_memory": (_I32, [_P, ctypes.POINTER(ctypes.c_uint64)]),
    "beacon_cuda_gguf_open": (_I32, [ctypes.c_char_p, _PP]),
    "beacon_cuda_gguf_close": (None, [_P]),
    "beacon_cuda_gguf_version": (_I32, [_P, ctypes.POINTER(ctypes.c_uint32)]),
    "beacon_cuda_gguf_tensor_count": (_I32, [_P, ctypes.POINTER(_I64)]),
    "beacon_cuda_gguf_tensor_info": (_I32, [_P, _I64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_I32), _P,
                                            ctypes.POINTER(_SZ), _PP, ctypes.POINTER(ctypes.c_uint64)]),
    "beacon_cuda_gguf_find_tensor": (_I32, [_P, ctypes.c_char_p, ctypes.POINTER(_I64)]),
    "beacon_cuda_gguf_get_int": (_I32, [_P, ctypes.c_char_p, ctypes.POINTER(_I64)]),
    "beacon_cuda_gguf_get_float": (_I32, [_P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)]),
    "beacon_cuda_gguf_get_string": (_I32, [_P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p)]),
    "beacon_cuda_gguf_get_array_len": (_I32, [_P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64)]),
    "beacon_cuda_gguf_model_config": (_I32, [_P, _P]),
    "beacon_cuda_model_load_gguf": (_I32, [_P, _P]),
    "beacon_cuda_comm_unique_id": (_I32, [_P]),
    "beacon_cuda_comm_init": (_I32, [_P, _I32, _I32, _P, _I32]),
    "beacon_cuda_op_all_reduce_f32": (_I32, [_P, _P, _P]),
    "beacon_cuda_last_error_message": (ctypes.c_char_p, []),
}


def header_symbols() -> list[str]:
    """Every function name declared in include/beacon_cuda.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(beacon_cuda_[a-z0-9_]+)\s*\(", text)))


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libbeacon_cuda.so is not built ({LIB_PATH}); run __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != OK:
        msg = lib().beacon_cuda_last_error_message()
        raise BeaconCudaError(status, msg.decode() if msg else "")
