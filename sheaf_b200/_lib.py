"""ctypes binding of ``libsheaf_b200.so`` (the C ABI in ``include/``).

The library is built in-tree by :mod:`sheaf_b200.build`. There is no CPU
fallback: if the shared library is missing, loading raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libsheaf_b200.so"

ELEM_F16 = 0x21000010
ELEM_F32 = 0x21000020
ELEM_BF16 = 0x22000010
ELEM_I32 = 0x10000020

_lib = None


class GptConfig(C.Structure):
    """sb_gpt_config (include/sheaf_b200.h)."""
    _fields_ = [("n_layer", C.c_int32), ("n_head", C.c_int32), ("n_embd", C.c_int32), ("block_size", C.c_int32),
                ("vocab_size", C.c_int32), ("batch", C.c_int32), ("seq", C.c_int32), ("elem_type", C.c_uint32)]


class AdamwConfig(C.Structure):
    """sb_adamw_config (include/sheaf_b200.h)."""
    _fields_ = [("b1", C.c_float), ("b2", C.c_float), ("eps", C.c_float), ("weight_decay", C.c_float),
                ("max_norm", C.c_float)]


class SamplerConfig(C.Structure):
    """sb_sampler_config (include/sheaf_b200.h)."""
    _fields_ = [("n_new", C.c_int32), ("top_k", C.c_int32), ("temperature", C.c_float)]


class SessionStats(C.Structure):
    """sb_session_stats (include/sheaf_b200.h)."""
    _fields_ = [("calls", C.c_uint64), ("graph_captures", C.c_uint64), ("graph_replays", C.c_uint64),
                ("kernel_launches", C.c_uint64)]


_P = C.c_void_p
# name -> (restype, argtypes); every symbol declared in include/*.h.
SIGNATURES: dict[str, tuple] = {
    # sheaf_b200_ops.h
    "sb_op_matmul": (C.c_int, [C.c_uint32, _P, C.c_int64, C.c_int, _P, C.c_int64, C.c_int, C.c_int32, C.c_int32,
                               C.c_int32, _P, C.c_int64, C.c_uint32, _P, C.c_size_t, _P]),
    "sb_op_matmul_gelu": (C.c_int, [C.c_uint32, _P, C.c_int64, _P, C.c_int64, C.c_int32, C.c_int32, C.c_int32, _P,
                                    _P, C.c_int64, _P]),
    "sb_op_matmul_mul": (C.c_int, [C.c_uint32, _P, C.c_int64, C.c_int, _P, C.c_int64, C.c_int, C.c_int32, C.c_int32,
                                   C.c_int32, _P, C.c_int64, _P, C.c_int64, _P]),
    "sb_op_matmul_workspace_size": (C.c_size_t, [C.c_uint32, C.c_int, C.c_int, C.c_int32, C.c_int32, C.c_int32]),
    "sb_op_layernorm_fwd": (C.c_int, [C.c_uint32, _P, _P, _P, _P, _P, C.c_int32, C.c_int32, _P]),
    "sb_op_layernorm_bwd_workspace_size": (C.c_size_t, [C.c_int32, C.c_int32]),
    "sb_op_layernorm_bwd": (C.c_int, [C.c_uint32, _P, _P, _P, _P, _P, _P, _P, _P, C.c_size_t, C.c_int32, C.c_int32,
                                      _P]),
    "sb_op_layernorm_bwd_noalloc": (C.c_int, [C.c_uint32, _P, _P, _P, _P, _P, _P, _P, C.c_int32, C.c_int32, _P]),
    "sb_op_cross_entropy_workspace_size": (C.c_size_t, [C.c_int32]),
    "sb_op_cross_entropy": (C.c_int, [C.c_uint32, _P, C.c_int64, C.c_int32, C.c_int32, _P, _P, C.c_int64, _P,
                                      C.c_size_t, _P, _P]),
    "sb_op_gelu_fwd": (C.c_int, [C.c_uint32, _P, _P, C.c_int64, _P]),
    "sb_op_gelu_bwd": (C.c_int, [C.c_uint32, _P, _P, _P, C.c_int64, _P]),
    "sb_op_embedding_fwd": (C.c_int, [C.c_uint32, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P]),
    "sb_op_embedding_bwd_workspace_size": (C.c_size_t, [C.c_int32, C.c_int32]),
    "sb_op_embedding_bwd": (C.c_int, [C.c_uint32, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P,
                                      _P, _P, C.c_size_t, _P]),
    "sb_op_attention_fwd": (C.c_int, [C.c_uint32, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P]),
    "sb_op_attention_bwd_workspace_size": (C.c_size_t, [C.c_uint32, C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    "sb_op_attention_bwd": (C.c_int, [C.c_uint32, _P, _P, _P, _P, _P, _P, C.c_size_t, C.c_int32, C.c_int32,
                                      C.c_int32, C.c_int32, _P]),
    "sb_op_adamw_workspace_size": (C.c_size_t, [C.POINTER(C.c_int64), C.c_int32]),
    "sb_op_adamw_step": (C.c_int, [C.c_uint32, C.c_int32, C.POINTER(C.c_int64), C.POINTER(_P), C.POINTER(_P),
                                   C.POINTER(_P), C.POINTER(_P), C.POINTER(_P), C.POINTER(_P), C.POINTER(_P), _P, _P,
                                   _P, C.c_float, C.c_float, C.c_float, C.c_float, C.c_float, _P, _P, C.c_size_t,
                                   _P]),
    "sb_op_global_norm": (C.c_int, [C.c_uint32, C.c_int32, C.POINTER(C.c_int64), C.POINTER(_P), _P, _P, C.c_size_t,
                                    _P]),
    "sb_op_device_error": (C.c_int, []),
    # sheaf_b200.h
    "sb_status_is_ok": (C.c_bool, [_P]),
    "sb_status_code": (C.c_int, [_P]),
    "sb_status_message": (C.c_char_p, [_P]),
    "sb_status_free": (None, [_P]),
    "sb_session_create": (_P, [C.c_int, C.POINTER(_P)]),
    "sb_session_retain": (None, [_P]),
    "sb_session_release": (None, [_P]),
    "sb_session_synchronize": (_P, [_P, C.c_int64]),
    "sb_session_stream": (_P, [_P]),
    "sb_session_get_stats": (_P, [_P, C.POINTER(SessionStats)]),
    "sb_nccl_unique_id": (_P, [_P, C.c_size_t]),
    "sb_session_join_group": (_P, [_P, _P, C.c_size_t, C.c_int, C.c_int]),
    "sb_session_leave_group": (_P, [_P, C.c_int]),
    "sb_buffer_alloc_copy": (_P, [_P, C.POINTER(C.c_int64), C.c_size_t, C.c_uint32, _P, C.c_size_t, C.POINTER(_P)]),
    "sb_buffer_alloc": (_P, [_P, C.POINTER(C.c_int64), C.c_size_t, C.c_uint32, C.POINTER(_P)]),
    "sb_buffer_h2d": (_P, [_P, _P, C.c_size_t]),
    "sb_buffer_d2h": (_P, [_P, _P, C.c_size_t, C.c_int64]),
    "sb_buffer_retain": (None, [_P]),
    "sb_buffer_release": (None, [_P]),
    "sb_buffer_release_many": (None, [_P, C.c_size_t]),
    "sb_buffer_rank": (C.c_size_t, [_P]),
    "sb_buffer_dim": (C.c_int64, [_P, C.c_size_t]),
    "sb_buffer_elem_type": (C.c_uint32, [_P]),
    "sb_buffer_byte_length": (C.c_size_t, [_P]),
    "sb_buffer_device_ptr": (_P, [_P]),
    "sb_module_load_stablehlo": (_P, [_P, C.c_char_p, C.c_size_t, C.POINTER(C.c_char_p)]),
    "sb_op_get_batch": (C.c_int, [_P, C.c_int64, _P, C.c_int32, C.c_int32, _P, _P, _P]),
    "sb_op_random_split": (C.c_int, [_P, C.c_int32, _P, _P]),
    "sb_safetensors_save": (_P, [_P, C.c_char_p, C.POINTER(C.c_char_p), C.POINTER(_P), C.c_size_t]),
    "sb_safetensors_open": (_P, [C.c_char_p, C.POINTER(_P)]),
    "sb_safetensors_count": (C.c_size_t, [_P]),
    "sb_safetensors_key": (C.c_char_p, [_P, C.c_size_t]),
    "sb_safetensors_info": (_P, [_P, C.c_size_t, C.POINTER(C.c_uint32), C.POINTER(C.c_int64), C.c_size_t,
                                 C.POINTER(C.c_size_t)]),
    "sb_safetensors_read": (_P, [_P, _P, C.c_size_t, C.POINTER(_P)]),
    "sb_safetensors_close": (None, [_P]),
    "sb_module_create_gpt_vag": (_P, [_P, C.c_char_p, C.POINTER(GptConfig)]),
    "sb_module_create_gpt_train": (_P, [_P, C.c_char_p, C.POINTER(GptConfig), C.POINTER(AdamwConfig)]),
    "sb_module_create_gpt_sampler": (_P, [_P, C.c_char_p, C.POINTER(GptConfig), C.POINTER(SamplerConfig)]),
    "sb_module_describe": (_P, [_P, C.c_char_p, C.c_char_p, C.c_size_t]),
    "sb_stablehlo_validate": (_P, [C.c_char_p, C.c_size_t, C.c_char_p, C.c_size_t]),
    "sb_call": (_P, [_P, C.c_char_p, C.POINTER(_P), C.c_size_t, C.POINTER(_P), C.c_size_t, C.POINTER(C.c_size_t)]),
}


class LibraryMissing(RuntimeError):
    pass


def lib() -> C.CDLL:
    """Returns the loaded library, raising if it has not been built."""
    global _lib
    if _lib is None:
        path = Path(os.environ.get("SHEAF_B200_LIB", LIB_PATH))
        if not path.exists():
            raise LibraryMissing(f"{path} not found; run `python -m sheaf_b200.build` (needs nvcc)")
        handle = C.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed with sheaf_b200 error code {rc}")
