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

# name -> (restype, argtypes); every symbol declared in include/*.h.
SIGNATURES: dict[str, tuple] = {
    "sb_op_matmul": (C.c_int, [C.c_uint32, C.c_void_p, C.c_int64, C.c_int, C.c_void_p, C.c_int64, C.c_int,
                               C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_int64, C.c_uint32, C.c_void_p,
                               C.c_size_t, C.c_void_p]),
    "sb_op_matmul_workspace_size": (C.c_size_t, [C.c_uint32, C.c_int, C.c_int, C.c_int32, C.c_int32, C.c_int32]),
    "sb_op_device_error": (C.c_int, []),
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
