"""bf16 round-to-nearest-even, as Sheaf converts host f32 data to bf16.

Restates sheaf/src/core/dtype.rs:204-216 (f32_to_bf16_bits / bf16_bits_to_f32),
which sheaf/src/runtime/buffer_convert.rs:28-50 applies on the host before
uploading a bf16 argument.
"""
from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32)
    with np.errstate(over="ignore"):
        rounded = ((bits + np.uint32(0x7FFF) + ((bits >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16))
    nan = np.isnan(x)
    out = rounded.astype(np.uint16)
    out[nan] = ((bits[nan] >> np.uint32(16)).astype(np.uint16)) | np.uint16(0x0040)
    return out


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def round_bf16(x) -> np.ndarray:
    """f32 -> nearest bf16 (ties to even) -> f32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x)).reshape(np.shape(x))
