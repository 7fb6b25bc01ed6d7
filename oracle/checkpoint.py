"""safetensors save / load as the reference writes and reads them (test-only).

Restates sheaf/src/interpreter/builtins/safetensors.rs:
  * save_safetensors (:200-239): pytree flattened to dot-separated keys
    (dicts by key, lists by index, flatten_into :255-310), entries sorted by
    key, header = compact JSON of {key: {"data_offsets": [a, b], "dtype": D,
    "shape": [...]}} (serde_json's map keeps keys sorted), padded with spaces
    so 8 + len(header) is a multiple of 8, then the little-endian data.
  * load_safetensors (:13-81) with decode_raw (:83-133): F32, F64 -> f32,
    F16, BF16, I32, I64 -> i32 (through f32), BOOL, U8 -> i32; keys nested on
    '.', contiguous numeric siblings become lists (:135-190).
"""
from __future__ import annotations

import json
import struct

import numpy as np

from . import dtype as odt

_DT = {"F32": np.float32, "F16": np.float16, "I32": np.int32, "F64": np.float64, "I64": np.int64, "U8": np.uint8,
       "BOOL": np.uint8}


def flatten(tree, prefix: str = "") -> list[tuple[str, object]]:
    """flatten_into: (key, leaf) pairs; a leaf at the root is named 'tensor'."""
    if isinstance(tree, dict):
        out = []
        for k in sorted(tree):
            out += flatten(tree[k], f"{prefix}.{k}" if prefix else str(k))
        return out
    if isinstance(tree, (list, tuple)):
        out = []
        for i, v in enumerate(tree):
            out += flatten(v, f"{prefix}.{i}" if prefix else str(i))
        return out
    return [(prefix or "tensor", tree)]


def nest(flat: dict[str, object]):
    """nest_flat_keys + tree_to_value."""
    root: dict = {}
    for key in sorted(flat):
        node = root
        segs = key.split(".")
        for s in segs[:-1]:
            node = node.setdefault(s, {})
        node[segs[-1]] = flat[key]

    def fix(node):
        if not isinstance(node, dict):
            return node
        items = {k: fix(v) for k, v in node.items()}
        if items and all(k.isdigit() for k in items) and max(int(k) for k in items) + 1 == len(items):
            return [items[str(i)] for i in range(len(items))]
        return items
    return fix(root)


def save_bytes(entries: list[tuple[str, str, tuple, bytes]]) -> bytes:
    """entries: (key, dtype string, shape, raw little-endian bytes)."""
    entries = sorted(entries, key=lambda e: e[0])
    header, off = {}, 0
    data = bytearray()
    for key, dt, shape, raw in entries:
        header[key] = {"data_offsets": [off, off + len(raw)], "dtype": dt, "shape": list(shape)}
        data += raw
        off += len(raw)
    # serde_json writes strings as UTF-8, escaping only '"', '\\' and control
    # characters (\b \f \n \r \t, else \u00xx): json's ensure_ascii=False form
    h = json.dumps(header, separators=(",", ":"), sort_keys=True, ensure_ascii=False).encode("utf-8")
    h += b" " * ((8 - (8 + len(h)) % 8) % 8)
    return struct.pack("<Q", len(h)) + h + bytes(data)


def entry_of(key: str, a: np.ndarray, dt: str) -> tuple[str, str, tuple, bytes]:
    """A host array as the reference stores a tensor of element type dt."""
    a = np.asarray(a)
    if dt == "BF16":
        raw = odt.f32_to_bf16_bits(a.astype(np.float32)).astype("<u2").tobytes()
    elif dt == "F16":
        raw = a.astype("<f2").tobytes()
    elif dt == "I32":
        raw = a.astype("<i4").tobytes()
    else:
        raw = a.astype("<f4").tobytes()
    return key, dt, a.shape, raw


def load_bytes(data: bytes) -> dict[str, tuple[str, np.ndarray]]:
    """key -> (element type after decode_raw, values as f32 / i32 / bf16 bits)."""
    (hsize,) = struct.unpack("<Q", data[:8])
    header = json.loads(data[8:8 + hsize])
    body = data[8 + hsize:]
    out = {}
    for key, info in header.items():
        if key == "__metadata__":
            continue
        a, b = info["data_offsets"]
        raw, dt, shape = body[a:b], info["dtype"], tuple(info["shape"])
        if dt == "BF16":
            v = odt.bf16_bits_to_f32(np.frombuffer(raw, "<u2"))
            kind = "BF16"
        elif dt in ("F32", "F64", "F16"):
            v = np.frombuffer(raw, "<" + np.dtype(_DT[dt]).str[1:]).astype(np.float32)
            kind = "F16" if dt == "F16" else "F32"
        elif dt in ("I64",):
            v = np.frombuffer(raw, "<i8").astype(np.float32).astype(np.int32)
            kind = "I32"
        elif dt in ("U8", "BOOL"):
            u = np.frombuffer(raw, np.uint8)
            v = (u != 0).astype(np.int32) if dt == "BOOL" else u.astype(np.int32)
            kind = "I32"
        else:
            v = np.frombuffer(raw, "<i4").astype(np.int32)
            kind = "I32"
        out[key] = (kind, v.reshape(shape))
    return out
