"""Checkpoint format on the host (no GPU): the safetensors oracle against an
independent implementation (the `safetensors` package), the library's header
parser (sb_safetensors_open / info) on files from both, its errors on broken
files, and the pytree key flattening of the reference's io "save"."""
import struct

import numpy as np
import pytest

from oracle import checkpoint as ock
from oracle import data as odata
from oracle import prng

st_np = pytest.importorskip("safetensors.numpy")

F32, BF16, F16, I32 = 0x21000020, 0x22000010, 0x21000010, 0x10000020


def _arrays():
    rng = np.random.default_rng(0)
    return {
        "params.lm_head.weight": rng.standard_normal((65, 8)).astype(np.float32),
        "params.transformer.h.0.attn.c_attn.weight": rng.standard_normal((24, 8)).astype(np.float16),
        "t": np.array(3.0, np.float32),
        "ids": rng.integers(-5, 70000, (4, 5)).astype(np.int32),
    }


def _dt(a):
    return {np.float32: "F32", np.float16: "F16", np.int32: "I32"}[a.dtype.type]


def test_oracle_writer_reads_back_with_the_safetensors_package(tmp_path):
    arrs = _arrays()
    data = ock.save_bytes([ock.entry_of(k, v, _dt(v)) for k, v in arrs.items()])
    (hsize,) = struct.unpack("<Q", data[:8])
    assert (8 + hsize) % 8 == 0  # data section 8-byte aligned (safetensors.rs:226-229)
    p = tmp_path / "a.safetensors"
    p.write_bytes(data)
    back = st_np.load_file(str(p))
    assert sorted(back) == sorted(arrs)
    for k, v in arrs.items():
        assert back[k].dtype == v.dtype and np.array_equal(back[k], v)


def test_oracle_reader_reads_files_of_the_safetensors_package(tmp_path):
    arrs = _arrays()
    arrs["w64"] = np.linspace(-2, 2, 7, dtype=np.float64)
    arrs["i64"] = np.array([1, -2, 3], np.int64)
    arrs["mask"] = np.array([True, False, True])
    arrs["bytes"] = np.array([0, 7, 255], np.uint8)
    p = tmp_path / "b.safetensors"
    st_np.save_file(arrs, str(p), metadata={"format": "np"})
    got = ock.load_bytes(p.read_bytes())
    assert got["w64"][0] == "F32" and np.array_equal(got["w64"][1], arrs["w64"].astype(np.float32))
    assert got["i64"][0] == "I32" and np.array_equal(got["i64"][1], [1, -2, 3])
    assert got["mask"][0] == "I32" and np.array_equal(got["mask"][1], [1, 0, 1])
    assert got["bytes"][0] == "I32" and np.array_equal(got["bytes"][1], [0, 7, 255])
    assert np.array_equal(got["t"][1], arrs["t"])


def _open(path):
    import ctypes as C

    from sheaf_b200.runtime import _check, lib

    f = C.c_void_p()
    _check(lib().sb_safetensors_open(str(path).encode(), C.byref(f)))
    L = lib()
    out = {}
    for i in range(L.sb_safetensors_count(f)):
        elem = C.c_uint32()
        shape = (C.c_int64 * 8)()
        rank = C.c_size_t()
        _check(L.sb_safetensors_info(f, i, C.byref(elem), shape, 8, C.byref(rank)))
        out[L.sb_safetensors_key(f, i).decode()] = (elem.value, tuple(shape[: rank.value]))
    L.sb_safetensors_close(f)
    return out


def test_library_parses_headers_of_both_writers(tmp_path):
    arrs = _arrays()
    p1 = tmp_path / "o.safetensors"
    p1.write_bytes(ock.save_bytes([ock.entry_of(k, v, _dt(v)) for k, v in arrs.items()] +
                                  [ock.entry_of("bf", np.ones((2, 3), np.float32), "BF16")]))
    info = _open(p1)
    assert list(info) == sorted(list(arrs) + ["bf"])
    assert info["bf"] == (BF16, (2, 3)) and info["t"] == (F32, ()) and info["ids"] == (I32, (4, 5))
    assert info["params.transformer.h.0.attn.c_attn.weight"] == (F16, (24, 8))
    p2 = tmp_path / "p.safetensors"
    st_np.save_file({"a": np.zeros((3,), np.float64), "b": np.zeros((2, 2), np.int64)}, str(p2),
                    metadata={"k": "v"})
    assert _open(p2) == {"a": (F32, (3,)), "b": (I32, (2, 2))}


def test_library_rejects_broken_files(tmp_path):
    from sheaf_b200.runtime import SheafB200Error

    good = ock.save_bytes([ock.entry_of("w", np.ones((4, 4), np.float32), "F32")])
    (hsize,) = struct.unpack("<Q", good[:8])
    cases = {
        "short": good[:5],
        "header_too_big": struct.pack("<Q", 1 << 40) + good[8:],
        "not_json": struct.pack("<Q", 8) + b"{{{{{{{{" + good[8 + hsize:],
        "truncated_data": good[:-4],
        "bad_dtype": good.replace(b'"F32"', b'"X32"'),
        "bad_count": good.replace(b"[4,4]", b"[4,5]"),
    }
    for name, data in cases.items():
        p = tmp_path / f"{name}.safetensors"
        p.write_bytes(data)
        with pytest.raises(SheafB200Error):
            _open(p)
    with pytest.raises(SheafB200Error):
        _open(tmp_path / "missing.safetensors")


def test_pytree_keys_match_the_reference_flattening():
    from sheaf_b200.runtime import _flatten_tree, _nest_keys

    tree = {"params": {"h": [{"w": 1, "b": 2}, {"w": 3, "b": 4}], "ln": 5}, "t": 6, "m": [7, [8, 9]]}
    flat = _flatten_tree(tree)
    assert flat == ock.flatten(tree)
    assert [k for k, _ in flat] == ["m.0", "m.1.0", "m.1.1", "params.h.0.b", "params.h.0.w", "params.h.1.b",
                                    "params.h.1.w", "params.ln", "t"]
    assert _nest_keys(dict(flat)) == ock.nest(dict(flat)) == tree
    assert _flatten_tree(np.zeros(2))[0][0] == "tensor"


def test_get_batch_oracle_properties():
    data = np.arange(1000, dtype=np.float32) * 3.0
    for seed in range(5):
        x, y, starts = odata.get_batch(data, prng.random_key(seed), 64, 16)
        assert x.shape == y.shape == (16, 64)
        assert np.array_equal(y, x + 3.0)  # y is x shifted by one position
        assert (starts >= 0).all() and (starts <= 1000 - 64 - 2).all()
