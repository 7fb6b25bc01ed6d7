"""Device-direct checkpoints and the device data path on the GPU.

* sb_safetensors_save writes the file the reference's save_safetensors
  writes for the same tensors, byte for byte (oracle.checkpoint);
* sb_safetensors_read loads every dtype decode_raw accepts as the oracle
  decodes it; save -> load round trips are bitwise, also past the staging
  chunk size;
* a train-step state saved, reloaded into a fresh session and continued
  gives the same next step as continuing in place (train.shf resume);
* random-split and get-batch on the device match the oracle bit for bit.
"""
import numpy as np
import pytest

from oracle import checkpoint as ock
from oracle import data as odata
from oracle import dtype as odt
from oracle import models, prng

pytestmark = pytest.mark.gpu

F32, BF16, F16, I32 = 0x21000020, 0x22000010, 0x21000010, 0x10000020
KIND = {F32: "F32", BF16: "BF16", F16: "F16", I32: "I32"}


@pytest.fixture(scope="module")
def session(cuda):
    from sheaf_b200.runtime import Session

    return Session(0)


def _dev_f16(session, a):
    # the Python upload has no f16 path: bf16-free raw copy through the C ABI
    import ctypes as C

    from sheaf_b200.runtime import Buffer, _check, lib

    a = np.ascontiguousarray(a, np.float16)
    shape = (C.c_int64 * max(1, a.ndim))(*a.shape)
    h = C.c_void_p()
    _check(lib().sb_buffer_alloc_copy(session.handle, shape, a.ndim, F16, a.ctypes.data_as(C.c_void_p), a.nbytes,
                                      C.byref(h)))
    return Buffer(h)


def test_save_matches_the_reference_layout_byte_for_byte(session, tmp_path):
    rng = np.random.default_rng(1)
    w = odt.round_bf16(rng.standard_normal((65, 16)).astype(np.float32))
    m = rng.standard_normal((16,)).astype(np.float32)
    ids = rng.integers(0, 65, (3, 7)).astype(np.int32)
    h = rng.standard_normal((5, 4)).astype(np.float16)
    tree = {"params": {"lm_head": {"weight": session.upload(w, BF16)}, "ln": [session.upload(m, F32)]},
            "t": session.upload(np.float32(4.0).reshape(()), F32), "ids": session.upload(ids, I32),
            "half": _dev_f16(session, h),
            # escaped the way serde_json escapes: short forms, \u00xx, UTF-8 kept
            'odd"key\\\n\t\x01\x1f\u00e9': session.upload(m, F32)}
    p = tmp_path / "ckpt.safetensors"
    session.save_safetensors(p, tree)
    want = ock.save_bytes([ock.entry_of("params.lm_head.weight", w, "BF16"), ock.entry_of("params.ln.0", m, "F32"),
                           ock.entry_of("t", np.float32(4.0), "F32"), ock.entry_of("ids", ids, "I32"),
                           ock.entry_of("half", h, "F16"), ock.entry_of('odd"key\\\n\t\x01\x1f\u00e9', m, "F32")])
    assert p.read_bytes() == want
    assert b'"odd\\"key\\\\\\n\\t\\u0001\\u001f\xc3\xa9"' in want


def test_load_decodes_every_dtype_like_the_reference(session, tmp_path):
    st_np = pytest.importorskip("safetensors.numpy")
    rng = np.random.default_rng(2)
    arrs = {"f32": rng.standard_normal((3, 4)).astype(np.float32), "f64": rng.standard_normal(5),
            "f16": rng.standard_normal((2, 2)).astype(np.float16), "i32": np.array([1, -7], np.int32),
            "i64": np.array([3, -4, 2**30], np.int64), "u8": np.array([0, 9, 255], np.uint8),
            "b": np.array([True, False]), "s": np.array(2.5, np.float32)}
    p = tmp_path / "in.safetensors"
    st_np.save_file(arrs, str(p))
    want = ock.load_bytes(p.read_bytes())
    got = session.load_safetensors(p, nested=False)
    assert sorted(got) == sorted(arrs)
    for k, (kind, v) in want.items():
        assert KIND[got[k].elem] == kind, k
        assert np.array_equal(got[k].to_host(), v), k


def test_round_trip_is_bitwise_and_nested(session, tmp_path):
    rng = np.random.default_rng(3)
    big = rng.standard_normal(20 << 20).astype(np.float32)  # 80 MB: several staging chunks
    tree = {"params": {"h": [{"w": session.upload(big, F32)},
                             {"w": session.upload(odt.round_bf16(big[:1000]), BF16)}]},
            "t": session.upload(np.float32(7.0).reshape(()), F32)}
    p = tmp_path / "rt.safetensors"
    session.save_safetensors(p, tree)
    back = session.load_safetensors(p)
    assert set(back) == {"params", "t"} and isinstance(back["params"]["h"], list)
    assert np.array_equal(back["params"]["h"][0]["w"].to_host(), big)
    assert back["params"]["h"][1]["w"].elem == BF16
    assert np.array_equal(back["params"]["h"][1]["w"].to_host(), odt.round_bf16(big[:1000]))
    assert float(back["t"].to_host()) == 7.0


def test_train_state_resume_continues_identically(cuda, tmp_path):
    """Checkpoint {params, m, v, t} after two train steps (train.shf:84-87),
    reload it in a fresh session (train.shf:46-49) and take a third step: the
    result equals the third step of the uninterrupted run, bit for bit."""
    from sheaf_b200.runtime import Session

    cfg = models.GPTConfig(n_layer=1, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=2, seq=64)
    names = models.gpt_leaf_names(cfg)
    p0, x, y = models.gpt_inputs(cfg)
    p0 = [odt.round_bf16(a) for a in p0]
    lr = np.float32(6e-4).reshape(())

    def module(s):
        s.create_gpt_train("gpt", n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd,
                           block_size=cfg.block_size, vocab_size=cfg.vocab_size, batch=cfg.batch, seq=cfg.seq,
                           elem=BF16)

    def step(s, state):
        n = len(names)
        ins = ([state["loss"]] + state["m"] + state["params"] + [state["t"]] + state["v"] +
               [s.upload(x, F32), s.upload(y, F32), s.upload(lr, F32)])
        o = s.call("gpt.train_step", ins)
        return {"loss": o[0], "m": o[1:1 + n], "params": o[1 + n:1 + 2 * n], "t": o[1 + 2 * n],
                "v": o[2 + 2 * n:]}

    s1 = Session(0)
    module(s1)
    zeros = [np.zeros_like(a) for a in p0]
    state = {"loss": s1.upload(np.float32(0).reshape(()), BF16), "m": [s1.upload(a, BF16) for a in zeros],
             "params": [s1.upload(a, BF16) for a in p0], "t": s1.upload(np.float32(0).reshape(()), F32),
             "v": [s1.upload(a, BF16) for a in zeros]}
    for _ in range(2):
        state = step(s1, state)
    ckpt = tmp_path / "ckpt.safetensors"
    s1.save_safetensors(ckpt, {"params": dict(zip(names, state["params"])), "m": dict(zip(names, state["m"])),
                               "v": dict(zip(names, state["v"])), "t": state["t"]})
    cont = step(s1, state)

    s2 = Session(0)
    module(s2)
    back = s2.load_safetensors(ckpt, nested=False)  # leaf names hold dots themselves
    resumed = {"loss": s2.upload(np.float32(0).reshape(()), BF16),
               "m": [back["m." + k] for k in names], "params": [back["params." + k] for k in names],
               "t": back["t"], "v": [back["v." + k] for k in names]}
    again = step(s2, resumed)
    assert float(again["t"].to_host()) == float(cont["t"].to_host()) == 3.0
    for part in ("params", "m", "v"):
        for a, b in zip(cont[part], again[part]):
            assert np.array_equal(a.to_host(), b.to_host()), part
    assert float(again["loss"].to_host()) == float(cont["loss"].to_host())


def test_random_split_and_get_batch_match_the_oracle(session):
    rng = np.random.default_rng(4)
    data = rng.integers(0, 65, 20000).astype(np.float32)
    d = session.upload(data, F32)
    for seed in [0, 7, 1 << 20, 4294967295]:
        key = prng.random_key(seed)
        kids = session.random_split(session.upload(key, F32), 3).to_host()
        want = prng.random_split(key, 3)
        for i in range(3):
            assert np.array_equal(kids[i], want[i])
        k1 = want[0]
        x, y = session.get_batch(d, session.upload(k1, F32), 256, 64)
        ex, ey, _ = odata.get_batch(data, k1, 256, 64)
        assert np.array_equal(x.to_host(), ex) and np.array_equal(y.to_host(), ey)
    from sheaf_b200.runtime import SheafB200Error

    with pytest.raises(SheafB200Error):  # no room for a window
        session.get_batch(session.upload(data[:100], F32), session.upload(prng.random_key(0), F32), 256, 4)
