"""The StableHLO front door on the GPU (sb_module_load_stablehlo + sb_call).

* the module printed in the reference's docs (docs/key-concepts.md:170-184);
* modules built from the reference's own value-and-grad goldens
  (sheaf/tests/vag_tests.yaml) in the emitter's text forms: the executor must
  reproduce the expected loss and gradient;
* the MLP value_and_grad (the MLP workload) against the oracle;
* the nanoGPT value_and_grad: recognised, run through the fused plan after a
  first-call check against the generic executor, and compared to the oracle.
"""
import json
import re
from pathlib import Path

import numpy as np
import pytest

from oracle import dtype as odt
from oracle import hlo_emit, hlo_eval, models
from tests.hlo_cases import GOLDEN_CASES, golden_module
from tests.parity import TOL_BF16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_goldens.json").read_text())
NUM = re.compile(r"-?\d+(?:\.\d*)?(?:e-?\d+)?")
F32, BF16 = 0x21000020, 0x22000010


@pytest.fixture(scope="module")
def session(cuda):
    from sheaf_b200.runtime import Session

    return Session(0)


def run(session, text, inputs, elems):
    name = session.load_stablehlo(text)
    fn = re.search(r"func\.func @([\w]+)", text).group(1)
    bufs = [session.upload(a, e) for a, e in zip(inputs, elems)]
    outs = session.call(f"{name}.{fn}", bufs)
    return name, [o.to_host() for o in outs]


def test_docs_forward_module(session):
    rng = np.random.default_rng(0)
    W = rng.standard_normal((768, 768)).astype(np.float32) * 0.05
    b = rng.standard_normal(768).astype(np.float32)
    x = rng.standard_normal((4, 768)).astype(np.float32)
    _, (out,) = run(session, GOLD["docs_mlir_forward"], [W, b, x], [F32] * 3)
    assert_close(out, x.astype(np.float64) @ W + b, TOL_F32, "forward")


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_vag_goldens_through_the_front_door(session, name):
    text, x = golden_module(name)
    _, (loss, grad) = run(session, text, [x], [F32])
    got = np.concatenate([[float(loss)], grad.reshape(-1)])
    exp = np.array([float(v) for v in NUM.findall(GOLD["vag"][name]["expected"])])
    np.testing.assert_allclose(got, exp, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_mlp_vag_front_door(session, dt):
    leaves, x, y = models.mlp_inputs()
    text = hlo_emit.mlp_vag_module(dt=dt)
    elem = F32 if dt == "f32" else BF16
    ins = [np.asarray(v, np.float32) for v in leaves + [x, y]]
    if dt == "bf16":
        ins = [odt.round_bf16(v) for v in ins]
        leaves = ins[:4]
    name, outs = run(session, text, ins, [elem] * 6)
    assert "generic executor" in session.describe(name)
    # the module's own arithmetic: every op rounded to its element type, as
    # the reference compiles it (oracle/hlo_eval.py)
    ref = hlo_eval.evaluate(text, ins)
    tol = TOL_F32 if dt == "f32" else TOL_BF16
    assert abs(float(outs[0]) - float(ref[0])) <= tol * abs(float(ref[0]))
    for nm, g, r in zip(["dW1", "db1", "dW2", "db2"], outs[1:], ref[1:]):
        assert_close(g, r, tol, nm)
    if dt == "f32":  # and in f32 the composed VJPs of the model oracle
        ref_loss, ref_grads = models.mlp_value_and_grad(ins[:4], ins[4], ins[5], dtype=np.float64)
        assert abs(float(outs[0]) - ref_loss) <= tol * abs(ref_loss)
        for nm, g, r in zip(["dW1", "db1", "dW2", "db2"], outs[1:], ref_grads):
            assert_close(g, r, tol, nm)


@pytest.mark.parametrize("dt", ["bf16", "f32"])
def test_nanogpt_vag_front_door_uses_verified_fused_plan(session, dt):
    cfg = models.GPTConfig(n_layer=2, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=4, seq=64)
    leaves, x, y = models.gpt_inputs(cfg)
    if dt == "bf16":
        leaves = [odt.round_bf16(l) for l in leaves]
    elem = BF16 if dt == "bf16" else F32
    text = hlo_emit.gpt_vag_module(cfg, dt)
    name = session.load_stablehlo(text)
    assert "pending first-call verification" in session.describe(name)
    bufs = [session.upload(l, elem) for l in leaves] + [session.upload(x, F32), session.upload(y, F32)]
    first = [o.to_host() for o in session.call(f"{name}.value_and_grad", bufs)]
    assert "verified" in session.describe(name), session.describe(name)
    second = [o.to_host() for o in session.call(f"{name}.value_and_grad", bufs)]
    ref_loss, ref_grads = models.gpt_value_and_grad(leaves, x, y, cfg, dtype=np.float64)
    tol = TOL_F32 if dt == "f32" else TOL_BF16
    per_op = hlo_eval.evaluate(text, leaves + [x, y])  # the module's ops, each rounded to its type
    for outs in (first, second):
        assert abs(float(outs[0]) - ref_loss) <= tol * abs(ref_loss)
        assert abs(float(outs[0]) - float(per_op[0])) <= tol * abs(float(per_op[0]))
        for nm, g, r, p in zip(models.gpt_leaf_names(cfg), outs[1:], ref_grads, per_op[1:]):
            assert_close(g, r, tol, nm)
            assert_close(g, p, tol, nm + " (per-op rounding)")


def test_first_call_check_rejects_a_deviation_above_its_tolerance(cuda, monkeypatch):
    """The first-call check holds the fused plan to the parity bar against
    the generic executor and reports the deviation it measured; with the
    tolerance set below that deviation the same text is rejected and the
    generic executor's results (the module's per-op arithmetic) come back."""
    from sheaf_b200.runtime import Session

    cfg = models.GPTConfig(n_layer=1, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=2, seq=64)
    leaves, x, y = models.gpt_inputs(cfg)
    leaves = [odt.round_bf16(l) for l in leaves]
    text = hlo_emit.gpt_vag_module(cfg, "bf16")

    def load_and_call():
        s = Session(0)
        name = s.load_stablehlo(text)
        bufs = [s.upload(l, BF16) for l in leaves] + [s.upload(x, F32), s.upload(y, F32)]
        outs = [o.to_host() for o in s.call(f"{name}.value_and_grad", bufs)]
        return s.describe(name), outs

    note, _ = load_and_call()
    assert "verified against the generic executor" in note, note
    dev = float(re.search(r"max deviation ([0-9.e+-]+)", note).group(1))
    assert 0 < dev <= TOL_BF16
    monkeypatch.setenv("SHEAF_B200_VERIFY_RTOL", repr(dev / 2))
    note, outs = load_and_call()
    assert "generic executor (fused plan disagreed" in note, note
    per_op = hlo_eval.evaluate(text, leaves + [x, y])
    for g, p in zip(outs, per_op):
        assert_close(np.asarray(g, np.float64).reshape(np.shape(p)), p, TOL_BF16)


@pytest.mark.parametrize("dt,key", [("bf16", False), ("bf16", True), ("f32", False)])
def test_nanogpt_train_step_text_uses_the_fused_train_plan(session, dt, key):
    """The train-step module (value_and_grad + clip-by-global-norm + AdamW in
    one text, examples/nanogpt/train.shf:26-33) is recognised, checked against
    the generic executor on the first call and then run on the fused train
    plan; two steps in a row (the second on the first's state) against the
    model and optimizer oracles; a key leaf passes through unchanged."""
    from oracle import optim

    cfg = models.GPTConfig(n_layer=2, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=4, seq=64)
    leaves, x, y = models.gpt_inputs(cfg)
    # the state training starts from: m and v are tree-map-zeros params, t = 0
    # (train.shf:54-59); the second step runs on the first one's state
    m = [np.zeros_like(l) for l in leaves]
    v = [np.zeros_like(l) for l in leaves]
    bf = dt == "bf16"
    rnd = odt.round_bf16 if bf else (lambda a: np.asarray(a, np.float32))
    leaves, m, v = [rnd(a) for a in leaves], [rnd(a) for a in m], [rnd(a) for a in v]
    elem = BF16 if bf else F32
    n = len(leaves)
    text = hlo_emit.gpt_train_module(cfg, dt, with_key=key)
    name = session.load_stablehlo(text)
    assert "fused nanoGPT train-step plan pending first-call verification" in session.describe(name)
    keyv = np.array([7.0, 1.0, 0.0, 3.0], np.float32)
    t, lr = 0.0, 6e-4
    state = [np.float32(0.0)] + m + leaves + [np.float32(t)] + v
    elems = [elem] + [elem] * n + [elem] * n + [F32] + [elem] * n
    tol = TOL_F32 if not bf else TOL_BF16
    for step in range(2):
        ins = ([keyv] if key else []) + state + [x, y, np.float32(lr)]
        ies = ([F32] if key else []) + elems + [F32, F32, F32]
        bufs = [session.upload(a, e) for a, e in zip(ins, ies)]
        outs = [o.to_host() for o in session.call(f"{name}.train_step", bufs)]
        if step == 0:
            assert "fused nanoGPT train-step plan (verified" in session.describe(name), session.describe(name)
        if key:
            assert np.array_equal(outs[0], keyv)
            outs = outs[1:]
        mm, pp, tt, vv = state[1:1 + n], state[1 + n:1 + 2 * n], float(state[1 + 2 * n]), state[2 + 2 * n:]
        loss, grads = models.gpt_value_and_grad(pp, x, y, cfg, dtype=np.float64)
        if bf:
            grads = [odt.round_bf16(g) for g in grads]
        p2, m2, v2, t2 = optim.adamw_step(pp, grads, mm, vv, tt, lr, bf16=bf)
        assert abs(float(outs[0]) - loss) <= tol * abs(loss)
        assert float(outs[1 + 2 * n]) == t2
        flips = total = 0
        for i in range(n):
            assert_close(outs[1 + i], m2[i], tol, f"m {i}")
            assert_close(outs[2 + 2 * n + i], v2[i], 2 * tol, f"v {i}")
            # an AdamW step moves p by about lr * sign(g): within 3 lr
            # everywhere, and beyond 1% of lr only where g is within its
            # rounding of zero
            d = np.abs(np.asarray(outs[1 + n + i], np.float64) - p2[i])
            slack = np.abs(p2[i]) * (2.0 ** -7 if bf else 1e-6)
            assert (d <= 3 * lr + slack).all(), f"p {i}"
            flips += int((d > 1e-2 * lr + slack).sum())
            total += d.size
        assert flips <= 0.02 * total, (flips, total)
        state = [np.asarray(o, np.float32) for o in outs]


def test_full_nanogpt_text_module_verifies_at_full_size(session):
    """The 1948-op nanoGPT-char value_and_grad text (B=64, T=256): the first
    call runs the generic executor and the fused plan on the same inputs and
    keeps the fused plan; the loss agrees with the oracle's forward."""
    from oracle import ops

    cfg = models.NANOGPT_CHAR
    leaves, x, y = models.gpt_inputs(cfg)
    leaves = [odt.round_bf16(l) for l in leaves]
    name = session.load_stablehlo(hlo_emit.gpt_vag_module(cfg, "bf16"))
    bufs = [session.upload(l, BF16) for l in leaves] + [session.upload(x, F32), session.upload(y, F32)]
    out = session.call(f"{name}.value_and_grad", bufs)
    assert "verified" in session.describe(name), session.describe(name)
    loss = float(out[0].to_host())
    ref = float(ops.cross_entropy(models.gpt_forward_logits(leaves, x, cfg, dtype=np.float32), y))
    assert abs(loss - ref) <= TOL_BF16 * abs(ref)
    out2 = session.call(f"{name}.value_and_grad", bufs)
    assert abs(float(out2[0].to_host()) - loss) <= 1e-6 * abs(loss)


def test_unimplemented_op_fails_like_a_compile_error(session):
    from sheaf_b200.runtime import SheafB200Error

    text = ("module @m {\n func.func @f(%arg0: tensor<4xf32>) -> tensor<4xf32> {\n"
            "    %0 = stablehlo.cbrt %arg0 : tensor<4xf32>\n    return %0 : tensor<4xf32>\n }\n}\n")
    with pytest.raises(SheafB200Error) as e:
        session.load_stablehlo(text)
    assert e.value.code == 12


def test_reverse_and_dynamic_slices(session):
    """stablehlo.reverse, dynamic_slice and both dynamic_update_slice forms,
    with start indices inside and outside the operand (clamped to
    [0, dim - size] as StableHLO specifies)."""
    from tests.test_stablehlo_parse import INDEXING

    I32 = 0x10000020
    x = np.arange(24, dtype=np.float32).reshape(4, 6)
    u = np.array([[100.0, 200.0]], np.float32)

    def clamp(v, hi):
        return min(max(v, 0), hi)

    for i, j in [(1, 2), (7, -3), (-1, 5), (2, 4)]:
        _, (rev, ds, dus, dus2) = run(session, INDEXING, [x, np.int32(i).reshape(()), np.int32(j).reshape(()), u],
                                      [F32, I32, I32, F32])
        assert np.array_equal(rev, x[:, ::-1])
        a, b = clamp(i, 2), clamp(j, 3)
        assert np.array_equal(ds, x[a:a + 2, b:b + 3])
        e = x.copy()
        a, b = clamp(i, 3), clamp(j, 4)
        e[a:a + 1, b:b + 2] = u
        assert np.array_equal(dus, e)
        e = x.copy()
        a, b = clamp(j, 3), clamp(i, 4)
        e[a:a + 1, b:b + 2] = u
        assert np.array_equal(dus2, e)


@pytest.mark.parametrize("direction,key,n", [("GT", "f32", 1000), ("LT", "f32", 1000), ("GT", "bf16", 1000),
                                             # rows beyond one CTA's shared memory (chunked merge sort):
                                             # GPT-2's 50304-entry top_k, just past the limit, a partial chunk
                                             ("GT", "f32", 50304), ("LT", "bf16", 50304), ("GT", "bf16", 16385),
                                             ("GT", "f32", 70001)])
def test_top_k_sort(session, direction, key, n):
    """top_k through the emitter's sort: stable (ties keep index order, -0.0
    ties with 0.0), the first k of every row, indices converted to f32;
    compared bit-exactly with numpy's stable argsort."""
    from tests.test_stablehlo_parse import top_k_module

    rows, k = 5, 37 if n < 10000 else 200
    rng = np.random.default_rng(3)
    x = rng.integers(-20, 20, (rows, n)).astype(np.float32) * 0.25  # many ties
    x[0, :7] = 3.5
    x[1, 5:9] = [0.0, -0.0, 0.0, -0.0]
    x[1, 10:12] = 100.0
    if key == "bf16":
        x = odt.round_bf16(x)
    _, (vals, idx) = run(session, top_k_module(rows, n, k, direction, key), [x], [BF16 if key == "bf16" else F32])
    order = np.argsort(-x if direction == "GT" else x, axis=1, kind="stable")[:, :k]
    assert np.array_equal(idx, order.astype(np.float32))
    assert np.array_equal(np.asarray(vals, np.float32), np.take_along_axis(x, order, 1))


def test_plan_cache_records_and_reuses_the_verified_plan(cuda, tmp_path, monkeypatch):
    """With SHEAF_B200_CACHE_DIR set, the first-call check's outcome lands in
    manifest.json; a new session loading the same text starts on the verified
    fused plan (no check), a recorded rejection keeps the module generic, and
    an unreadable manifest is ignored."""
    from sheaf_b200.runtime import Session

    monkeypatch.setenv("SHEAF_B200_CACHE_DIR", str(tmp_path))
    cfg = models.GPTConfig(n_layer=1, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=2, seq=64)
    leaves, x, y = models.gpt_inputs(cfg)
    leaves = [odt.round_bf16(l) for l in leaves]
    text = hlo_emit.gpt_vag_module(cfg, "bf16")

    def load_and_call(expect):
        s = Session(0)
        name = s.load_stablehlo(text)
        assert expect in s.describe(name), s.describe(name)
        bufs = [s.upload(l, BF16) for l in leaves] + [s.upload(x, F32), s.upload(y, F32)]
        loss = float(s.call(f"{name}.value_and_grad", bufs)[0].to_host())
        return s, name, loss

    s1, name, loss1 = load_and_call("pending first-call verification")
    assert "verified against the generic executor" in s1.describe(name)
    manifest = json.loads((tmp_path / "manifest.json").read_text())
    entry = manifest["entries"][f"{name}.value_and_grad"]
    assert entry["plan"] == "fused-verified" and len(entry["hash"]) == 16
    s2, _, loss2 = load_and_call("plan cache")
    assert loss2 == loss1
    # a recorded rejection: the fused plan is not built
    manifest["entries"][f"{name}.value_and_grad"]["plan"] = "fused-rejected"
    (tmp_path / "manifest.json").write_text(json.dumps(manifest))
    load_and_call("generic executor (plan cache")
    # an unreadable manifest is ignored
    (tmp_path / "manifest.json").write_text("{not json")
    load_and_call("pending first-call verification")
