"""Pins oracle/hlo_eval.py, the op-by-op StableHLO evaluator that the
front-door tests compare against.

* the modules of the reference's value-and-grad goldens
  (sheaf/tests/vag_tests.yaml, printed in the emitter's forms) evaluate to
  the reference's expected loss and gradient;
* evaluated in f32, the MLP and nanoGPT value_and_grad modules agree with the
  oracle's composed VJPs (oracle/models.py) to f32 rounding;
* evaluated in bf16, each op is rounded to bf16 (a bf16 module differs from
  its fp64 evaluation by a few bf16 ulps, and exactly matches a hand
  rounding on a small case);
* the text forms the executor accepts beyond those: gather clamping, pad,
  slice, iota, compare / select, convert truncation.
"""
import json
import re
from pathlib import Path

import numpy as np
import pytest

from oracle import dtype as odt
from oracle import hlo_emit, hlo_eval, models
from tests.hlo_cases import GOLDEN_CASES, golden_module

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_goldens.json").read_text())
NUM = re.compile(r"-?\d+(?:\.\d*)?(?:e-?\d+)?")


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_golden_modules_evaluate_to_the_reference_values(name):
    text, x = golden_module(name)
    loss, grad = hlo_eval.evaluate(text, [x])
    got = np.concatenate([[float(loss)], np.asarray(grad).reshape(-1)])
    exp = np.array([float(v) for v in NUM.findall(GOLD["vag"][name]["expected"])])
    np.testing.assert_allclose(got, exp, rtol=1e-5, atol=1e-6)


def test_docs_forward_module():
    rng = np.random.default_rng(0)
    W = rng.standard_normal((768, 768)).astype(np.float32) * 0.05
    b = rng.standard_normal(768).astype(np.float32)
    x = rng.standard_normal((4, 768)).astype(np.float32)
    (out,) = hlo_eval.evaluate(GOLD["docs_mlir_forward"], [W, b, x])
    np.testing.assert_allclose(out, x.astype(np.float64) @ W + b, rtol=1e-5, atol=1e-5)


def _max_rel(a, b):
    return max(np.abs(np.asarray(x, np.float64) - y).max() / max(np.abs(y).max(), 1e-30) for x, y in zip(a, b))


def test_mlp_module_f32_matches_the_model_oracle():
    leaves, x, y = models.mlp_inputs()
    ins = [np.asarray(v, np.float32) for v in leaves + [x, y]]
    out = hlo_eval.evaluate(hlo_emit.mlp_vag_module(dt="f32"), ins)
    loss, grads = models.mlp_value_and_grad(ins[:4], ins[4], ins[5], dtype=np.float64)
    assert abs(float(out[0]) - loss) <= 1e-6 * abs(loss)
    assert _max_rel(out[1:], grads) <= 1e-6


def test_gpt_module_f32_matches_the_model_oracle():
    cfg = models.GPTConfig(n_layer=2, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=4, seq=64)
    leaves, x, y = models.gpt_inputs(cfg)
    out = hlo_eval.evaluate(hlo_emit.gpt_vag_module(cfg, "f32"), leaves + [x, y])
    loss, grads = models.gpt_value_and_grad(leaves, x, y, cfg, dtype=np.float64)
    assert abs(float(out[0]) - loss) <= 1e-6 * abs(loss)
    assert _max_rel(out[1:], grads) <= 1e-5


def test_bf16_module_rounds_every_op():
    e = hlo_emit.Emitter()
    a = hlo_emit.arg(0, (3,), "bf16")
    b = hlo_emit.arg(1, (3,), "bf16")
    s = e.add(e.mul(a, b), a)
    text = e.module("m", "f", [a, b], [s])
    av = odt.round_bf16(np.array([1.0 + 2 ** -7, 3.0, -1.5], np.float32))
    bv = odt.round_bf16(np.array([1.0 + 2 ** -7, 1.0 / 3.0, 2.0], np.float32))
    (out,) = hlo_eval.evaluate(text, [av, bv])
    exp = odt.round_bf16(odt.round_bf16(av * bv) + av)  # rounded after the multiply and after the add
    np.testing.assert_array_equal(out.astype(np.float32), exp)


def test_indexing_forms():
    from tests.test_stablehlo_parse import INDEXING  # reverse / dynamic slices are not needed here

    del INDEXING
    e = hlo_emit.Emitter()
    t = hlo_emit.arg(0, (5, 2), "f32")
    ids = hlo_emit.arg(1, (4,), "f32")
    g = e.gather_rows(t, ids)
    oh = e.one_hot(ids, 5)
    p = e.pad(e.slice(t, (1, 0), (3, 2)), (1, 0), (2, 1))
    text = e.module("m", "f", [t, ids], [g, oh, p])
    tv = np.arange(10, dtype=np.float32).reshape(5, 2)
    iv = np.array([2.5, -3.0, 7.0, 4.0], np.float32)
    gg, ohv, pv = hlo_eval.evaluate(text, [tv, iv])
    np.testing.assert_array_equal(gg, tv[[2, 0, 4, 4]])  # truncation, then clamping of the start index
    np.testing.assert_array_equal(ohv.sum(1), [0, 0, 0, 1])  # f32 compare: only 4.0 has a class
    exp = np.zeros((5, 3))
    exp[1:3, 0:2] = tv[1:3]
    np.testing.assert_array_equal(pv, exp)


@pytest.mark.parametrize("with_key", [False, True])
def test_train_step_module_f32_matches_the_model_and_optimizer_oracles(with_key):
    """The train-step text (value_and_grad + clip-by-global-norm + AdamW,
    examples/nanogpt/train.shf:26-33 with lib/optim.shf inlined), evaluated
    in f32, against oracle.models + oracle.optim."""
    from oracle import optim

    cfg = models.GPTConfig(n_layer=1, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=2, seq=64)
    leaves, x, y = models.gpt_inputs(cfg)
    rng = np.random.default_rng(3)
    m = [rng.standard_normal(l.shape).astype(np.float32) * 1e-3 for l in leaves]
    v = [np.abs(rng.standard_normal(l.shape)).astype(np.float32) * 1e-6 for l in leaves]
    t, lr = 3.0, 6e-4
    key = [np.arange(4, dtype=np.float32)] if with_key else []
    ins = key + [np.float32(0.0)] + m + leaves + [np.float32(t)] + v + [x, y, np.float32(lr)]
    out = hlo_eval.evaluate(hlo_emit.gpt_train_module(cfg, "f32", with_key=with_key), ins)
    n = len(leaves)
    if with_key:
        np.testing.assert_array_equal(out[0], key[0])
        out = out[1:]
    loss, grads = models.gpt_value_and_grad(leaves, x, y, cfg, dtype=np.float64)
    p2, m2, v2, t2 = optim.adamw_step(leaves, grads, m, v, t, lr)
    assert abs(float(out[0]) - loss) <= 1e-6 * abs(loss)
    assert float(out[1 + 2 * n]) == t2
    assert _max_rel(out[1:1 + n], m2) <= 2e-5
    assert _max_rel(out[1 + n:1 + 2 * n], p2) <= 1e-5
    assert _max_rel(out[2 + 2 * n:], v2) <= 2e-5
