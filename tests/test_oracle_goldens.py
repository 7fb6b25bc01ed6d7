"""Pins the CPU oracle against the reference's own golden vectors.

Fixture: tests/golden/reference_goldens.json (made by
tests/golden/make_reference_goldens.py from sheaf/tests/vag_tests.yaml,
sheaf/tests/interpreter_tests.yaml and sheaf/src/core/prng.rs). Each VAG
case below restates the Sheaf expression of the same name with the oracle's
rules, in float32 like the reference, and must reproduce the expected value
and gradient.
"""
import json
import re
from pathlib import Path

import numpy as np
import pytest

from oracle import dtype as odt
from oracle import ops, prng

GOLD = json.loads((Path(__file__).parent / "golden" / "reference_goldens.json").read_text())
F = np.float32
NUM = re.compile(r"-?\d+(?:\.\d*)?(?:e-?\d+)?")


def parse_numbers(s: str) -> np.ndarray:
    return np.array([float(v) for v in NUM.findall(s)], dtype=np.float64)


def a(x):
    return np.array(x, dtype=F)


def _ce_slice(w):
    full = a([[1, 2, 3, 4]]) @ w
    logits = full[:, 0:3]
    loss = ops.cross_entropy(logits, a([2]))
    dfull = np.zeros_like(full)
    dfull[:, 0:3] = ops.cross_entropy_vjp(logits, a([2]))
    return loss, ops.matmul_vjp(a([[1, 2, 3, 4]]), w, dfull)[1]


def _shared_emb_head(w):
    idx = a([[0], [1]])
    left = ops.embedding(w, idx)
    A = a([[[1, 2]], [[3, 4]]])
    right = A @ w.T
    loss = left.sum() + right.sum()
    g_left = ops.embedding_vjp(w.shape, idx, np.ones_like(left), F)
    g_wt = ops.matmul_vjp(A, w.T, np.ones_like(right))[1]
    return loss, g_left + g_wt.T


def _batched_transpose(w):
    h = np.ones((2, 2, 2), F)
    y = h @ w
    yt = np.transpose(y, (0, 2, 1))
    s = y @ yt
    g = np.ones_like(s)
    dy, dyt = ops.matmul_vjp(y, yt, g)
    dy = dy + np.transpose(dyt, (0, 2, 1))
    return s.sum(), ops.matmul_vjp(h, w, dy)[1]


def _mm(w, scale=1.0):
    x = a([[1, 2]])
    return F(scale) * (x @ w).sum(), F(scale) * ops.matmul_vjp(x, w, np.ones((1, 2), F))[1]


VAG = {
    "vag-add": (a([1, 2]), lambda x: ((x + a([10, 20])).sum(), np.ones_like(x))),
    "vag-sub": (a([1, 2]), lambda x: ((x - a([10, 20])).sum(), np.ones_like(x))),
    "vag-neg": (a([1, 2]), lambda x: ((-x).sum(), -np.ones_like(x))),
    "vag-mul": (a([1, 2]), lambda x: ((x * a([3, 4])).sum(), a([3, 4]))),
    "vag-div": (a([1, 2]), lambda x: ((x / a([2, 4])).sum(), F(1) / a([2, 4]))),
    "vag-pow": (a([1, 2]), lambda x: ((x ** 3).sum(), F(3) * x ** 2)),
    "vag-exp": (a([0, 1]), lambda x: (np.exp(x).sum(), np.exp(x))),
    "vag-log": (a([1, 2]), lambda x: (np.log(x).sum(), F(1) / x)),
    "vag-sqrt": (a([4, 9]), lambda x: (np.sqrt(x).sum(), F(1) / (F(2) * np.sqrt(x)))),
    "vag-abs": (a([-3, 2]), lambda x: (np.abs(x).sum(), np.where(x >= 0, F(1), F(-1)))),
    "vag-tanh": (a([0, 1]), lambda x: (np.tanh(x).sum(), F(1) - np.tanh(x) ** 2)),
    "vag-relu": (a([-1, 2]), lambda x: (np.maximum(x, 0).sum(), np.where(x >= 0, F(1), F(0)))),
    "vag-sigmoid": (a([0]), lambda x: ((F(1) / (F(1) + np.exp(-x))).sum(),
                                       (F(1) / (F(1) + np.exp(-x))) * (F(1) - F(1) / (F(1) + np.exp(-x))))),
    "vag-gelu": (a([0, 1]), lambda x: (ops.gelu(x).sum(), ops.gelu_vjp(x, np.ones_like(x)))),
    "vag-softmax": (a([1, 2, 3]), lambda x: ((ops.softmax(x) * a([1, 0, 0])).sum(),
                                             ops.softmax_vjp(ops.softmax(x), a([1, 0, 0])))),
    "vag-log-softmax": (a([1, 2, 3]), lambda x: (ops.log_softmax(x).sum(), ops.log_softmax_vjp(x, np.ones_like(x)))),
    "vag-sum": (a([1, 2, 3]), lambda x: (x.sum(), np.ones_like(x))),
    "vag-mean": (a([1, 2, 3]), lambda x: (x.mean(), np.full_like(x, F(1) / F(3)))),
    "vag-maximum": (a([-1, 2, -3]), lambda x: (np.maximum(x, 0).sum(), np.where(x >= 0, F(1), F(0)))),
    "vag-matmul": (a([[1, 0], [0, 1]]), _mm),
    "vag-einsum": (a([[1, 0], [0, 1]]), _mm),
    "vag-let-lambda": (a([[1, 0], [0, 1]]), _mm),
    "vag-defn-calling-defn": (a([[1, 0], [0, 1]]), _mm),
    "vag-dict-capture": (a([[1, 0], [0, 1]]), lambda w: _mm(w, 0.5)),
    "vag-slice": (a([1, 2, 3, 4]), lambda x: (x[0:2].sum(), ops.slice_rows_vjp(x.shape, 0, np.ones(2, F)))),
    "vag-slice-axis": (a([[1, 2, 3], [4, 5, 6]]),
                       lambda x: (x[:, 0:2].sum(), ops.slice_rows_vjp((3, 2), 0, np.ones((2, 2), F)).T)),
    "vag-ce-slice": (np.eye(4, dtype=F), _ce_slice),
    "vag-get-embedding": (a([[1, 2], [3, 4], [5, 6]]), lambda e: (ops.embedding(e, a([0, 1])).sum(),
                                                                  ops.embedding_vjp(e.shape, a([0, 1]),
                                                                                    np.ones((2, 2), F), F))),
    "vag-get-embedding-repeated": (a([[1, 2], [3, 4], [5, 6]]),
                                   lambda e: (ops.embedding(e, a([0, 0, 1])).sum(),
                                              ops.embedding_vjp(e.shape, a([0, 0, 1]), np.ones((3, 2), F), F))),
    "vag-shared-embedding-head": (a([[1, 0], [0, 1], [1, 1]]), _shared_emb_head),
    "vag-where": (a([-2, 3]), lambda x: (np.where(x > 0, x, x * F(0.1)).sum(), np.where(x > 0, F(1), F(0.1)))),
    "vag-cross-entropy-loss": (np.eye(3, dtype=F),
                               lambda w: (ops.cross_entropy(a([[1, 2, 3]]) @ w, a([2])),
                                          ops.matmul_vjp(a([[1, 2, 3]]), w,
                                                         ops.cross_entropy_vjp(a([[1, 2, 3]]) @ w, a([2])))[1])),
    "vag-matmul-batched-transpose": (np.ones((2, 2), F), _batched_transpose),
}


def test_every_golden_case_is_restated():
    assert set(GOLD["vag"]) == set(VAG)


@pytest.mark.parametrize("name", sorted(VAG))
def test_vag_golden(name):
    x, fn = VAG[name]
    loss, grad = fn(x.copy())
    got = np.concatenate([[float(loss)], np.asarray(grad, dtype=np.float64).reshape(-1)])
    exp = parse_numbers(GOLD["vag"][name]["expected"])
    assert got.shape == exp.shape, (got, exp)
    np.testing.assert_allclose(got, exp, rtol=2e-6, atol=2e-6)


FWD = {
    "(tanh 0.0)": lambda: np.tanh(F(0)),
    "(tanh 1.0)": lambda: np.tanh(F(1)),
    "(gelu 0.0)": lambda: ops.gelu(a(0.0)),
    "(gelu 1.0)": lambda: ops.gelu(a(1.0)),
    "(softmax [1.0 1.0])": lambda: ops.softmax(a([1, 1])),
    "(softmax [1.0 2.0 3.0] :axis -1)": lambda: ops.softmax(a([1, 2, 3])),
    "(log-softmax [1.0 2.0])": lambda: ops.log_softmax(a([1, 2])),
}


def test_forward_goldens():
    assert len(GOLD["forward"]) == len(FWD)
    for case in GOLD["forward"]:
        got = np.asarray(FWD[case["test"]](), dtype=np.float64).reshape(-1)
        np.testing.assert_allclose(got, parse_numbers(case["expected"]), rtol=2e-6, atol=2e-7)


def test_layer_norm_analytic():
    """sheaf/tests/interpreter_tests.rs:146-170: loss = sum(ln(x)^2), gamma [2,1]."""
    x = a([3, 5])
    g, b = a([2, 1]), a([0, 0])
    y, cache = ops.layer_norm_nb(x, g)
    y = y + b
    loss = (y * y).sum()
    dx, _ = ops.layer_norm_nb_vjp(cache, g, F(2) * y)
    eps = 1e-5
    assert abs(float(loss) - 5.0 / (1.0 + eps)) <= 5 * np.finfo(np.float32).eps
    slope = 5.0 * eps / (1.0 + eps) ** 2
    np.testing.assert_allclose(dx.astype(np.float64), [-slope, slope], atol=5 * np.finfo(np.float32).eps)
    np.testing.assert_allclose(ops.layer_norm(x, g, b), y, rtol=1e-6)


def test_threefry_known_answers():
    for kat in GOLD["threefry_kat"]:
        x0, x1 = prng.threefry(kat["key"], np.array([kat["counter"][0]], np.uint32),
                               np.array([kat["counter"][1]], np.uint32))
        assert [int(x0[0]), int(x1[0])] == kat["expected"]


def test_key_roundtrip_and_endpoints():
    """sheaf/src/core/prng.rs:181-205."""
    for s in [0, 42, -1, -(2 ** 63), 2 ** 63 - 1, 16777217, 4294967295]:
        w = prng.seed(s)
        assert prng.decode(prng.encode(w)) == w
        for i in [0, 1, 17]:
            child = prng.split_words(w, i + 1)[i]
            assert prng.decode(prng.encode(child)) == child
    assert prng.uniform_from_bits(np.array([0], np.uint32))[0] == 0.0
    assert prng.uniform_from_bits(np.array([0xFFFFFFFF], np.uint32))[0] == F(1.0 - 1.0 / 16777216.0)
    for w in [(0, 0), (0xFFFFFFFF, 0xFFFFFFFF), (0, 0xFFFFFFFF)]:
        assert np.isfinite(prng.normal_from_bits(np.array([w[0]], np.uint32), np.array([w[1]], np.uint32))).all()
        r = prng.randint_from_bits(np.array([w[0]], np.uint32), -3, 7)
        assert -3 <= r[0] < 7


def test_bf16_round_to_nearest_even():
    """sheaf/src/core/dtype.rs:204-216."""
    vals = a([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 65504.0, 1e-40])
    bits = odt.f32_to_bf16_bits(vals)
    assert [int(b) for b in bits[:3]] == [0x3F80, 0x3F80, 0x3F82]
    assert int(odt.f32_to_bf16_bits(a([np.nan]))[0]) & 0x0040
    r = odt.round_bf16(vals)
    # half an ulp: relative for normals, absolute (2^-134) for subnormals
    assert np.all(np.abs(r - vals) <= np.maximum(np.abs(vals) * 2 ** -8, 2.0 ** -134))


def test_gpt_grad_matches_finite_differences():
    """The composed nanoGPT VJP against central differences on a tiny model
    (1 layer, 2 heads, d=16, T=8, V=16: the check-nanogpt shape of
    sheaf/tests/regressions.shf:121-154)."""
    from oracle import models

    cfg = models.GPTConfig(n_layer=1, n_head=2, n_embd=16, block_size=8, vocab_size=16, batch=2, seq=8)
    leaves, x, y = models.gpt_inputs(cfg)
    leaves = [l.astype(np.float64) for l in leaves]
    loss, grads = models.gpt_value_and_grad(leaves, x, y, cfg)
    rng = np.random.default_rng(0)
    for li in range(len(leaves)):
        for _ in range(2):
            idx = tuple(rng.integers(0, s) for s in leaves[li].shape)
            h = 1e-6
            lp = [l.copy() for l in leaves]
            lm = [l.copy() for l in leaves]
            lp[li][idx] += h
            lm[li][idx] -= h
            fd = (models.gpt_value_and_grad(lp, x, y, cfg)[0] - models.gpt_value_and_grad(lm, x, y, cfg)[0]) / (2 * h)
            assert abs(fd - grads[li][idx]) <= 1e-6 * (1 + abs(fd)), (li, idx, fd, grads[li][idx])


def test_mlp_grad_matches_finite_differences():
    from oracle import models

    leaves, x, y = models.mlp_inputs(batch=4, d_in=6, d_hidden=5, d_out=3)
    leaves = [l.astype(np.float64) + 0.1 for l in leaves]
    loss, grads = models.mlp_value_and_grad(leaves, x, y)
    for li in range(4):
        idx = (0,) * leaves[li].ndim
        h = 1e-6
        lp = [l.copy() for l in leaves]
        lm = [l.copy() for l in leaves]
        lp[li][idx] += h
        lm[li][idx] -= h
        fd = (models.mlp_value_and_grad(lp, x, y)[0] - models.mlp_value_and_grad(lm, x, y)[0]) / (2 * h)
        assert abs(fd - grads[li][idx]) <= 1e-6 * (1 + abs(fd))


EDGE = a([2.5, 3.0, -1.0, -0.0, 0.75, -2.5, 15.0, 16.0, 21.0, 1e6, 15.75, 5.0])


def test_one_hot_compares_f32_ids():
    """tensor_ops.rs:163-217: compare(id, iota) in f32, so only ids that are
    exactly an integer in [0, n) select a class (-0.0 selects class 0)."""
    oh = ops.one_hot(EDGE, 16, F)
    assert oh.sum(1).tolist() == [0, 1, 0, 1, 0, 0, 1, 0, 0, 0, 0, 1]
    assert oh[1, 3] == 1 and oh[3, 0] == 1 and oh[6, 15] == 1


def test_embedding_edge_ids_follow_gather_and_one_hot():
    """Forward: convert (truncation) + gather with clamping; VJP: exactly the
    one_hot(ids)^T @ adj matmul the reference emits (reverse.rs:1108-1121)."""
    w = np.arange(16 * 3, dtype=F).reshape(16, 3)
    assert ops.embedding(w, EDGE)[:, 0].tolist() == [6, 9, 0, 0, 0, 0, 45, 45, 45, 45, 45, 15]
    g = np.random.default_rng(0).standard_normal((len(EDGE), 3))
    np.testing.assert_array_equal(ops.embedding_vjp((16, 3), EDGE, g, np.float64),
                                  ops.one_hot(EDGE, 16, np.float64).T @ g)


def test_cross_entropy_vjp_with_edge_targets_matches_finite_differences():
    """A target without a class adds nothing to the loss and gets a zero
    gradient row; the others get (softmax - one_hot) / rows."""
    rng = np.random.default_rng(1)
    logits = rng.standard_normal((len(EDGE), 16))
    d = ops.cross_entropy_vjp(logits, EDGE)
    h = 1e-6
    for r in range(len(EDGE)):
        for c in (0, 3, 15):
            lp, lm = logits.copy(), logits.copy()
            lp[r, c] += h
            lm[r, c] -= h
            fd = (ops.cross_entropy(lp, EDGE) - ops.cross_entropy(lm, EDGE)) / (2 * h)
            assert abs(fd - d[r, c]) <= 1e-7 * (1 + abs(fd)), (r, c, fd, d[r, c])
    assert not d[[0, 2, 4, 5, 7, 8, 9, 10]].any()
