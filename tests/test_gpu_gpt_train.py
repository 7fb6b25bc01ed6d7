"""nanoGPT train-step module (examples/nanogpt/train.shf:26-33: value_and_grad,
clip-by-global-norm, adamw-step) through the C ABI against the oracle.

Each step feeds the GPU's own state to both sides, so a step's error does not
compound. The oracle's gradients are the fp64 restatement, rounded to the
leaves' element type as the module's gradient buffers are.
"""
import numpy as np
import pytest

from oracle import dtype as odt
from oracle import models, optim
from tests.parity import TOL_BF16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu

BF16 = 0x22000010
F32 = 0x21000020
CFG = models.GPTConfig(n_layer=2, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=4, seq=64)
LR = 6e-4


def _module(s, kind):
    elem = BF16 if kind == "bf16" else F32
    c = CFG
    s.create_gpt_train("gpt", n_layer=c.n_layer, n_head=c.n_head, n_embd=c.n_embd, block_size=c.block_size,
                       vocab_size=c.vocab_size, batch=c.batch, seq=c.seq, elem=elem)
    return elem


def _step(s, elem, loss, m, p, t, v, x, y):
    n = len(p)
    ins = ([s.upload(np.float32(loss).reshape(()), elem)] + [s.upload(a, elem) for a in m] +
           [s.upload(a, elem) for a in p] + [s.upload(np.float32(t).reshape(()), F32)] +
           [s.upload(a, elem) for a in v] + [s.upload(x, F32), s.upload(y, F32), s.upload(np.float32(LR).reshape(()), F32)])
    outs = [o.to_host() for o in s.call("gpt.train_step", ins)]
    assert len(outs) == 3 * n + 2
    return (float(outs[0]), outs[1:1 + n], outs[1 + n:1 + 2 * n], float(outs[1 + 2 * n]), outs[2 + 2 * n:])


@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_train_step_matches_oracle(kind, cuda):
    from sheaf_b200.runtime import Session

    s = Session(0)
    elem = _module(s, kind)
    bf = kind == "bf16"
    p, x, y = models.gpt_inputs(CFG)
    rnd = odt.round_bf16 if bf else (lambda a: a.astype(np.float32))
    p = [rnd(a) for a in p]
    m = [np.zeros_like(a) for a in p]  # tree-map-zeros params (train.shf:58-59)
    v = [np.zeros_like(a) for a in p]
    t = 0.0
    tol = TOL_BF16 if bf else TOL_F32
    for step in range(2):
        loss, m2, p2, t2, v2 = _step(s, elem, 0.0, m, p, t, v, x, y)
        ref_loss, g = models.gpt_value_and_grad(p, x, y, CFG, dtype=np.float64)
        if bf:
            g = [odt.round_bf16(a) for a in g]
        rp, rm, rv, rt = optim.adamw_step(p, g, m, v, t, LR, bf16=bf)
        assert t2 == rt == t + 1
        assert abs(loss - ref_loss) <= tol * abs(ref_loss), (step, loss, ref_loss)
        for name, got, ref in (("m", m2, rm), ("v", v2, rv)):
            for i, (a, e) in enumerate(zip(got, ref)):
                assert_close(a, e, tol if name == "m" else 2 * tol, f"step {step} {name}[{i}]")
        # p' - p = -lr (wd p + m_hat / (sqrt(v_hat) + eps)): at step 1 the
        # Adam part is lr * sign(g), so it can only differ where the gradient
        # is within its own numerical error of zero
        flips = 0
        for a, e, p0, gg in zip(p2, rp, p, g):
            d = np.abs(np.asarray(a, np.float64) - np.asarray(e, np.float64))
            slack = (odt.round_bf16(np.abs(np.asarray(e, np.float32))) * 2.0 ** -7 if bf else 1e-6 * np.abs(e))
            ok = d <= 1e-2 * LR + slack
            flips += int((~ok).sum())
            assert (d <= 3.0 * LR + slack).all()
        total = sum(a.size for a in p)
        assert flips <= 0.02 * total, (step, flips, total)
        loss, m, p, t, v = loss, m2, p2, t2, v2


def test_train_step_graph_replay_is_deterministic(cuda):
    from sheaf_b200.runtime import Session

    s = Session(0)
    elem = _module(s, "bf16")
    p, x, y = models.gpt_inputs(CFG)
    p = [odt.round_bf16(a) for a in p]
    z = [np.zeros_like(a) for a in p]
    runs = [_step(s, elem, 0.0, z, p, 0.0, z, x, y) for _ in range(3)]  # eager, capture, replay
    for r in runs[1:]:
        assert r[0] == runs[0][0] and r[3] == runs[0][3]
        for part in (1, 2, 4):
            for a, b in zip(runs[0][part], r[part]):
                assert np.array_equal(a, b)
    # value_and_grad on the same module still works
    ins = [s.upload(a, elem) for a in p] + [s.upload(x, F32), s.upload(y, F32)]
    outs = s.call("gpt.value_and_grad", ins)
    assert len(outs) == 1 + len(p)


def test_train_step_rejects_bad_inputs(cuda):
    from sheaf_b200.runtime import SheafB200Error, Session

    s = Session(0)
    elem = _module(s, "bf16")
    p, x, y = models.gpt_inputs(CFG)
    ins = [s.upload(np.float32(0).reshape(()), elem)] + [s.upload(a, elem) for a in p]
    with pytest.raises(SheafB200Error) as e:
        s.call("gpt.train_step", ins)
    assert e.value.code == 3
