"""StableHLO modules for the reference's value-and-grad goldens, printed in
the emitter's text forms (shared by the CPU evaluator tests and the GPU
front-door tests). Each case restates the Sheaf expression of the same name
in sheaf/tests/vag_tests.yaml; golden_module returns the module text and the
value of its single argument.
"""
import numpy as np

from oracle import hlo_emit
from oracle.hlo_emit import Emitter, arg

GOLDEN_CASES = ["vag-matmul", "vag-gelu", "vag-softmax", "vag-cross-entropy-loss", "vag-get-embedding-repeated"]


def golden_module(name):
    """Sheaf expression of vag_tests.yaml -> (module text, wrt argument)."""
    e = Emitter()
    if name == "vag-matmul":
        w = arg(0, (2, 2), "f32")
        x = e.const_array([[1.0, 2.0]])
        y = e.matmul(x, w)
        loss = e.sum_all(y)
        g = e.matmul(e.transpose(x, [1, 0]), e.splat(1.0, (1, 2), "f32"))
        return e.module("__vag_g", "value_and_grad", [w], [loss, g]), np.eye(2, dtype=np.float32)
    if name == "vag-gelu":
        x = arg(0, (2,), "f32")
        loss = e.sum_all(hlo_emit.gelu(e, x))
        g = hlo_emit.gelu_vjp(e, x, e.splat(1.0, (2,), "f32"))
        return e.module("__vag_g", "value_and_grad", [x], [loss, g]), np.array([0.0, 1.0], np.float32)
    if name == "vag-softmax":
        x = arg(0, (3,), "f32")
        sm = hlo_emit.softmax(e, x)
        sel = e.const_array([1.0, 0.0, 0.0])
        loss = e.sum_all(e.mul(sm, sel))
        g = e.mul(sm, e.sub(sel, e.sum(e.mul(sel, sm), -1, keepdims=True)))
        return e.module("__vag_g", "value_and_grad", [x], [loss, g]), np.array([1.0, 2.0, 3.0], np.float32)
    if name == "vag-cross-entropy-loss":
        w = arg(0, (3, 3), "f32")
        x = e.const_array([[1.0, 2.0, 3.0]])
        logits = e.matmul(x, w)
        tgt = e.const_array([[2.0]])
        loss, dlogits = hlo_emit.cross_entropy(e, e.reshape(logits, (1, 1, 3)), tgt)
        g = e.matmul(e.transpose(x, [1, 0]), e.reshape(dlogits, (1, 3)))
        return e.module("__vag_g", "value_and_grad", [w], [loss, g]), np.eye(3, dtype=np.float32)
    if name == "vag-get-embedding-repeated":
        emb = arg(0, (3, 2), "f32")
        ids = e.const_array([0.0, 0.0, 1.0])
        loss = e.sum_all(e.gather_rows(emb, ids))
        oh = e.one_hot(ids, 3)
        g = e.matmul(e.transpose(oh, [1, 0]), e.splat(1.0, (3, 2), "f32"))
        return e.module("__vag_g", "value_and_grad", [emb], [loss, g]), \
            np.array([[1, 2], [3, 4], [5, 6]], np.float32)
    raise KeyError(name)
