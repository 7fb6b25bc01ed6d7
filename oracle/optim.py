"""Optimizer step of nanoGPT's train-step (numpy restatement, test-only).

examples/nanogpt/train.shf:26-33 compiles, as one module,
    [loss g] = value-and-grad(loss-fn)(params)
    g        = clip-by-global-norm(g, 1.0)
    [p m v t] = adamw-step(params, g, m, v, t, lr, 0.9, 0.95, 1e-8, 0.1)
with the stdlib definitions in sheaf/lib/optim.shf:
  * global-norm (:42-45): sqrt of the sum over leaves of sum(g**2), each
    leaf's sum taken in the leaf's dtype and cast to f32;
  * clip-by-global-norm (:48-51): factor = min(1, max_norm / (norm + 1e-8)),
    cast like each leaf, g * factor;
  * adamw-step (:19-32): t' = t + 1; m' = b1 m + (1 - b1) g;
    v' = b2 v + (1 - b2) g*g; bc_m = 1 / (1 - b1**t'); bc_v = 1 / (1 - b2**t');
    p' = p - lr (wd p + (m' bc_m) / (sqrt(v' bc_v) + eps)).
m and v are `tree-map-zeros params` (train.shf:58-59): same dtype as params.
Arrays keep the dtype they are given; `bf16=True` rounds every leaf result
to bf16 (the element type of the leaves), as the module's outputs are.
"""
from __future__ import annotations

import numpy as np

from . import dtype as odt

CLIP_EPS = 1e-8  # lib/optim.shf:50


def global_norm(grads) -> float:
    """lib/optim.shf:42-45 (sums accumulated in float64 here)."""
    return float(np.sqrt(sum(float(np.sum(np.asarray(g, np.float64) ** 2)) for g in grads)))


def clip_factor(grads, max_norm: float) -> float:
    """lib/optim.shf:48-51."""
    return min(1.0, max_norm / (global_norm(grads) + CLIP_EPS))


def adamw_step(params, grads, m, v, t: float, lr: float, b1=0.9, b2=0.95, eps=1e-8, wd=0.1, max_norm=1.0,
               bf16: bool = False):
    """clip-by-global-norm then adamw-step (train.shf:29-32, optim.shf:19-32,
    48-51). Returns (new_params, new_m, new_v, new_t)."""
    f = clip_factor(grads, max_norm) if max_norm > 0 else 1.0
    rnd = odt.round_bf16 if bf16 else (lambda x: x)
    if bf16:
        f_leaf = float(odt.round_bf16(np.float32(f)))  # __cast-like factor g
    else:
        f_leaf = f
    t_new = t + 1.0
    bcm = 1.0 / (1.0 - b1 ** t_new)
    bcv = 1.0 / (1.0 - b2 ** t_new)
    out_p, out_m, out_v = [], [], []
    for p, g, mm, vv in zip(params, grads, m, v):
        p = np.asarray(p, np.float64)
        g = np.asarray(g, np.float64) * f_leaf
        if bf16:
            g = rnd(g)
        mm = b1 * np.asarray(mm, np.float64) + (1.0 - b1) * g
        vv = b2 * np.asarray(vv, np.float64) + (1.0 - b2) * (g * g)
        pn = p - lr * (wd * p + (mm * bcm) / (np.sqrt(vv * bcv) + eps))
        out_p.append(rnd(pn))
        out_m.append(rnd(mm))
        out_v.append(rnd(vv))
    return out_p, out_m, out_v, t_new
