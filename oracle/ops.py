"""Forward and VJP rules of the ops on Sheaf's compiled fwd+VJP path (numpy).

Each rule restates the reference's definition:
  * stdlib math, inlined into primitives before AD: sheaf/lib/nn.shf
  * VJP rules: sheaf/src/autodiff/reverse.rs
  * unbroadcast of gradients: reverse.rs:360-376 / lowering/codegen/builtins.rs:173-206
Arrays keep the dtype they are given (float32 or float64).
"""
from __future__ import annotations

import numpy as np

GELU_K = 0.7978846  # lib/nn.shf:11
GELU_C = 0.044715   # lib/nn.shf:11
LN_EPS = 1e-5       # examples/nanogpt/model.shf:14, lib/nn.shf:54
MASK_FILL = -1e10   # examples/nanogpt/model.shf:8


def unbroadcast(g: np.ndarray, shape) -> np.ndarray:
    """Sum a gradient down to `shape` (maybe_unbroadcast, reverse.rs:360-376)."""
    shape = tuple(shape)
    while g.ndim > len(shape):
        g = g.sum(axis=0)
    for ax, n in enumerate(shape):
        if n == 1 and g.shape[ax] != 1:
            g = g.sum(axis=ax, keepdims=True)
    return g


# ---- matmul (`@`) ---------------------------------------------------------

def matmul(a, b):
    return a @ b


def matmul_vjp(a, b, g):
    """reverse.rs:585-689: dA = g @ swapaxes(B), dB = swapaxes(A) @ g, then unbroadcast."""
    if b.ndim == 1:
        da = np.multiply.outer(g, b) if a.ndim > 1 else g * b
        db = (a.reshape(-1, a.shape[-1]).T @ g.reshape(-1)) if a.ndim > 1 else g * a
        return da, db
    if a.ndim == 1:
        da = (g.reshape(1, -1) @ np.swapaxes(b, -1, -2)).reshape(a.shape[0])
        db = unbroadcast(np.multiply.outer(a, g), b.shape)
        return da, db
    da = unbroadcast(g @ np.swapaxes(b, -1, -2), a.shape)
    db = unbroadcast(np.swapaxes(a, -1, -2) @ g, b.shape)
    return da, db


# ---- gelu (tanh form) -----------------------------------------------------

def gelu(x):
    """lib/nn.shf:10-11: 0.5 * (x * (1 + tanh(0.7978846 * (x + 0.044715 * (x * (x * x))))))."""
    t = x.dtype.type
    return t(0.5) * (x * (t(1.0) + np.tanh(t(GELU_K) * (x + t(GELU_C) * (x * (x * x))))))


def gelu_vjp(x, g):
    """Chain rule through the inlined tanh/multiply/add ops (reverse.rs:969-975 tanh rule)."""
    t = x.dtype.type
    x2 = x * x
    th = np.tanh(t(GELU_K) * (x + t(GELU_C) * (x * x2)))
    d = t(0.5) * (t(1.0) + th) + t(0.5) * x * (t(1.0) - th * th) * t(GELU_K) * (t(1.0) + t(3.0 * GELU_C) * x2)
    return g * d


# ---- softmax / log-softmax ------------------------------------------------

def softmax(x, axis=-1):
    """lib/nn.shf:24-26: e = exp(x - max); e / sum(e)."""
    e = np.exp(x - x.max(axis=axis, keepdims=True))
    return e / e.sum(axis=axis, keepdims=True)


def softmax_vjp(y, g, axis=-1):
    """reverse.rs:814-828: sm * (g - sum(g * sm))."""
    return y * (g - (g * y).sum(axis=axis, keepdims=True))


def log_softmax(x, axis=-1):
    """lib/nn.shf:28-30: s = x - max; s - log(sum(exp(s)))."""
    s = x - x.max(axis=axis, keepdims=True)
    return s - np.log(np.exp(s).sum(axis=axis, keepdims=True))


def log_softmax_vjp(x, g, axis=-1):
    """reverse.rs:830-845: g - exp(lsm) * sum(g)."""
    return g - np.exp(log_softmax(x, axis)) * g.sum(axis=axis, keepdims=True)


# ---- reductions -----------------------------------------------------------

def var(x, axis=-1):
    """Two-pass population variance (lowering/codegen/reduction_builtins.rs:287-358)."""
    m = x.mean(axis=axis, keepdims=True)
    d = x - m
    return (d * d).mean(axis=axis, keepdims=True)


# ---- layer norm -----------------------------------------------------------

def layer_norm_nb(x, gamma):
    """examples/nanogpt/model.shf:11-14: (x - mean) / sqrt(var + 1e-5) * gamma."""
    t = x.dtype.type
    m = x.mean(axis=-1, keepdims=True)
    v = var(x, -1)
    rstd = t(1.0) / np.sqrt(v + t(LN_EPS))
    xhat = (x - m) * rstd
    return xhat * gamma, (xhat, rstd)


def layer_norm_nb_vjp(cache, gamma, g):
    """VJP of layer_norm_nb composed from the `/`, `-`, `sqrt`, `var` and `mean`
    rules (reverse.rs:551-583, 888-914, 961-967, 847-886)."""
    xhat, rstd = cache
    dgamma = unbroadcast(g * xhat, gamma.shape)
    dxhat = g * gamma
    n = xhat.shape[-1]
    dx = rstd * (dxhat - dxhat.mean(axis=-1, keepdims=True) - xhat * (dxhat * xhat).mean(axis=-1, keepdims=True))
    return dx, dgamma


def layer_norm(x, gamma, beta, axis=-1):
    """lib/nn.shf:53-59 (with beta)."""
    t = x.dtype.type
    m = x.mean(axis=axis, keepdims=True)
    v = var(x, axis)
    return (x - m) / np.sqrt(v + t(LN_EPS)) * gamma + beta


# ---- losses ---------------------------------------------------------------

def one_hot(idx, n, dtype):
    """tensor_ops.rs:163-217: compare(broadcast(idx), iota) == in f32, then
    select 1 / 0. The ids stay f32, so a fractional id (2.5) or one outside
    [0, n) matches no class and gives an all-zero row."""
    idx = np.asarray(idx, dtype=np.float32)
    return (idx[..., None] == np.arange(n, dtype=np.float32)).astype(dtype)


def cross_entropy(logits, targets):
    """lib/nn.shf:44-50: -mean(sum(log_softmax(logits[-1,V]) * one_hot(targets[-1], V), -1))."""
    V = logits.shape[-1]
    lp = log_softmax(logits.reshape(-1, V))
    mask = one_hot(np.asarray(targets).reshape(-1), V, logits.dtype)
    return -((lp * mask).sum(axis=-1)).mean()


def cross_entropy_vjp(logits, targets, g=1.0):
    """Composition of the mean, sum, multiply and log-softmax VJP rules:
    (softmax(logits) * sum(one_hot) - one_hot) / N. A row whose one-hot is all
    zero (a fractional or out-of-range target) gets a zero gradient; every
    other row gets (softmax - one_hot) / N."""
    V = logits.shape[-1]
    flat = logits.reshape(-1, V)
    n = flat.shape[0]
    mask = one_hot(np.asarray(targets).reshape(-1), V, logits.dtype)
    t = logits.dtype.type
    d = (softmax(flat) * mask.sum(axis=-1, keepdims=True) - mask) * t(g / n)
    return d.reshape(logits.shape)


def mse(pred, true):
    """lib/nn.shf:115-117."""
    d = pred - true
    return (d * d).mean()


def mse_vjp(pred, true, g=1.0):
    t = pred.dtype.type
    return t(2.0 * g / pred.size) * (pred - true)


# ---- embedding gather -----------------------------------------------------

def ids_to_index(ids):
    """`stablehlo.convert` f32 -> i32 before the gather (indexing_ops.rs:426-427):
    truncation toward zero."""
    return np.trunc(np.asarray(ids, dtype=np.float32)).astype(np.int64)


def embedding(w, ids):
    """`get` on a tensor with an index tensor -> `stablehlo.gather` of rows
    (indexing_ops.rs:416-484). Gather clamps start indices into range."""
    return w[np.clip(ids_to_index(ids), 0, w.shape[0] - 1)]


def embedding_vjp(w_shape, ids, g, dtype):
    """reverse.rs:1077-1122: one_hot(idx, V)^T @ adj, i.e. a scatter-add of
    rows. The one-hot compares the f32 id with an f32 iota, so only an id that
    is exactly an integer in [0, V) adds its row; a fractional id (which the
    forward gather truncates) or one outside [0, V) (which the gather clamps)
    adds nothing."""
    out = np.zeros(w_shape, dtype=dtype)
    f = np.asarray(ids, dtype=np.float32).reshape(-1)
    idx = ids_to_index(f)
    rows = g.reshape((len(idx),) + tuple(w_shape[1:]))
    ok = (idx >= 0) & (idx < w_shape[0]) & (idx.astype(np.float32) == f)
    np.add.at(out, idx[ok], rows[ok])
    return out


def slice_rows_vjp(full_shape, start, g):
    """`slice_grad` -> `stablehlo.pad` back to the full shape (codegen/builtins.rs:208-271)."""
    out = np.zeros(full_shape, dtype=g.dtype)
    out[start:start + g.shape[0]] = g
    return out
