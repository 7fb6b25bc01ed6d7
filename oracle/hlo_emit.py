"""StableHLO text in the form Sheaf's emitter prints. TEST INFRASTRUCTURE ONLY.

Restates the printers of sheaf/src/lowering/stablehlo (module/func layout
emit.rs:73-139,240-257; elementwise operations.rs:9-158 with explicit
broadcast_in_dim of operands, broadcast.rs:36-100; reshape/transpose/iota
shape_ops.rs; dot_general dot_ops.rs:12-229; reduce reduce_ops.rs:11-107;
comparisons as subtract/sign/clamp/abs arithmetic and select through
`compare NE` compare_ops.rs:9-128; the generic row gather indexing_ops.rs:416-484;
one-hot tensor_ops.rs:163-217; slice_grad as pad codegen/builtins.rs:208-271)
so the executor's StableHLO front door can be driven with modules shaped like
the ones Sheaf's JIT hands to iree-compile: the MLP value_and_grad and the
nanoGPT value_and_grad (forward of examples/nanogpt/model.shf plus a backward
built from the VJP rules of sheaf/src/autodiff/reverse.rs).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import models


@dataclass(frozen=True)
class V:
    reg: str
    shape: tuple
    dt: str  # "f32" | "bf16" | "i32" | "i1"

    @property
    def ty(self) -> str:
        return ttype(self.shape, self.dt)


def ttype(shape, dt) -> str:
    return f"tensor<{'x'.join(str(d) for d in shape)}x{dt}>" if shape else f"tensor<{dt}>"


def fmt_float(v: float) -> str:
    if np.isinf(v):
        return "0xFF800000" if v < 0 else "0x7F800000"
    if float(v).is_integer() and abs(v) < 1e15:
        return f"{float(v):.1f}"
    return repr(float(v))


class Emitter:
    def __init__(self):
        self.lines: list[str] = []
        self.n = 0

    def _new(self) -> str:
        r = f"%{self.n}"
        self.n += 1
        return r

    def _op(self, text: str, shape, dt) -> V:
        r = self._new()
        self.lines.append(f"    {r} = {text}")
        return V(r, tuple(shape), dt)

    # ---- leaves -----------------------------------------------------------
    def const(self, v: float, dt: str = "f32") -> V:
        text = fmt_float(v)
        if np.isinf(v) and dt in ("bf16", "f16"):  # hex literals are the element's own bit pattern
            text = {("bf16", True): "0xFF80", ("bf16", False): "0x7F80", ("f16", True): "0xFC00",
                    ("f16", False): "0x7C00"}[(dt, v < 0)]
        return self._op(f"stablehlo.constant dense<{text}> : {ttype((), dt)}", (), dt)

    def const_array(self, values, dt: str = "f32") -> V:
        """dense<[[...]]> constant (constants.rs:90-115)."""
        a = np.asarray(values, dtype=np.float64)

        def lit(x):
            if x.ndim == 0:
                return fmt_float(float(x))
            return "[" + ", ".join(lit(y) for y in x) + "]"

        return self._op(f"stablehlo.constant dense<{lit(a)}> : {ttype(a.shape, dt)}", a.shape, dt)

    def bcast(self, x: V, shape, dims) -> V:
        d = ", ".join(str(i) for i in dims)
        return self._op(f"stablehlo.broadcast_in_dim {x.reg}, dims = [{d}] : ({x.ty}) -> {ttype(shape, x.dt)}", shape,
                        x.dt)

    def splat(self, v: float, shape, dt: str) -> V:
        return self.bcast(self.const(v, dt), shape, [])

    def to_shape(self, x: V, shape) -> V:
        """NumPy-style broadcast of x to `shape` (trailing alignment)."""
        shape = tuple(shape)
        if x.shape == shape:
            return x
        off = len(shape) - len(x.shape)
        if all(s == 1 for s in x.shape) and len(x.shape) > 0:
            x = self.reshape(x, ())
            return self.bcast(x, shape, [])
        return self.bcast(x, shape, [off + i for i in range(len(x.shape))])

    # ---- elementwise ------------------------------------------------------
    def binop(self, name: str, a: V, b: V) -> V:
        shape = tuple(np.broadcast_shapes(a.shape, b.shape))
        a, b = self.to_shape(a, shape), self.to_shape(b, shape)
        return self._op(f"stablehlo.{name} {a.reg}, {b.reg} : {ttype(shape, a.dt)}", shape, a.dt)

    def add(self, a, b):
        return self.binop("add", a, b)

    def sub(self, a, b):
        return self.binop("subtract", a, b)

    def mul(self, a, b):
        return self.binop("multiply", a, b)

    def div(self, a, b):
        return self.binop("divide", a, b)

    def maximum(self, a, b):
        return self.binop("maximum", a, b)

    def scal(self, v: float, like: V) -> V:
        return self.const(v, like.dt)

    def unary(self, name: str, a: V) -> V:
        return self._op(f"stablehlo.{name} {a.reg} : {a.ty}", a.shape, a.dt)

    def convert(self, a: V, dt: str) -> V:
        return self._op(f"stablehlo.convert {a.reg} : ({a.ty}) -> {ttype(a.shape, dt)}", a.shape, dt)

    def clamp(self, lo: V, x: V, hi: V) -> V:
        return self._op(f"stablehlo.clamp {lo.reg}, {x.reg}, {hi.reg} : {x.ty}", x.shape, x.dt)

    # ---- shape ------------------------------------------------------------
    def reshape(self, a: V, shape) -> V:
        return self._op(f"stablehlo.reshape {a.reg} : ({a.ty}) -> {ttype(shape, a.dt)}", shape, a.dt)

    def transpose(self, a: V, perm) -> V:
        shape = tuple(a.shape[p] for p in perm)
        d = ", ".join(str(p) for p in perm)
        return self._op(f"stablehlo.transpose {a.reg}, dims = [{d}] : ({a.ty}) -> {ttype(shape, a.dt)}", shape, a.dt)

    def swapaxes(self, a: V, i: int, j: int) -> V:
        perm = list(range(len(a.shape)))
        perm[i], perm[j] = perm[j], perm[i]
        return self.transpose(a, perm)

    def slice(self, a: V, starts, limits) -> V:
        shape = tuple(l - s for s, l in zip(starts, limits))
        d = ", ".join(f"{s}:{l}:1" for s, l in zip(starts, limits))
        return self._op(f"stablehlo.slice {a.reg} [{d}] : ({a.ty}) -> {ttype(shape, a.dt)}", shape, a.dt)

    def pad(self, a: V, low, high) -> V:
        z = self.const(0.0, a.dt)
        shape = tuple(s + l + h for s, l, h in zip(a.shape, low, high))
        j = lambda v: ", ".join(str(x) for x in v)  # noqa: E731
        return self._op(f"stablehlo.pad {a.reg}, {z.reg}, low = [{j(low)}], high = [{j(high)}], interior = "
                        f"[{j([0] * len(low))}] : ({a.ty}, {z.ty}) -> {ttype(shape, a.dt)}", shape, a.dt)

    def iota(self, shape, dim: int) -> V:
        return self._op(f"stablehlo.iota dim = {dim} : {ttype(shape, 'f32')}", shape, "f32")

    # ---- reductions -------------------------------------------------------
    def reduce(self, kind: str, a: V, axis: int, keepdims: bool) -> V:
        axis = axis % len(a.shape)
        init = self.const(0.0 if kind == "add" else float("-inf"), a.dt)
        shape = tuple(s for i, s in enumerate(a.shape) if i != axis)
        r = self._op(f"stablehlo.reduce({a.reg} init: {init.reg}) applies stablehlo.{kind} across dimensions = "
                     f"[{axis}] : ({a.ty}, {init.ty}) -> {ttype(shape, a.dt)}", shape, a.dt)
        if keepdims:
            r = self.reshape(r, tuple(1 if i == axis else s for i, s in enumerate(a.shape)))
        return r

    def sum(self, a: V, axis: int, keepdims=False) -> V:
        return self.reduce("add", a, axis, keepdims)

    def mean(self, a: V, axis: int, keepdims=False) -> V:
        n = a.shape[axis % len(a.shape)]
        return self.div(self.sum(a, axis, keepdims), self.scal(float(n), a))

    def sum_all(self, a: V) -> V:
        while a.shape:
            a = self.sum(a, 0)
        return a

    # ---- dot --------------------------------------------------------------
    def dot(self, a: V, b: V, lc, rc, lb=(), rb=()) -> V:
        lb, rb, lc, rc = list(lb), list(rb), list(lc), list(rc)
        batch = [a.shape[i] for i in lb]
        lfree = [a.shape[i] for i in range(len(a.shape)) if i not in lb and i not in lc]
        rfree = [b.shape[i] for i in range(len(b.shape)) if i not in rb and i not in rc]
        shape = tuple(batch + lfree + rfree)
        j = lambda v: ", ".join(str(x) for x in v)  # noqa: E731
        bd = f"batching_dims = [{j(lb)}] x [{j(rb)}], " if lb else ""
        return self._op(f"stablehlo.dot_general {a.reg}, {b.reg}, {bd}contracting_dims = [{j(lc)}] x [{j(rc)}] : "
                        f"({a.ty}, {b.ty}) -> {ttype(shape, a.dt)}", shape, a.dt)

    def matmul(self, a: V, b: V) -> V:
        """`@` (dot_ops.rs): rank-n x rank-2 contracts a's last dim with b's
        first; rank-4 x rank-4 batches the two leading dims."""
        if len(b.shape) == 2:
            return self.dot(a, b, [len(a.shape) - 1], [0])
        nb = len(a.shape) - 2
        return self.dot(a, b, [len(a.shape) - 1], [len(b.shape) - 2], list(range(nb)), list(range(nb)))

    # ---- comparisons, select (compare_ops.rs) ------------------------------
    def cmp(self, op: str, a: V, b: V) -> V:
        shape = tuple(np.broadcast_shapes(a.shape, b.shape))
        a, b = self.to_shape(a, shape), self.to_shape(b, shape)
        zero = self.splat(0.0, shape, a.dt)
        one = self.splat(1.0, shape, a.dt)
        if op in (">=", ">", "<=", "<"):
            first, second = (a, b) if op in (">=", ">") else (b, a)
            d = self.sub(first, second)
            sg = self.unary("sign", d)
            if op in (">=", "<="):
                sg = self.add(sg, one)
            return self.clamp(zero, sg, one)
        d = self.sub(a, b)
        diff = self.unary("abs", self.unary("sign", d))
        return diff if op == "!=" else self.sub(one, diff)

    def select(self, pred: V, t: V, f: V) -> V:
        """`where`: predicate and branches broadcast to one shape first."""
        shape = tuple(np.broadcast_shapes(pred.shape, t.shape, f.shape))
        pred = self.to_shape(pred, shape)
        zero = self.splat(0.0, shape, pred.dt)
        p = self._op(f"stablehlo.compare NE, {pred.reg}, {zero.reg}, FLOAT : ({pred.ty}, {pred.ty}) -> "
                     f"{ttype(shape, 'i1')}", shape, "i1")
        t, f = self.to_shape(t, shape), self.to_shape(f, shape)
        return self._op(f"stablehlo.select {p.reg}, {t.reg}, {f.reg} : {p.ty}, {t.ty}", shape, t.dt)

    # ---- gather / one-hot --------------------------------------------------
    def gather_rows(self, table: V, ids: V) -> V:
        idx = self.convert(ids, "i32")
        idx3 = self.reshape(idx, ids.shape + (1,))
        out = tuple(ids.shape) + tuple(table.shape[1:])
        r = self._new()
        nb = len(ids.shape)
        offs = ", ".join(str(nb + i) for i in range(len(table.shape) - 1))
        sizes = ", ".join(["1"] + [str(s) for s in table.shape[1:]])
        self.lines.append(
            f"    {r} = \"stablehlo.gather\"({table.reg}, {idx3.reg}) {{\n"
            f"      dimension_numbers = #stablehlo.gather<\n"
            f"        offset_dims = [{offs}],\n"
            f"        collapsed_slice_dims = [0],\n"
            f"        operand_batching_dims = [],\n"
            f"        start_indices_batching_dims = [],\n"
            f"        start_index_map = [0],\n"
            f"        index_vector_dim = {nb}>,\n"
            f"      slice_sizes = array<i64: {sizes}>,\n"
            f"      indices_are_sorted = false\n"
            f"    }} : ({table.ty}, {idx3.ty}) -> {ttype(out, table.dt)}")
        return V(r, out, table.dt)

    def one_hot(self, ids: V, n: int) -> V:
        shape = ids.shape + (n,)
        iota = self.iota(shape, len(shape) - 1)
        idx = self.reshape(ids, ids.shape + (1,))
        idx = self.bcast(idx, shape, list(range(len(shape))))
        mask = self.cmp("==", idx, iota)
        return self.select(mask, self.splat(1.0, shape, "f32"), self.splat(0.0, shape, "f32"))

    # ---- module -----------------------------------------------------------
    def module(self, name: str, fn: str, args: list[V], rets: list[V]) -> str:
        a = ", ".join(f"{x.reg}: {x.ty}" for x in args)
        r = rets[0].ty if len(rets) == 1 else "(" + ", ".join(x.ty for x in rets) + ")"
        out = ["// Generated by Sheaf", "//", "", f"module @{name} {{", f" func.func @{fn}({a}) -> {r} {{"]
        out += self.lines
        out.append(f"    return {', '.join(x.reg for x in rets)} : {', '.join(x.ty for x in rets)}")
        out += [" }", "}"]
        return "\n".join(out) + "\n"


def arg(i: int, shape, dt: str) -> V:
    return V(f"%arg{i}", tuple(shape), dt)


# ---------------------------------------------------------------------------
# composite ops (lib/nn.shf, inlined) and their VJPs (reverse.rs rules)
# ---------------------------------------------------------------------------

def layer_norm_nb(e: Emitter, x: V, g: V):
    """examples/nanogpt/model.shf:11-14; var two-pass (reduction_builtins.rs:287-358)."""
    m = e.mean(x, -1, keepdims=True)
    d = e.sub(x, m)
    v = e.mean(e.mul(d, d), -1, keepdims=True)
    s = e.unary("sqrt", e.add(v, e.scal(1e-5, x)))
    xh = e.div(d, s)
    return e.mul(xh, g), (d, s, xh)


def layer_norm_nb_vjp(e: Emitter, cache, g: V, dy: V):
    """`*`, `/`, `sqrt`, `var`, `mean`, `-` rules composed (reverse.rs:551-583,
    847-914, 961-967): returns dx, dgamma."""
    d, s, xh = cache
    n = float(xh.shape[-1])
    dg = e.mul(dy, xh)
    while len(dg.shape) > 1:
        dg = e.sum(dg, 0)
    dxh = e.mul(dy, g)
    # through (x - m) / s with s = sqrt(var + eps)
    dd = e.div(dxh, s)
    ds = e.sum(e.mul(e.mul(dxh, xh), e.scal(-1.0, xh)), -1, keepdims=True)
    ds = e.div(ds, s)                                   # d(1/s)-term: -sum(dxh*d)/s^2
    dv = e.div(ds, e.mul(e.scal(2.0, s), s))             # sqrt rule: /(2 sqrt)
    dd = e.add(dd, e.mul(e.mul(dv, e.scal(2.0 / n, d)), d))  # var rule: 2/n (x-m) adj
    dm = e.mul(e.sum(dd, -1, keepdims=True), e.scal(-1.0 / n, d))  # mean rule through (x - m)
    return e.add(dd, dm), dg


def gelu(e: Emitter, x: V) -> V:
    """lib/nn.shf:10-11."""
    inner = e.add(x, e.mul(e.scal(0.044715, x), e.mul(x, e.mul(x, x))))
    t = e.unary("tanh", e.mul(e.scal(0.7978846, x), inner))
    return e.mul(e.scal(0.5, x), e.mul(x, e.add(e.scal(1.0, x), t)))


def gelu_vjp(e: Emitter, x: V, g: V) -> V:
    x2 = e.mul(x, x)
    t = e.unary("tanh", e.mul(e.scal(0.7978846, x), e.add(x, e.mul(e.scal(0.044715, x), e.mul(x, x2)))))
    a = e.mul(e.scal(0.5, x), e.add(e.scal(1.0, x), t))
    sech2 = e.sub(e.scal(1.0, x), e.mul(t, t))
    kp = e.mul(e.scal(0.7978846, x), e.add(e.scal(1.0, x), e.mul(e.scal(0.134145, x), x2)))
    b = e.mul(e.scal(0.5, x), e.mul(e.mul(x, sech2), kp))
    return e.mul(g, e.add(a, b))


def softmax(e: Emitter, x: V) -> V:
    """lib/nn.shf:24-26."""
    ex = e.unary("exponential", e.sub(x, e.reduce("maximum", x, -1, True)))
    return e.div(ex, e.sum(ex, -1, keepdims=True))


def cross_entropy(e: Emitter, logits: V, y: V):
    """lib/nn.shf:44-50 and its VJP (softmax * sum(one_hot) - one_hot) / N
    (the mean, sum, multiply and log-softmax rules composed: a row whose
    one-hot is all zero gets no gradient)."""
    Vn = logits.shape[-1]
    flat = e.reshape(logits, (int(np.prod(logits.shape[:-1])), Vn))
    s = e.sub(flat, e.reduce("maximum", flat, -1, True))
    lse = e.unary("log", e.sum(e.unary("exponential", s), -1, keepdims=True))
    logp = e.sub(s, lse)
    yf = e.reshape(y, (flat.shape[0],))
    mask = e.one_hot(yf, Vn)
    if logits.dt != "f32":
        mask = e.convert(mask, logits.dt)
    tl = e.sum(e.mul(logp, mask), -1)
    loss = e.mul(e.mean(tl, 0), e.scal(-1.0, tl))
    n = float(flat.shape[0])
    p = e.unary("exponential", logp)
    dflat = e.div(e.sub(e.mul(p, e.sum(mask, -1, keepdims=True)), mask), e.scal(n, p))
    return loss, e.reshape(dflat, logits.shape)


# ---------------------------------------------------------------------------
# modules
# ---------------------------------------------------------------------------

def mlp_vag_module(batch=64, d_in=784, d_hidden=256, d_out=10, dt="f32") -> str:
    """MLP value_and_grad: mse(linear(gelu(linear(x, W1, b1)), W2, b2), y).
    Args: l1.W, l1.b, l2.W, l2.b (wrt), x, y. Returns loss, dW1, db1, dW2, db2."""
    e = Emitter()
    w1, b1, w2, b2 = arg(0, (d_in, d_hidden), dt), arg(1, (d_hidden,), dt), arg(2, (d_hidden, d_out), dt), \
        arg(3, (d_out,), dt)
    x, y = arg(4, (batch, d_in), dt), arg(5, (batch, d_out), dt)
    h = e.add(e.matmul(x, w1), b1)
    a = gelu(e, h)
    o = e.add(e.matmul(a, w2), b2)
    diff = e.sub(o, y)
    loss = e.mean(e.mean(e.mul(diff, diff), 1), 0)
    do = e.mul(diff, e.scal(2.0 / (batch * d_out), diff))
    dw2 = e.matmul(e.transpose(a, [1, 0]), do)
    db2 = e.sum(do, 0)
    da = e.matmul(do, e.transpose(w2, [1, 0]))
    dh = gelu_vjp(e, h, da)
    dw1 = e.matmul(e.transpose(x, [1, 0]), dh)
    db1 = e.sum(dh, 0)
    return e.module("__vag_mlp", "value_and_grad", [w1, b1, w2, b2, x, y], [loss, dw1, db1, dw2, db2])


def gpt_vag_module(cfg: models.GPTConfig, dt: str = "bf16") -> str:
    """nanoGPT value_and_grad (examples/nanogpt/train.shf:27-28): the forward
    of model.shf:85-113 + cross-entropy and a backward following the VJP
    rules. Args: the params leaves in sorted-key order, then x, y ids (f32)."""
    e = Emitter()
    B, T = cfg.batch, cfg.seq
    shapes = models.gpt_leaf_shapes(cfg)
    params = [arg(i, s, dt) for i, s in enumerate(shapes)]
    xid = arg(len(shapes), (B, T), "f32")
    yid = arg(len(shapes) + 1, (B, T), "f32")
    loss, grads = gpt_vag_graph(e, cfg, dt, params, xid, yid)
    return e.module("__vag_nanogpt", "value_and_grad", params + [xid, yid], [loss] + grads)


def gpt_vag_graph(e: Emitter, cfg: models.GPTConfig, dt: str, params, xid: V, yid: V):
    """Emits the nanoGPT loss and its gradients (one per params leaf)."""
    L, H, D, Vv, P, B, T = cfg.n_layer, cfg.n_head, cfg.n_embd, cfg.vocab_size, cfg.block_size, cfg.batch, cfg.seq
    Hd = D // H
    head = params[0]
    blocks = [params[1 + 6 * l: 7 + 6 * l] for l in range(L)]
    lnf, wpe, wte = params[1 + 6 * L], params[2 + 6 * L], params[3 + 6 * L]
    causal = e.cmp("==", _tril(e, T, dt), e.scal(1.0, V("", (), dt)))  # (== (tril (ones [T T])) 1.0)

    # forward
    x = e.add(e.gather_rows(wte, xid), e.reshape(e.slice(wpe, [0, 0], [T, D]), (1, T, D)))
    caches = []
    for (w_attn, w_proj, g1, g2, w_fc, w_fc2) in blocks:
        h1, c1 = layer_norm_nb(e, x, g1)
        qkv = []
        for i in range(3):
            w = e.slice(w_attn, [i * D, 0], [(i + 1) * D, D])
            z = e.matmul(h1, e.transpose(w, [1, 0]))
            qkv.append(e.swapaxes(e.reshape(z, (B, T, H, Hd)), 1, 2))
        q, k, v = qkv
        s = e.div(e.matmul(q, e.swapaxes(k, 2, 3)), e.scal(float(np.sqrt(Hd)), q))
        s = e.select(causal, s, e.scal(-1e10, s))
        p = softmax(e, s)
        o = e.reshape(e.swapaxes(e.matmul(p, v), 1, 2), (B, T, D))
        x_mid = e.add(x, e.matmul(o, e.transpose(w_proj, [1, 0])))
        h2, c2 = layer_norm_nb(e, x_mid, g2)
        u = e.matmul(h2, e.transpose(w_fc, [1, 0]))
        gu = gelu(e, u)
        x_new = e.add(x_mid, e.matmul(gu, e.transpose(w_fc2, [1, 0])))
        caches.append((x, h1, c1, q, k, v, p, o, x_mid, h2, c2, u, gu))
        x = x_new
    hf, cf = layer_norm_nb(e, x, lnf)
    logits = e.matmul(hf, e.transpose(head, [1, 0]))
    loss, dlogits = cross_entropy(e, logits, yid)

    # backward
    N = B * T
    flat = lambda t, w: e.reshape(t, (N, w))  # noqa: E731
    grads = [None] * len(params)
    grads[0] = e.matmul(e.transpose(flat(dlogits, Vv), [1, 0]), flat(hf, D))
    dhf = e.matmul(dlogits, head)
    dx, grads[1 + 6 * L] = layer_norm_nb_vjp(e, cf, lnf, dhf)
    for l in reversed(range(L)):
        w_attn, w_proj, g1, g2, w_fc, w_fc2 = blocks[l]
        x_in, h1, c1, q, k, v, p, o, x_mid, h2, c2, u, gu = caches[l]
        b0 = 1 + 6 * l
        grads[b0 + 5] = e.matmul(e.transpose(flat(dx, D), [1, 0]), flat(gu, 4 * D))
        du = gelu_vjp(e, u, e.matmul(dx, w_fc2))
        grads[b0 + 4] = e.matmul(e.transpose(flat(du, 4 * D), [1, 0]), flat(h2, D))
        dxl, grads[b0 + 3] = layer_norm_nb_vjp(e, c2, g2, e.matmul(du, w_fc))
        dx = e.add(dx, dxl)
        grads[b0 + 1] = e.matmul(e.transpose(flat(dx, D), [1, 0]), flat(o, D))
        do = e.swapaxes(e.reshape(e.matmul(dx, w_proj), (B, T, H, Hd)), 1, 2)
        dv = e.matmul(e.swapaxes(p, 2, 3), do)
        dp = e.matmul(do, e.swapaxes(v, 2, 3))
        ds = e.mul(p, e.sub(dp, e.sum(e.mul(dp, p), -1, keepdims=True)))
        ds = e.select(causal, ds, e.scal(0.0, ds))
        ds = e.div(ds, e.scal(float(np.sqrt(Hd)), ds))
        dq = e.matmul(ds, k)
        dk = e.matmul(e.swapaxes(ds, 2, 3), q)
        dws = []
        dh1 = None
        for i, dz in enumerate((dq, dk, dv)):
            dzf = flat(e.swapaxes(dz, 1, 2), D)
            dws.append(e.matmul(e.transpose(dzf, [1, 0]), flat(h1, D)))
            w = e.slice(w_attn, [i * D, 0], [(i + 1) * D, D])
            t = e.matmul(e.reshape(dzf, (B, T, D)), w)
            dh1 = t if dh1 is None else e.add(dh1, t)
        grads[b0 + 0] = e.pad(dws[0], [0, 0], [2 * D, 0])
        grads[b0 + 0] = e.add(grads[b0 + 0], e.pad(dws[1], [D, 0], [D, 0]))
        grads[b0 + 0] = e.add(grads[b0 + 0], e.pad(dws[2], [2 * D, 0], [0, 0]))
        dxl, grads[b0 + 2] = layer_norm_nb_vjp(e, c1, g1, dh1)
        dx = e.add(dx, dxl)
    # embedding: one_hot(idx, V)^T @ adj (reverse.rs:1108-1121); wpe: pad
    oh = e.one_hot(e.reshape(xid, (N,)), Vv)
    if dt != "f32":
        oh = e.convert(oh, dt)
    grads[3 + 6 * L] = e.matmul(e.transpose(oh, [1, 0]), flat(dx, D))
    grads[2 + 6 * L] = e.pad(e.sum(dx, 0), [0, 0], [P - T, 0])
    return loss, grads


def gpt_train_module(cfg: models.GPTConfig, dt: str = "bf16", b1=0.9, b2=0.95, eps=1e-8, wd=0.1, max_norm=1.0,
                     with_key=False) -> str:
    """nanoGPT train-step (examples/nanogpt/train.shf:26-33) as one module:
    value_and_grad, clip-by-global-norm and adamw-step (sheaf/lib/optim.shf,
    inlined with the literals train-step passes). Args: the state pytree's
    leaves in sorted-key order -- [key [4] when the state carries one], loss,
    m leaves, params leaves, t (f32), v leaves -- then x, y ids and lr (f32);
    returns the new state in the same order (`assoc` keeps the key)."""
    e = Emitter()
    B, T = cfg.batch, cfg.seq
    shapes = models.gpt_leaf_shapes(cfg)
    n = len(shapes)
    i = 0
    key = None
    if with_key:
        key = arg(0, (4,), "f32")
        i = 1
    loss0 = arg(i, (), dt)
    m = [arg(i + 1 + j, s, dt) for j, s in enumerate(shapes)]
    params = [arg(i + 1 + n + j, s, dt) for j, s in enumerate(shapes)]
    t = arg(i + 1 + 2 * n, (), "f32")
    v = [arg(i + 2 + 2 * n + j, s, dt) for j, s in enumerate(shapes)]
    xid = arg(i + 2 + 3 * n, (B, T), "f32")
    yid = arg(i + 3 + 3 * n, (B, T), "f32")
    lr = arg(i + 4 + 3 * n, (), "f32")
    loss, grads = gpt_vag_graph(e, cfg, dt, params, xid, yid)
    # clip-by-global-norm (optim.shf): sqrt of the f32 sum of every leaf's sum of squares
    total = e.const(0.0, "f32")
    for g in grads:
        sq = e.binop("power", g, e.scal(2.0, g))
        total = e.add(total, e.convert(e.sum_all(sq), "f32") if dt != "f32" else e.sum_all(sq))
    gnorm = e.unary("sqrt", total)
    factor = e.binop("minimum", e.const(1.0, "f32"), e.div(e.const(max_norm, "f32"),
                                                          e.add(gnorm, e.const(1e-8, "f32"))))
    fac = e.convert(factor, dt) if dt != "f32" else factor
    grads = [e.mul(g, fac) for g in grads]
    # adamw-step
    t1 = e.add(t, e.const(1.0, "f32"))
    bcm = e.div(e.const(1.0, "f32"), e.sub(e.const(1.0, "f32"), e.binop("power", e.const(b1, "f32"), t1)))
    bcv = e.div(e.const(1.0, "f32"), e.sub(e.const(1.0, "f32"), e.binop("power", e.const(b2, "f32"), t1)))
    cast = (lambda x: e.convert(x, dt)) if dt != "f32" else (lambda x: x)  # noqa: E731
    bcm_t, bcv_t, lr_t = cast(bcm), cast(bcv), cast(lr)
    new_m, new_v, new_p = [], [], []
    for mj, vj, pj, gj in zip(m, v, params, grads):
        nm = e.add(e.mul(e.const(b1, dt), mj), e.mul(e.const(1.0 - b1, dt), gj))
        nv = e.add(e.mul(e.const(b2, dt), vj), e.mul(e.const(1.0 - b2, dt), e.mul(gj, gj)))
        upd = e.div(e.mul(nm, bcm_t), e.add(e.unary("sqrt", e.mul(nv, bcv_t)), e.const(eps, dt)))
        np_ = e.sub(pj, e.mul(lr_t, e.add(e.mul(e.const(wd, dt), pj), upd)))
        new_m.append(nm)
        new_v.append(nv)
        new_p.append(np_)
    ins = ([key] if key else []) + [loss0] + m + params + [t] + v + [xid, yid, lr]
    outs = ([key] if key else []) + [loss] + new_m + new_p + [t1] + new_v
    return e.module("__jit_train_step", "train_step", ins, outs)


def _tril(e: Emitter, T: int, dt: str) -> V:
    """tril(ones [T T]) as the emitter builds it (tensor_ops.rs:101-118):
    where(col <= row, 1, 0) from two iotas."""
    row = e.iota((T, T), 0)
    col = e.iota((T, T), 1)
    keep = e.cmp("<=", col, row)
    ones = e.splat(1.0, (T, T), "f32")
    zeros = e.splat(0.0, (T, T), "f32")
    t = e.select(keep, ones, zeros)
    return e.convert(t, dt) if dt != "f32" else t
