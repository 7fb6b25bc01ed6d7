"""Evaluates StableHLO text op by op on the CPU. TEST INFRASTRUCTURE ONLY.

An oracle for modules run through the executor's text front door that rounds
where the reference rounds: the reference compiles every op of the module in
the op's own declared element type (a bf16 module computes every
elementwise op, dot_general and reduce in bf16; sheaf/src/lowering/stablehlo
operations.rs:9-158, dot_ops.rs:444-449 `dot_result_type`, reduce_ops.rs:37-51
with the init typed as the input), so each op's result here is the exact
(fp64) value of the op on its already-rounded operands, rounded once to the
op's result type (bf16 round-to-nearest-even as core/dtype.rs:204-216, f32,
i32 by truncation as `stablehlo.convert`, i1). dot_general and reduce are
evaluated in fp64 and rounded once: the correctly rounded result of the op,
against which a bf16 accumulation (the reference's) and the executor's f32
accumulation are both approximations.

Supported forms: the ones the reference's emitter prints for value_and_grad
modules (Appendix of the op text forms: constant incl. hex and dense arrays,
broadcast_in_dim, elementwise binary and unary ops, convert, clamp, reshape,
transpose, slice, pad, iota, reduce add/maximum/minimum/multiply,
dot_general, compare, select, the generic row gather, return).
"""
from __future__ import annotations

import re
import struct

import numpy as np

from . import dtype as odt

_TYPE = re.compile(r"tensor<([^>]*)>")


def parse_type(t: str):
    """'tensor<4x8xbf16>' -> ((4, 8), 'bf16'); 'tensor<f32>' -> ((), 'f32')."""
    m = _TYPE.fullmatch(t.strip())
    if not m:
        raise ValueError(f"not a tensor type: {t!r}")
    parts = m.group(1).split("x")
    return tuple(int(p) for p in parts[:-1]), parts[-1]


def round_to(x, dt: str) -> np.ndarray:
    """Rounds fp64 values to the element type `dt` (kept as fp64 for floats)."""
    x = np.asarray(x)
    if dt == "f32":
        return np.asarray(x, np.float64).astype(np.float32).astype(np.float64)
    if dt == "bf16":
        return odt.round_bf16(np.asarray(x, np.float64).astype(np.float32)).astype(np.float64)
    if dt == "f16":
        return np.asarray(x, np.float64).astype(np.float16).astype(np.float64)
    if dt == "i32":
        return np.asarray(x).astype(np.int64)
    if dt == "i1":
        return np.asarray(x).astype(bool)
    raise ValueError(f"element type {dt}")


def _ints(s: str) -> list[int]:
    return [int(v) for v in re.findall(r"-?\d+", s)]


def _hex_value(h: str, dt: str) -> float:
    bits = int(h, 16)
    if dt == "bf16":
        return struct.unpack("<f", struct.pack("<I", bits << 16))[0]
    if dt == "f16":
        return float(np.frombuffer(struct.pack("<H", bits), np.float16)[0])
    return struct.unpack("<f", struct.pack("<I", bits))[0]


def _dense(lit: str, shape, dt: str) -> np.ndarray:
    lit = lit.strip()
    if lit.startswith("0x"):
        v = np.array(_hex_value(lit, dt))
    elif lit in ("true", "false"):
        v = np.array(lit == "true")
    else:
        v = np.array(eval(lit, {"__builtins__": {}}, {"inf": np.inf, "nan": np.nan}), np.float64)  # nested lists
    if v.shape != tuple(shape):
        v = np.broadcast_to(v, shape)
    return round_to(v, dt)


_BIN = {
    "add": np.add, "subtract": np.subtract, "multiply": np.multiply, "divide": np.divide,
    "maximum": np.maximum, "minimum": np.minimum, "power": np.power, "remainder": np.fmod,
    "atan2": np.arctan2,
}
_UN = {
    "tanh": np.tanh, "sqrt": np.sqrt, "rsqrt": lambda v: 1.0 / np.sqrt(v), "exponential": np.exp, "log": np.log,
    "abs": np.abs, "negate": np.negative, "sign": np.sign, "sine": np.sin, "cosine": np.cos, "floor": np.floor,
    "ceil": np.ceil, "logistic": lambda v: 1.0 / (1.0 + np.exp(-v)), "not": np.logical_not,
}
_CMP = {"EQ": np.equal, "NE": np.not_equal, "LT": np.less, "LE": np.less_equal, "GT": np.greater,
        "GE": np.greater_equal}
_RED = {"add": (np.add, np.sum), "maximum": (np.maximum, np.max), "minimum": (np.minimum, np.min),
        "multiply": (np.multiply, np.prod)}
_REG = re.compile(r"%[\w.]+")


def _broadcast_in_dim(a, dims, shape):
    dims = list(dims)
    order = sorted(range(len(dims)), key=lambda i: dims[i])
    a = np.transpose(a, order) if len(order) > 1 else a
    new = [1] * len(shape)
    for i, d in enumerate(sorted(dims)):
        new[d] = a.shape[i]
    return np.broadcast_to(a.reshape(new), shape)


def _pad(a, z, low, high, interior):
    if any(v < 0 for v in list(low) + list(high) + list(interior)):
        raise ValueError("pad: negative padding is not supported by the oracle")
    shape = [l + h + s + max(s - 1, 0) * i for s, l, h, i in zip(a.shape, low, high, interior)]
    out = np.full(shape, z, dtype=np.float64 if a.dtype != bool else bool)
    idx = tuple(slice(l, l + (s - 1) * (i + 1) + 1 if s else l, i + 1) for s, l, i in zip(a.shape, low, interior))
    out[idx] = a
    return out


def _dot_general(a, b, lb, rb, lc, rc):
    letters = iter("abcdefghijklmnopqrstuvwxyz")
    la = [None] * a.ndim
    lbb = [None] * b.ndim
    bat = []
    for i, j in zip(lb, rb):
        c = next(letters)
        la[i] = lbb[j] = c
        bat.append(c)
    for i, j in zip(lc, rc):
        c = next(letters)
        la[i] = lbb[j] = c
    lfree, rfree = [], []
    for i in range(a.ndim):
        if la[i] is None:
            la[i] = next(letters)
            lfree.append(la[i])
    for j in range(b.ndim):
        if lbb[j] is None:
            lbb[j] = next(letters)
            rfree.append(lbb[j])
    spec = f"{''.join(la)},{''.join(lbb)}->{''.join(bat + lfree + rfree)}"
    return np.einsum(spec, a, b, optimize=True)


def _statements(body_lines):
    """Joins each op with its continuation lines (the gather's attribute block)."""
    stmts = []
    for ln in body_lines:
        t = ln.strip()
        if not t or t.startswith("//"):
            continue
        if t.startswith("%") or t.startswith("return"):
            stmts.append(t)
        elif stmts:
            stmts[-1] += " " + t
    return stmts


def _eval_op(rhs: str, env: dict):
    """One statement's right-hand side -> its value (rounded to its type)."""
    shape, dt = parse_type(_TYPE.findall(rhs)[-1].join(("tensor<", ">")))
    if rhs.startswith('"stablehlo.gather"'):
        a, idx = (env[r] for r in _REG.findall(rhs.split(")")[0]))
        if "collapsed_slice_dims = [0]" not in rhs or "start_index_map = [0]" not in rhs:
            raise ValueError("gather: only the row gather form is supported")
        rows = np.clip(np.asarray(idx).astype(np.int64)[..., 0], 0, a.shape[0] - 1)  # start indices are clamped
        return round_to(a[rows], dt)
    m = re.match(r"stablehlo\.(\w+)", rhs)
    if not m:
        raise ValueError(f"unsupported statement: {rhs[:80]}")
    op = m.group(1)
    head = rhs.split(" : ")[0]
    regs = [env[r] for r in _REG.findall(head)]
    if op == "constant":
        lit = re.match(r"stablehlo\.constant dense<(.*)>\s*:\s*tensor<", rhs).group(1)
        return _dense(lit, shape, dt)
    if op in _BIN:
        with np.errstate(all="ignore"):
            return round_to(_BIN[op](regs[0], regs[1]), dt)
    if op in _UN:
        with np.errstate(all="ignore"):
            return round_to(_UN[op](regs[0]), dt)
    if op == "broadcast_in_dim":
        dims = _ints(re.search(r"dims = \[([^\]]*)\]", rhs).group(1))
        return _broadcast_in_dim(regs[0], dims, shape)
    if op == "convert":
        src = parse_type(re.search(r"\((tensor<[^>]*>)\)", rhs).group(1))[1]
        v = regs[0]
        if dt in ("i32",) and src not in ("i32", "i1"):
            v = np.trunc(v)
        return round_to(v, dt)
    if op == "clamp":
        return round_to(np.minimum(np.maximum(regs[1], regs[0]), regs[2]), dt)
    if op == "reshape":
        return regs[0].reshape(shape)
    if op == "transpose":
        return np.transpose(regs[0], _ints(re.search(r"dims = \[([^\]]*)\]", rhs).group(1)))
    if op == "slice":
        spec = re.search(r"\[([^\]]*)\]", head).group(1)
        sl = tuple(slice(*[int(v) for v in part.split(":")]) for part in spec.split(","))
        return regs[0][sl]
    if op == "pad":
        get = lambda k: _ints(re.search(k + r" = \[([^\]]*)\]", rhs).group(1))  # noqa: E731
        return _pad(regs[0], float(regs[1]), get("low"), get("high"), get("interior"))
    if op == "iota":
        d = int(re.search(r"dim = (\d+)", rhs).group(1))
        ar = np.arange(shape[d], dtype=np.float64).reshape([-1 if i == d else 1 for i in range(len(shape))])
        return round_to(np.broadcast_to(ar, shape), dt)
    if op == "reduce":
        kind = re.search(r"applies stablehlo\.(\w+)", rhs).group(1)
        dims = tuple(_ints(re.search(r"across dimensions = \[([^\]]*)\]", rhs).group(1)))
        comb, red = _RED[kind]
        return round_to(comb(red(regs[0], axis=dims), regs[1]), dt)
    if op == "dot_general":
        bm = re.search(r"batching_dims = \[([^\]]*)\] x \[([^\]]*)\]", rhs)
        cm = re.search(r"contracting_dims = \[([^\]]*)\] x \[([^\]]*)\]", rhs)
        lb, rb = (_ints(bm.group(1)), _ints(bm.group(2))) if bm else ([], [])
        return round_to(_dot_general(regs[0], regs[1], lb, rb, _ints(cm.group(1)), _ints(cm.group(2))), dt)
    if op == "compare":
        direction = re.match(r"stablehlo\.compare\s+(\w+)", rhs).group(1)
        return _CMP[direction](regs[0], regs[1])
    if op == "select":
        return np.where(regs[0], regs[1], regs[2])
    raise ValueError(f"stablehlo.{op} is not supported by the oracle evaluator")


def evaluate(text: str, inputs, fn: str | None = None) -> list[np.ndarray]:
    """Runs function `fn` (the first one by default) of the module `text` on
    `inputs` (host arrays, rounded to the argument types) and returns its
    results as fp64 arrays (booleans for i1)."""
    lines = [ln.split("//")[0].rstrip() for ln in text.splitlines()]
    starts = [i for i, ln in enumerate(lines) if "func.func @" in ln]
    if fn is not None:
        starts = [i for i in starts if re.search(r"func\.func @" + re.escape(fn) + r"\(", lines[i])]
    if not starts:
        raise ValueError("function not found")
    s = starts[0]
    header = lines[s]
    while not header.endswith("{"):  # a signature printed over several lines
        s += 1
        header += " " + lines[s].strip()
    args = re.findall(r"(%arg\d+): (tensor<[^>]*>)", header)
    if len(args) != len(inputs):
        raise ValueError(f"expected {len(args)} inputs, got {len(inputs)}")
    env = {}
    for (reg, ty), x in zip(args, inputs):
        shp, dt = parse_type(ty)
        v = round_to(np.asarray(x, np.float64 if dt not in ("i1",) else bool), dt)
        if v.shape != shp:
            raise ValueError(f"{reg}: shape {v.shape} != {shp}")
        env[reg] = v
    body = []
    for ln in lines[s + 1:]:
        if ln.strip() == "}":
            break
        body.append(ln)
    for st in _statements(body):
        if st.startswith("return"):
            regs = _REG.findall(st.split(" : ")[0])
            return [np.array(env[r]) for r in regs]
        lhs, rhs = st.split(" = ", 1)
        env[lhs.strip()] = _eval_op(rhs.strip(), env)
    raise ValueError("function has no return")
