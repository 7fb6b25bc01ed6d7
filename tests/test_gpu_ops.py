"""Per-kernel parity through the op-level C ABI (include/sheaf_b200_ops.h)
against the CPU oracle (oracle/ops.py): layer-norm fwd/VJP, fused
cross-entropy fwd+VJP, embedding gather (bit-exact) and its scatter-add VJP,
fused causal attention fwd/VJP. Device memory comes from torch (plumbing only).
"""
import numpy as np
import pytest

from oracle import dtype as odt
from oracle import ops
from tests.parity import TOL_BF16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu

ELEMS = {"f32": 0x21000020, "bf16": 0x22000010}


def _dev(a, dt, dev):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dt).to(dev)


def _rt(a, kind):
    """Round host data the way it is uploaded (bf16 RNE for bf16)."""
    return odt.round_bf16(a) if kind == "bf16" else np.asarray(a, np.float32)


def _stream():
    import torch

    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("kind", ["f32", "bf16"])
@pytest.mark.parametrize("rows,D", [(1000, 384), (77, 768), (64, 4096),
                                    # block-per-row kernels: more rows than blocks, a ragged last chunk
                                    (1500, 4096), (700, 1024), (33, 8192), (2000, 2052)])
def test_layernorm(kind, rows, D, cuda):
    import torch
    import sheaf_b200 as sb

    L = sb.lib()
    dt = torch.float32 if kind == "f32" else torch.bfloat16
    rng = np.random.default_rng(rows + D)
    x = (rng.standard_normal((rows, D)) * 3 + 1).astype(np.float32)
    g = _rt(rng.standard_normal(D).astype(np.float32), kind)
    dy = rng.standard_normal((rows, D)).astype(np.float32)
    dres0 = rng.standard_normal((rows, D)).astype(np.float32)
    xd, gd = _dev(x, torch.float32, cuda), _dev(g, dt, cuda)
    yd = torch.empty(rows, D, dtype=dt, device=cuda)
    mean = torch.empty(rows, device=cuda)
    rstd = torch.empty(rows, device=cuda)
    assert L.sb_op_layernorm_fwd(ELEMS[kind], xd.data_ptr(), gd.data_ptr(), yd.data_ptr(), mean.data_ptr(),
                                 rstd.data_ptr(), rows, D, _stream()) == 0
    y_ref, cache = ops.layer_norm_nb(x.astype(np.float64), g.astype(np.float64))
    tol = TOL_F32 if kind == "f32" else TOL_BF16
    assert_close(yd.float().cpu().numpy(), y_ref, tol, "ln y")
    dyd, dres = _dev(dy, torch.float32, cuda), _dev(dres0, torch.float32, cuda)
    dg = torch.empty(D, dtype=dt, device=cuda)
    wsb = L.sb_op_layernorm_bwd_workspace_size(rows, D)
    ws = torch.empty(wsb // 4 + 1, device=cuda)
    assert L.sb_op_layernorm_bwd(ELEMS[kind], dyd.data_ptr(), xd.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
                                 gd.data_ptr(), dres.data_ptr(), dg.data_ptr(), ws.data_ptr(), wsb, rows, D,
                                 _stream()) == 0
    dx_ref, dg_ref = ops.layer_norm_nb_vjp(cache, g.astype(np.float64), dy.astype(np.float64))
    assert_close(dres.cpu().numpy() - dres0, dx_ref, 1e-5 if kind == "f32" else 1e-5, "ln dx")
    xd64 = x.astype(np.float64)
    terms = np.abs(dy.astype(np.float64) * ((xd64 - xd64.mean(1, keepdims=True)) /
                                            np.sqrt(xd64.var(1, keepdims=True) + 1e-5))).sum(0)
    assert_close(dg.float().cpu().numpy(), dg_ref, tol, "ln dgamma", sum_abs=terms)
    torch.cuda.synchronize()


@pytest.mark.parametrize("kind", ["f32", "bf16"])
@pytest.mark.parametrize("rows,V,ld", [(4096, 65, 72), (300, 1000, 1000), (64, 50304, 50304),
                                       # wide rows: 16-byte chunks plus a scalar tail (V % 8 != 0), an
                                       # unaligned row stride (scalar warp path), more rows than blocks
                                       (2000, 50257, 50264), (37, 4099, 4099), (1500, 2048, 2048)])
def test_cross_entropy(kind, rows, V, ld, cuda):
    import torch
    import sheaf_b200 as sb

    L = sb.lib()
    dt = torch.float32 if kind == "f32" else torch.bfloat16
    rng = np.random.default_rng(V)
    logits = _rt((rng.standard_normal((rows, V)) * 2).astype(np.float32), kind)
    tgt = rng.integers(0, V, rows).astype(np.float32)
    full = np.zeros((rows, ld), np.float32)
    full[:, :V] = logits
    ld_ = _dev(full, dt, cuda)
    dl = torch.zeros(rows, ld, dtype=dt, device=cuda)
    td = _dev(tgt, torch.float32, cuda)
    loss = torch.zeros(1, device=cuda)
    wsb = L.sb_op_cross_entropy_workspace_size(rows)
    ws = torch.empty(wsb // 4 + 1, device=cuda)
    assert L.sb_op_cross_entropy(ELEMS[kind], ld_.data_ptr(), ld, rows, V, td.data_ptr(), dl.data_ptr(), ld,
                                 ws.data_ptr(), wsb, loss.data_ptr(), _stream()) == 0
    ref_loss = ops.cross_entropy(logits.astype(np.float64), tgt)
    ref_d = ops.cross_entropy_vjp(logits.astype(np.float64), tgt)
    assert abs(loss.item() - ref_loss) <= 1e-5 * abs(ref_loss)
    tol = TOL_F32 if kind == "f32" else TOL_BF16
    assert_close(dl[:, :V].float().cpu().numpy(), ref_d, tol, "dlogits")


@pytest.mark.parametrize("kind", ["f32", "bf16"])
@pytest.mark.parametrize("V", [65, 5000])
def test_embedding(kind, V, cuda):
    import torch
    import sheaf_b200 as sb

    L = sb.lib()
    dt = torch.float32 if kind == "f32" else torch.bfloat16
    B, T, P, D = 8, 96, 128, 384
    rng = np.random.default_rng(V)
    wte = _rt(rng.standard_normal((V, D)).astype(np.float32) * 0.02, kind)
    wpe = _rt(rng.standard_normal((P, D)).astype(np.float32) * 0.02, kind)
    ids = rng.integers(0, V, (B, T)).astype(np.float32)
    ids[0, :5] = [0, V - 1, 3, 3, 3]
    x = torch.empty(B * T, D, device=cuda)
    idd = _dev(ids, torch.float32, cuda)
    assert L.sb_op_embedding_fwd(ELEMS[kind], idd.data_ptr(), _dev(wte, dt, cuda).data_ptr(),
                                 _dev(wpe, dt, cuda).data_ptr(), x.data_ptr(), B * T, T, V, D, _stream()) == 0
    ref = (ops.embedding(wte, ids) + wpe[:T][None]).reshape(B * T, D).astype(np.float32)
    assert np.array_equal(x.cpu().numpy(), ref), "gathered rows must be bit-exact"
    dx = rng.standard_normal((B * T, D)).astype(np.float32)
    dwte = torch.empty(V, D, dtype=dt, device=cuda)
    dwpe = torch.empty(P, D, dtype=dt, device=cuda)
    wsb = L.sb_op_embedding_bwd_workspace_size(V, D)
    ws = torch.empty(wsb // 4 + 1, device=cuda)
    assert L.sb_op_embedding_bwd(ELEMS[kind], idd.data_ptr(), _dev(dx, torch.float32, cuda).data_ptr(), B, T, P, V, D,
                                 dwte.data_ptr(), dwpe.data_ptr(), ws.data_ptr(), wsb, _stream()) == 0
    tol = TOL_F32 if kind == "f32" else TOL_BF16
    assert_close(dwte.float().cpu().numpy(), ops.embedding_vjp((V, D), ids, dx.astype(np.float64), np.float64), tol,
                 "dwte")
    assert_close(dwpe.float().cpu().numpy(),
                 ops.slice_rows_vjp((P, D), 0, dx.reshape(B, T, D).astype(np.float64).sum(0)), tol, "dwpe")


# Token ids at the edges of the reference's semantics: the forward gather
# converts f32 -> i32 (truncation) and clamps into [0, V) (indexing_ops.rs:
# 416-484), while the one-hot of the VJP and of the cross-entropy compares the
# f32 id with an f32 iota (tensor_ops.rs:163-217), so a fractional or
# out-of-range id matches no class there.
def _edge_list(V):
    return [2.5, 3.0, -1.0, -0.0, 0.75, -2.5, V - 1, V, V + 5, 1e6, V - 0.25, 5.0]


EDGE_IDS = _edge_list(65)


def _edge_ids(V, n, rng):
    """n uniform ids in [0, V) whose first entries are the edge cases."""
    ids = rng.integers(0, V, n).astype(np.float32)
    ed = np.array(_edge_list(V), np.float32)
    ids[:len(ed)] = ed
    return ids


@pytest.mark.parametrize("kind", ["f32", "bf16"])
@pytest.mark.parametrize("V", [65, 5000])
def test_embedding_edge_ids(kind, V, cuda):
    """Fractional, negative and out-of-range f32 ids: the gather truncates and
    clamps (rows compared bit-exactly); the scatter-add drops every id that is
    not exactly an integer in [0, V), so a row reached only through such ids
    stays exactly zero."""
    import torch
    import sheaf_b200 as sb

    L = sb.lib()
    dt = torch.float32 if kind == "f32" else torch.bfloat16
    B, T, P, D = 2, 64, 64, 128
    rng = np.random.default_rng(11 + V)
    wte = _rt(rng.standard_normal((V, D)).astype(np.float32) * 0.02, kind)
    wpe = _rt(rng.standard_normal((P, D)).astype(np.float32) * 0.02, kind)
    ids = _edge_ids(V, B * T, rng)
    # row 2 is reached only through 2.5 / -2.5 (truncated to 2 / -2): keep other ids off it
    ids[len(EDGE_IDS):][ids[len(EDGE_IDS):] == 2.0] = 3.0
    ids = ids.reshape(B, T)
    idd = _dev(ids, torch.float32, cuda)
    x = torch.empty(B * T, D, device=cuda)
    assert L.sb_op_embedding_fwd(ELEMS[kind], idd.data_ptr(), _dev(wte, dt, cuda).data_ptr(),
                                 _dev(wpe, dt, cuda).data_ptr(), x.data_ptr(), B * T, T, V, D, _stream()) == 0
    ref = (ops.embedding(wte, ids) + wpe[:T][None]).reshape(B * T, D).astype(np.float32)
    assert np.array_equal(x.cpu().numpy(), ref), "gathered rows must be bit-exact"
    dx = rng.standard_normal((B * T, D)).astype(np.float32)
    dwte = torch.full((V, D), float("nan"), dtype=dt, device=cuda)
    dwpe = torch.empty(P, D, dtype=dt, device=cuda)
    wsb = L.sb_op_embedding_bwd_workspace_size(V, D)
    ws = torch.empty(wsb // 4 + 1, device=cuda)
    assert L.sb_op_embedding_bwd(ELEMS[kind], idd.data_ptr(), _dev(dx, torch.float32, cuda).data_ptr(), B, T, P, V, D,
                                 dwte.data_ptr(), dwpe.data_ptr(), ws.data_ptr(), wsb, _stream()) == 0
    got = dwte.float().cpu().numpy()
    exp = ops.embedding_vjp((V, D), ids, dx.astype(np.float64), np.float64)
    # which rows receive anything is index work: the zero pattern is exact
    assert np.array_equal(got == 0, exp == 0)
    assert not got[2].any(), "row 2 is reached only through fractional ids"
    assert_close(got, exp, TOL_F32 if kind == "f32" else TOL_BF16, "dwte")


@pytest.mark.parametrize("kind", ["f32", "bf16"])
@pytest.mark.parametrize("V", [65, 50304])
def test_cross_entropy_edge_targets(kind, V, cuda):
    """Targets that are fractional or outside [0, V) have an all-zero one-hot
    row: they add nothing to the loss (still divided by every row) and their
    dlogits rows are exactly zero."""
    import torch
    import sheaf_b200 as sb

    L = sb.lib()
    dt = torch.float32 if kind == "f32" else torch.bfloat16
    rows = 96
    ld = (V + 7) // 8 * 8
    rng = np.random.default_rng(5 + V)
    logits = _rt((rng.standard_normal((rows, V)) * 2).astype(np.float32), kind)
    tgt = _edge_ids(V, rows, rng)
    full = np.zeros((rows, ld), np.float32)
    full[:, :V] = logits
    dl = torch.full((rows, ld), float("nan"), dtype=dt, device=cuda)
    dl[:, V:] = 0
    td = _dev(tgt, torch.float32, cuda)
    loss = torch.zeros(1, device=cuda)
    wsb = L.sb_op_cross_entropy_workspace_size(rows)
    ws = torch.empty(wsb // 4 + 1, device=cuda)
    assert L.sb_op_cross_entropy(ELEMS[kind], _dev(full, dt, cuda).data_ptr(), ld, rows, V, td.data_ptr(),
                                 dl.data_ptr(), ld, ws.data_ptr(), wsb, loss.data_ptr(), _stream()) == 0
    ref_loss = ops.cross_entropy(logits.astype(np.float64), tgt)
    ref_d = ops.cross_entropy_vjp(logits.astype(np.float64), tgt)
    assert abs(loss.item() - ref_loss) <= 1e-5 * abs(ref_loss)
    got = dl[:, :V].float().cpu().numpy()
    invalid = ~((tgt == np.trunc(tgt)) & (tgt >= 0) & (tgt < V))
    assert invalid.sum() >= 8
    assert not got[invalid].any(), "rows without a class get no gradient"
    assert_close(got, ref_d, TOL_F32 if kind == "f32" else TOL_BF16, "dlogits")


def _attn_ref(qkv, B, T, H, Hd):
    q, k, v = (qkv[:, i * H * Hd:(i + 1) * H * Hd].reshape(B, T, H, Hd).transpose(0, 2, 1, 3) for i in range(3))
    s = q @ np.swapaxes(k, -1, -2) / np.sqrt(Hd)
    mask = np.tril(np.ones((T, T), bool))
    s = np.where(mask, s, ops.MASK_FILL)
    p = ops.softmax(s)
    o = (p @ v).transpose(0, 2, 1, 3).reshape(B * T, H * Hd)
    lse = (s.max(-1) + np.log(np.exp(s - s.max(-1, keepdims=True)).sum(-1))).reshape(-1)
    return q, k, v, p, o, lse


@pytest.mark.parametrize("kind", ["f32", "bf16"])
@pytest.mark.parametrize("B,T,H,Hd", [(2, 256, 2, 64), (1, 100, 3, 64), (2, 128, 4, 32), (1, 1024, 2, 64),
                                     (1, 300, 2, 64), (24, 300, 6, 64)])
def test_attention(kind, B, T, H, Hd, cuda):
    import torch
    import sheaf_b200 as sb

    L = sb.lib()
    dt = torch.float32 if kind == "f32" else torch.bfloat16
    D = H * Hd
    rng = np.random.default_rng(T + H)
    qkv = _rt(rng.standard_normal((B * T, 3 * D)).astype(np.float32), kind)
    do = _rt(rng.standard_normal((B * T, D)).astype(np.float32), kind)
    qd = _dev(qkv, dt, cuda)
    o = torch.empty(B * T, D, dtype=dt, device=cuda)
    lse = torch.empty(B * H * T, device=cuda)
    assert L.sb_op_attention_fwd(ELEMS[kind], qd.data_ptr(), o.data_ptr(), lse.data_ptr(), B, T, H, Hd,
                                 _stream()) == 0
    q, k, v, p, o_ref, lse_ref = _attn_ref(qkv.astype(np.float64), B, T, H, Hd)
    tol = TOL_F32 if kind == "f32" else TOL_BF16
    assert_close(o.float().cpu().numpy(), o_ref, tol, "o")
    assert_close(lse.cpu().numpy(), lse_ref, 1e-5, "lse")
    # VJP against the oracle's rules, with the device's own o as input
    dod = _dev(do, dt, cuda)
    dqkv = torch.empty(B * T, 3 * D, dtype=dt, device=cuda)
    wsb = L.sb_op_attention_bwd_workspace_size(ELEMS[kind], B, T, H, Hd)
    ws = torch.empty(wsb // 4 + 1, device=cuda)
    assert L.sb_op_attention_bwd(ELEMS[kind], qd.data_ptr(), o.data_ptr(), dod.data_ptr(), lse.data_ptr(),
                                 dqkv.data_ptr(), ws.data_ptr(), wsb, B, T, H, Hd, _stream()) == 0
    dO = do.astype(np.float64).reshape(B, T, H, Hd).transpose(0, 2, 1, 3)
    dv = np.swapaxes(p, -1, -2) @ dO
    dp = dO @ np.swapaxes(v, -1, -2)
    ds = ops.softmax_vjp(p, dp)
    ds = np.where(np.tril(np.ones((T, T), bool)), ds, 0.0) / np.sqrt(Hd)
    dq, dk = ds @ k, np.swapaxes(ds, -1, -2) @ q
    ref = np.concatenate([z.transpose(0, 2, 1, 3).reshape(B * T, D) for z in (dq, dk, dv)], axis=1)
    got = dqkv.float().cpu().numpy()
    for i, nm in enumerate(["dq", "dk", "dv"]):
        assert_close(got[:, i * D:(i + 1) * D], ref[:, i * D:(i + 1) * D], tol, nm)
    torch.cuda.synchronize()
    assert L.sb_op_device_error() == 0


@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_gelu(kind, cuda):
    import torch
    import sheaf_b200 as sb

    L = sb.lib()
    dt = torch.float32 if kind == "f32" else torch.bfloat16
    rng = np.random.default_rng(5)
    n = 100003  # not a multiple of 8: exercises the tail loop
    x = _rt((rng.standard_normal(n) * 3).astype(np.float32), kind)
    g = _rt(rng.standard_normal(n).astype(np.float32), kind)
    xd, gd = _dev(x, dt, cuda), _dev(g, dt, cuda)
    y = torch.empty(n, dtype=dt, device=cuda)
    assert L.sb_op_gelu_fwd(ELEMS[kind], xd.data_ptr(), y.data_ptr(), n, _stream()) == 0
    tol = TOL_F32 if kind == "f32" else TOL_BF16
    assert_close(y.float().cpu().numpy(), ops.gelu(x.astype(np.float64)), tol, "gelu")
    assert L.sb_op_gelu_bwd(ELEMS[kind], xd.data_ptr(), gd.data_ptr(), y.data_ptr(), n, _stream()) == 0
    assert_close(y.float().cpu().numpy(), ops.gelu_vjp(x.astype(np.float64), g.astype(np.float64)), tol, "gelu vjp")
