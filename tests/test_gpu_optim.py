"""clip-by-global-norm + AdamW (nanoGPT's train-step optimizer) through the C
ABI against the oracle restatement of sheaf/lib/optim.shf:19-32,42-51.

Leaves have ragged sizes (not multiples of the kernels' chunk) and there are
more of them than one launch's leaf table holds; the gradients are scaled so
that clipping is active in one case and inactive in another.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import dtype as odt
from oracle import optim

pytestmark = pytest.mark.gpu

SHAPES = [(65, 384), (384,), (1152, 384), (7,), (4097,), (3, 5, 11)] + [(100 + i,) for i in range(34)]


def _ptrs(ts):
    return (C.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _leaves(rng, scale):
    return [(rng.standard_normal(s) * scale).astype(np.float32) for s in SHAPES]


def _ulp_bf16(x):
    """One bf16 ulp of |x| (8 significant bits)."""
    a = np.abs(np.asarray(x, np.float64))
    e = np.floor(np.log2(np.where(a > 0, a, 2.0 ** -133)))
    return 2.0 ** (e - 7)


@pytest.mark.parametrize("kind", ["f32", "bf16"])
@pytest.mark.parametrize("gscale,max_norm", [(0.05, 1.0), (1e-4, 1.0), (0.05, 0.0)],
                         ids=["clipped", "unclipped", "no-clip"])
def test_adamw_step_matches_oracle(kind, gscale, max_norm, cuda):
    import torch
    import sheaf_b200 as sb

    rng = np.random.default_rng(7)
    p = _leaves(rng, 0.02)
    g = _leaves(rng, gscale)
    m = _leaves(rng, 1e-3)
    v = [np.abs(x) for x in _leaves(rng, 1e-4)]
    bf = kind == "bf16"
    if bf:
        p, g, m, v = ([odt.round_bf16(x) for x in lst] for lst in (p, g, m, v))
    dt = torch.bfloat16 if bf else torch.float32
    elem = sb.ELEM_BF16 if bf else sb.ELEM_F32
    dev = lambda lst: [torch.from_numpy(x.astype(np.float32)).to(dt).to(cuda) for x in lst]  # noqa: E731
    pd, gd, md, vd = dev(p), dev(g), dev(m), dev(v)
    po = [torch.empty_like(x) for x in pd]
    t0, lr = 3.0, 6e-4
    t_in = torch.tensor([t0], device=cuda)
    t_out = torch.zeros(1, device=cuda)
    lr_d = torch.tensor([lr], device=cuda)
    norm = torch.zeros(1, device=cuda)
    counts = (C.c_int64 * len(SHAPES))(*[int(np.prod(s)) for s in SHAPES])
    L = sb.lib()
    wsb = L.sb_op_adamw_workspace_size(counts, len(SHAPES))
    ws = torch.empty(wsb // 4 + 1, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    # m and v updated in place (outputs alias inputs); p to fresh buffers
    rc = L.sb_op_adamw_step(elem, len(SHAPES), counts, _ptrs(gd), _ptrs(pd), _ptrs(md), _ptrs(vd), _ptrs(po),
                            _ptrs(md), _ptrs(vd), t_in.data_ptr(), t_out.data_ptr(), lr_d.data_ptr(), 0.9, 0.95,
                            1e-8, 0.1, max_norm, norm.data_ptr(), ws.data_ptr(), wsb, stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert L.sb_op_device_error() == 0
    ref_p, ref_m, ref_v, ref_t = optim.adamw_step(p, g, m, v, t0, lr, max_norm=max_norm, bf16=bf)
    assert float(t_out.item()) == ref_t
    ref_norm = optim.global_norm(g)
    assert abs(norm.item() - ref_norm) <= 1e-5 * ref_norm
    if max_norm > 0:
        assert (optim.clip_factor(g, max_norm) < 1.0) == (gscale > 0.01)
    # magnitude of the terms each result sums (m' and p' can cancel to ~0,
    # where only an absolute bound of a few f32 roundings of the terms holds)
    f = optim.clip_factor(g, max_norm) if max_norm > 0 else 1.0
    gf = [np.abs(np.asarray(x, np.float64)) * f for x in g]
    terms = {"m": [0.9 * np.abs(mm) + 0.1 * x for mm, x in zip(m, gf)],
             "v": [0.95 * vv + 0.05 * x * x for vv, x in zip(v, gf)],
             "p": [np.abs(pp) + 2 * np.abs(np.asarray(e, np.float64) - pp) for pp, e in zip(p, ref_p)]}
    for name, got, ref in (("p", po, ref_p), ("m", md, ref_m), ("v", vd, ref_v)):
        for i, (a, e) in enumerate(zip(got, ref)):
            a = a.float().cpu().numpy().astype(np.float64)
            e = np.asarray(e, np.float64)
            cancel = 2.0 ** -20 * terms[name][i]
            if bf:
                # one bf16 ulp (of the larger magnitude: the two roundings may
                # straddle a power of two); exact ties round differently since
                # the kernel's f32 b1 = 0.9f lies below 0.9, float64's above
                bound = _ulp_bf16(np.maximum(np.abs(a), np.abs(e))) + cancel + 1e-30
            else:
                bound = 1e-5 * np.abs(e).max() + 2e-6 * np.abs(e) + cancel
            assert (np.abs(a - e) <= bound).all(), (name, i, np.abs(a - e).max())


def test_global_norm_op(cuda):
    import torch
    import sheaf_b200 as sb

    rng = np.random.default_rng(3)
    g = _leaves(rng, 0.3)
    gd = [torch.from_numpy(x).to(cuda) for x in g]
    counts = (C.c_int64 * len(SHAPES))(*[int(np.prod(s)) for s in SHAPES])
    L = sb.lib()
    wsb = L.sb_op_adamw_workspace_size(counts, len(SHAPES))
    ws = torch.empty(wsb // 4 + 1, device=cuda)
    out = torch.zeros(1, device=cuda)
    assert L.sb_op_global_norm(sb.ELEM_F32, len(SHAPES), counts, _ptrs(gd), out.data_ptr(), ws.data_ptr(), wsb,
                               torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    ref = optim.global_norm(g)
    assert abs(out.item() - ref) <= 1e-5 * ref


def test_adamw_rejects_bad_arguments(cuda):
    import torch
    import sheaf_b200 as sb

    L = sb.lib()
    x = torch.zeros(4, device=cuda)
    counts = (C.c_int64 * 1)(4)
    one = _ptrs([x])
    # workspace too small -> 5; zero-sized leaf -> 1
    assert L.sb_op_adamw_step(sb.ELEM_F32, 1, counts, one, one, one, one, one, one, one, x.data_ptr(), x.data_ptr(),
                              x.data_ptr(), 0.9, 0.95, 1e-8, 0.1, 1.0, None, x.data_ptr(), 4, None) == 5
    zero = (C.c_int64 * 1)(0)
    assert L.sb_op_adamw_step(sb.ELEM_F32, 1, zero, one, one, one, one, one, one, one, x.data_ptr(), x.data_ptr(),
                              x.data_ptr(), 0.9, 0.95, 1e-8, 0.1, 1.0, None, x.data_ptr(), 4096, None) == 1
