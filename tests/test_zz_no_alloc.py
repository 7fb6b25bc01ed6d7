"""sb_op_layernorm_bwd_noalloc: the layer-norm VJP for callers that cannot
allocate device memory while they run (a host runtime that owns the device
heap and hands this library only finished buffers and a stream, or a
latency-critical loop that cannot take cudaMalloc's device-wide sync).

The variant keeps its scratch in a fixed array inside the library instead of
a caller workspace. Checked through the C ABI against the workspace-taking
sb_op_layernorm_bwd and against the oracle's layer-norm VJP, on calls in a
row with different shapes (so contents left in the shared array by one call
must not leak into the next), up to the widest accepted row (4096, where
the array holds the partials of only 8 blocks and every block strides over
many rows), plus the size limit. This file is collected last on purpose.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ELEMS = {"f32": 0x21000020, "bf16": 0x22000010}
SB_OPERR_SCRATCH = 6


def _case(kind, rows, D, seed, dev):
    import torch

    dt = torch.float32 if kind == "f32" else torch.bfloat16
    rng = np.random.default_rng(seed)
    t = lambda a, d=torch.float32: torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(d).to(dev)
    x = t(rng.standard_normal((rows, D)) * 2 + 0.5)
    mean = x.mean(1)
    rstd = 1.0 / torch.sqrt(x.var(1, unbiased=False) + 1e-5)
    return dict(x=x, mean=mean, rstd=rstd, gamma=t(rng.standard_normal(D), dt), dy=t(rng.standard_normal((rows, D))),
                dres=t(rng.standard_normal((rows, D))), dt=dt)


def _with_workspace(L, kind, c, rows, D, stream):
    import torch

    dres = c["dres"].clone()
    dg = torch.empty(D, dtype=c["dt"], device=dres.device)
    wsb = L.sb_op_layernorm_bwd_workspace_size(rows, D)
    ws = torch.empty(wsb // 4 + 1, device=dres.device)
    rc = L.sb_op_layernorm_bwd(ELEMS[kind], c["dy"].data_ptr(), c["x"].data_ptr(), c["mean"].data_ptr(),
                               c["rstd"].data_ptr(), c["gamma"].data_ptr(), dres.data_ptr(), dg.data_ptr(),
                               ws.data_ptr(), wsb, rows, D, stream)
    assert rc == 0
    return dres, dg


def _no_alloc(L, kind, c, rows, D, stream):
    import torch

    dres = c["dres"].clone()
    dg = torch.full((D,), float("nan"), dtype=c["dt"], device=dres.device)
    rc = L.sb_op_layernorm_bwd_noalloc(ELEMS[kind], c["dy"].data_ptr(), c["x"].data_ptr(), c["mean"].data_ptr(),
                                       c["rstd"].data_ptr(), c["gamma"].data_ptr(), dres.data_ptr(), dg.data_ptr(),
                                       rows, D, stream)
    assert rc == 0
    return dres, dg


@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_no_alloc_matches_workspace_entry_point(kind, cuda):
    import torch
    import sheaf_b200 as sb

    L = sb.lib()
    stream = torch.cuda.current_stream().cuda_stream
    tol = 1e-5 if kind == "f32" else 2e-2
    # calls in a row, each with a different shape; the last at the widest
    # accepted rows
    for rows, D, seed in [(1000, 384, 1), (77, 768, 2), (300, 4096, 3), (1000, 384, 4)]:
        c = _case(kind, rows, D, seed, cuda)
        ref_dres, ref_dg = _with_workspace(L, kind, c, rows, D, stream)
        got_dres, got_dg = _no_alloc(L, kind, c, rows, D, stream)
        torch.cuda.synchronize()
        # dx rows do not depend on how rows are spread over blocks: identical
        assert torch.equal(got_dres, ref_dres)
        a, e = got_dg.double().cpu().numpy(), ref_dg.double().cpu().numpy()
        assert np.isfinite(a).all()
        assert np.abs(a - e).max() <= tol * np.abs(e).max()
        _check_oracle(c, got_dres, got_dg, tol)
    assert L.sb_op_device_error() == 0


def _check_oracle(c, got_dres, got_dg, tol):
    """dres - dres0 and dgamma against the oracle's layer-norm VJP (fp64)."""
    from oracle import ops
    from tests.parity import assert_close

    x = c["x"].double().cpu().numpy()
    g = c["gamma"].double().cpu().numpy()
    dy = c["dy"].double().cpu().numpy()
    _, cache = ops.layer_norm_nb(x, g)
    dx_ref, dg_ref = ops.layer_norm_nb_vjp(cache, g, dy)
    assert_close(got_dres.double().cpu().numpy() - c["dres"].double().cpu().numpy(), dx_ref, 1e-5, "dx")
    assert_close(got_dg.double().cpu().numpy(), dg_ref, tol, "dgamma")


def test_no_alloc_rejects_rows_wider_than_its_scratch(cuda):
    import torch
    import sheaf_b200 as sb

    L = sb.lib()
    D = 8192
    x = torch.zeros(8, D, device=cuda)
    v = torch.zeros(8, device=cuda)
    g = torch.zeros(D, device=cuda)
    rc = L.sb_op_layernorm_bwd_noalloc(ELEMS["f32"], x.data_ptr(), x.data_ptr(), v.data_ptr(), v.data_ptr(),
                                       g.data_ptr(), x.data_ptr(), g.data_ptr(), 8, D,
                                       torch.cuda.current_stream().cuda_stream)
    assert rc == SB_OPERR_SCRATCH
