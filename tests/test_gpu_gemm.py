"""GEMM parity (tcgen05 bf16 and CUDA-core fp32) through the C ABI.

The reference op is `stablehlo.dot_general` as Sheaf emits it for `@`
(sheaf/src/lowering/stablehlo/dot_ops.rs:32-79) and the transposed operands
of its VJP (sheaf/src/autodiff/reverse.rs:585-689). Checked against a plain
fp64 matmul of the same (bf16-rounded) operands.
"""
import ctypes as C

import pytest

pytestmark = pytest.mark.gpu

CASES = [
    # M, N, K, trans_a, trans_b, lda_pad, ldc_pad
    (256, 256, 128, 0, 1, 0, 0),
    (2048, 1152, 384, 0, 1, 0, 0),
    (300, 200, 136, 0, 1, 0, 0),
    (512, 384, 1536, 0, 0, 0, 0),
    (384, 1536, 4096, 1, 0, 0, 0),
    (1152, 384, 2048, 1, 0, 0, 0),
    (65, 384, 2048, 1, 0, 15, 0),
    (512, 65, 384, 0, 1, 0, 15),
    (640, 96, 192, 1, 1, 0, 0),
    (96, 66, 4096, 1, 1, 0, 2),  # one tile, long K, N not a multiple of 4: no split-K
    (512, 1536, 4096, 1, 0, 0, 0),  # CTA-pair tiles with split-K
    (4160, 256, 256, 0, 1, 0, 0),  # CTA pairs, the last pair tile half outside M
    (16384, 1152, 384, 0, 1, 0, 0),  # 256-wide pair tiles, the last column of tiles half outside N
    (16384, 384, 384, 0, 1, 0, 0),  # 384-wide pair tiles (N = 256 + 128 UMMAs), K-major B
    (8192, 384, 1536, 0, 0, 0, 0),  # 384-wide pair tiles, MN-major B
    (4096, 300, 256, 1, 1, 0, 4),  # 384-wide pair tiles, columns past N (the N = 128 part partly empty)
]


def _run(elem, M, N, K, ta, tb, lda_pad, ldc_pad, dev):
    import torch
    import sheaf_b200 as sb

    dt = torch.bfloat16 if elem == sb.ELEM_BF16 else torch.float32
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N * 3 + K)
    a_log = torch.randn(M, K, generator=g)
    b_log = torch.randn(K, N, generator=g)
    a_store = a_log.t().contiguous() if ta else a_log
    b_store = b_log.t().contiguous() if tb else b_log
    if lda_pad:
        pad = torch.zeros(a_store.shape[0], a_store.shape[1] + lda_pad)
        pad[:, : a_store.shape[1]] = a_store
        a_store = pad
    a_dev = a_store.to(dt).to(dev)
    b_dev = b_store.to(dt).to(dev)
    ldc = N + ldc_pad
    c_dev = torch.full((M, ldc), float("nan"), dtype=torch.float32, device=dev)
    L = sb.lib()
    ws_bytes = L.sb_op_matmul_workspace_size(elem, ta, tb, M, N, K)
    ws = torch.empty(max(ws_bytes // 4, 1), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream().cuda_stream
    rc = L.sb_op_matmul(elem, a_dev.data_ptr(), a_dev.stride(0), ta, b_dev.data_ptr(), b_dev.stride(0), tb, M, N, K,
                        c_dev.data_ptr(), ldc, sb.ELEM_F32, ws.data_ptr(), ws_bytes, stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert L.sb_op_device_error() == 0
    a_r = a_log.to(dt).double()
    b_r = b_log.to(dt).double()
    ref = a_r @ b_r
    out = c_dev[:, :N].double().cpu()
    return out, ref


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}x{c[1]}x{c[2]}_t{c[3]}{c[4]}" for c in CASES])
def test_matmul_bf16(case, cuda):
    import sheaf_b200 as sb

    out, ref = _run(sb.ELEM_BF16, *case, cuda)
    assert out.isfinite().all()
    err = (out - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 1e-5 * scale + 1e-4, (err, scale)


@pytest.mark.parametrize("case", CASES, ids=[f"{c[0]}x{c[1]}x{c[2]}_t{c[3]}{c[4]}" for c in CASES])
def test_matmul_f32(case, cuda):
    import sheaf_b200 as sb

    out, ref = _run(sb.ELEM_F32, *case, cuda)
    err = (out - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 1e-5 * scale, (err, scale)


@pytest.mark.parametrize("M,N,K,ldc", [(512, 256, 256, 256), (200, 200, 4096, 200), (130, 132, 4096, 135)])
def test_matmul_bf16_output(M, N, K, ldc, cuda):
    """bf16 output rounding (RNE) on the tcgen05 epilogue, and after the
    split-K reduction (long K, few tiles; odd output row stride)."""
    import torch
    import sheaf_b200 as sb

    g = torch.Generator(device="cpu").manual_seed(11)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16).to(cuda)
    b = torch.randn(N, K, generator=g).to(torch.bfloat16).to(cuda)
    cbuf = torch.full((M, ldc), float("nan"), dtype=torch.bfloat16, device=cuda)
    L = sb.lib()
    wsb = L.sb_op_matmul_workspace_size(sb.ELEM_BF16, 0, 1, M, N, K)
    ws = torch.empty(max(wsb // 4, 1), dtype=torch.float32, device=cuda)
    rc = L.sb_op_matmul(sb.ELEM_BF16, a.data_ptr(), K, 0, b.data_ptr(), K, 1, M, N, K, cbuf.data_ptr(), ldc,
                        sb.ELEM_BF16, ws.data_ptr(), wsb, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    c = cbuf[:, :N]
    exact = a.double() @ b.double().t()
    ref = exact.to(torch.bfloat16).double()
    diff = (c.double() - ref).abs()
    # one RNE rounding of the fp32 accumulator on each side (2^-8 relative
    # each) plus the fp32 accumulation error, which is absolute: K * 2^-24 of
    # sum |a_k b_k| (it dominates where the dot product cancels)
    acc_err = K * 2.0 ** -24 * (a.double().abs() @ b.double().abs().t())
    assert (diff <= 2.0 ** -8 * (ref.abs() + exact.abs()) + 2 * acc_err).all()


@pytest.mark.parametrize("kind,M,N,K", [("bf16", 16384, 1536, 384), ("bf16", 300, 520, 128), ("f32", 300, 520, 128)])
def test_matmul_gelu(kind, M, N, K, cuda):
    """The fc layer's fused epilogue (sb_op_matmul_gelu): y = gelu(u) and
    dy = gelu'(u) for u = A @ B^T, u rounded to bf16 first on the bf16 path
    (the module's dot_general result type). Oracle: lib/nn.shf:10-11 and its
    VJP in fp64 (oracle.ops)."""
    import numpy as np
    import torch
    import sheaf_b200 as sb

    from oracle import dtype as odt
    from oracle import ops

    bf = kind == "bf16"
    elem = sb.ELEM_BF16 if bf else sb.ELEM_F32
    dt = torch.bfloat16 if bf else torch.float32
    g = torch.Generator(device="cpu").manual_seed(M + N + K)
    a = (torch.randn(M, K, generator=g) * 0.1).to(dt)
    b = (torch.randn(N, K, generator=g) * 0.1).to(dt)
    y = torch.full((M, N), float("nan"), dtype=dt, device=cuda)
    dy = torch.full((M, N), float("nan"), dtype=dt, device=cuda)
    L = sb.lib()
    ad, bd = a.to(cuda), b.to(cuda)
    rc = L.sb_op_matmul_gelu(elem, ad.data_ptr(), K, bd.data_ptr(), K, M, N, K, y.data_ptr(), dy.data_ptr(), N,
                             torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert L.sb_op_device_error() == 0
    u = a.double().numpy() @ b.double().numpy().T
    if bf:
        u = odt.round_bf16(u.astype(np.float32)).astype(np.float64)
    ey = ops.gelu(u)
    edy = ops.gelu_vjp(u, np.ones_like(u))
    tol = 2e-2 if bf else 1e-5
    for got, ref, nm in ((y, ey, "gelu"), (dy, edy, "gelu'")):
        gg = got.float().cpu().double().numpy()
        assert np.isfinite(gg).all(), nm
        err = np.abs(gg - ref)
        assert err.max() <= tol * np.abs(ref).max(), (nm, err.max())
        assert (err <= tol * (1 + np.abs(ref))).all(), nm


@pytest.mark.parametrize("kind,M,N,K,tb", [("bf16", 16384, 1536, 384, 0), ("bf16", 300, 520, 128, 1),
                                           ("f32", 300, 520, 128, 0)])
def test_matmul_mul(kind, M, N, K, tb, cuda):
    """C = (A @ op(B)) * aux (sb_op_matmul_mul), the fc2 VJP through gelu'
    of the nanoGPT plan: the product rounded once, on the bf16 path, after
    the multiply in f32."""
    import numpy as np
    import torch
    import sheaf_b200 as sb

    bf = kind == "bf16"
    elem = sb.ELEM_BF16 if bf else sb.ELEM_F32
    dt = torch.bfloat16 if bf else torch.float32
    g = torch.Generator(device="cpu").manual_seed(M + 3 * N + K)
    a = (torch.randn(M, K, generator=g) * 0.1).to(dt)
    b_log = (torch.randn(K, N, generator=g) * 0.1).to(dt)
    b = b_log.t().contiguous() if tb else b_log
    aux = torch.randn(M, N, generator=g).to(dt)
    c = torch.full((M, N), float("nan"), dtype=dt, device=cuda)
    L = sb.lib()
    ad, bd, xd = a.to(cuda), b.to(cuda), aux.to(cuda)
    rc = L.sb_op_matmul_mul(elem, ad.data_ptr(), K, 0, bd.data_ptr(), bd.stride(0), tb, M, N, K, xd.data_ptr(), N,
                            c.data_ptr(), N, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert L.sb_op_device_error() == 0
    ref = (a.double().numpy() @ b_log.double().numpy()) * aux.double().numpy()
    got = c.float().cpu().double().numpy()
    tol = 2e-2 if bf else 1e-5
    err = np.abs(got - ref)
    assert np.isfinite(got).all() and err.max() <= tol * np.abs(ref).max()
    assert (err <= tol * (1 + np.abs(ref))).all()
