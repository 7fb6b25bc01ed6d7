"""nanoGPT value_and_grad through the executor C ABI against the CPU oracle.

Module: sb_module_create_gpt_vag (the fused graph of examples/nanogpt/model.shf
+ cross-entropy); invoked with sb_call("<module>.value_and_grad", leaves..., x, y)
exactly as Sheaf's try_jit_vag calls a compiled VAG module
(sheaf/src/interpreter/iree_dispatch.rs:172-176). Inputs are the seeded
synthetic workload of oracle.models (Threefry init, randint token ids).
"""
import numpy as np
import pytest

from oracle import dtype as odt
from oracle import models
from tests.parity import TOL_BF16, TOL_F32, assert_close, rel_err

pytestmark = pytest.mark.gpu

BF16 = 0x22000010
F32 = 0x21000020


def run_vag(cfg, kind, leaves, x, y, calls=1):
    from sheaf_b200.runtime import Session

    s = Session(0)
    elem = BF16 if kind == "bf16" else F32
    s.create_gpt_vag("gpt", n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd, block_size=cfg.block_size,
                     vocab_size=cfg.vocab_size, batch=cfg.batch, seq=cfg.seq, elem=elem)
    bufs = [s.upload(l, elem) for l in leaves] + [s.upload(x, F32), s.upload(y, F32)]
    results = []
    for _ in range(calls):
        outs = s.call("gpt.value_and_grad", bufs)
        results.append([o.to_host() for o in outs])
    s.synchronize()
    return results


CFGS = {
    "tiny": models.GPTConfig(n_layer=2, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=4, seq=64),
    "nanogpt_b2": models.GPTConfig(batch=2),
    # 4096 tokens: the weight-gradient GEMMs contract over more than one
    # 2048-token split, attention items outnumber the SMs
    "nanogpt_b16": models.GPTConfig(batch=16),
}


@pytest.mark.parametrize("kind", ["f32", "bf16"])
@pytest.mark.parametrize("name", list(CFGS))
def test_vag_matches_oracle(name, kind, cuda):
    cfg = CFGS[name]
    leaves, x, y = models.gpt_inputs(cfg)
    if kind == "bf16":
        leaves = [odt.round_bf16(l) for l in leaves]
    ref_loss, ref_grads = models.gpt_value_and_grad(leaves, x, y, cfg, dtype=np.float64)
    (out,) = run_vag(cfg, kind, leaves, x, y)
    tol = TOL_F32 if kind == "f32" else TOL_BF16
    assert out[0].shape == ()
    assert abs(float(out[0]) - ref_loss) <= tol * abs(ref_loss), (float(out[0]), ref_loss)
    names = models.gpt_leaf_names(cfg)
    assert len(out) == 1 + len(names)
    for nm, g, r in zip(names, out[1:], ref_grads):
        assert_close(g, r, tol, nm)


def test_vag_full_nanogpt_matches_oracle(cuda):
    """The benchmarked configuration itself (6L/6H/384, B=64, T=256, bf16):
    loss and all 40 gradients against the oracle (evaluated in f32, far inside
    the bf16 bar). This plan takes the paths smaller batches do not: 384-wide
    CTA-pair tiles, six-way split-K over 16,384 tokens on the side stream,
    persistent attention with several items per CTA."""
    cfg = models.NANOGPT_CHAR
    leaves, x, y = models.gpt_inputs(cfg)
    leaves = [odt.round_bf16(l) for l in leaves]
    (out,) = run_vag(cfg, "bf16", leaves, x, y)
    ref_loss, ref_grads = models.gpt_value_and_grad(leaves, x, y, cfg, dtype=np.float32)
    assert abs(float(out[0]) - ref_loss) <= TOL_BF16 * abs(ref_loss), (float(out[0]), ref_loss)
    names = models.gpt_leaf_names(cfg)
    assert len(out) == 1 + len(names)
    for nm, g, r in zip(names, out[1:], ref_grads):
        assert_close(g, r, TOL_BF16, nm)


@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_vag_edge_token_ids(kind, cuda):
    """Fractional, negative and out-of-range f32 ids in x and y: the gather
    truncates and clamps, the embedding VJP and the cross-entropy one-hot drop
    them (compare in f32, tensor_ops.rs:163-217)."""
    cfg = CFGS["tiny"]
    leaves, x, y = models.gpt_inputs(cfg)
    if kind == "bf16":
        leaves = [odt.round_bf16(l) for l in leaves]
    edge = np.array([2.5, -1.0, -0.0, 0.75, 64.0, 65.0, 70.0, 64.75, -2.5, 1e6], np.float32)
    x, y = x.copy(), y.copy()
    x[0, :len(edge)] = edge
    y[1, 3:3 + len(edge)] = edge
    ref_loss, ref_grads = models.gpt_value_and_grad(leaves, x, y, cfg, dtype=np.float64)
    (out,) = run_vag(cfg, kind, leaves, x, y)
    tol = TOL_F32 if kind == "f32" else TOL_BF16
    assert abs(float(out[0]) - ref_loss) <= tol * abs(ref_loss), (float(out[0]), ref_loss)
    for nm, g, r in zip(models.gpt_leaf_names(cfg), out[1:], ref_grads):
        assert_close(g, r, tol, nm)


def test_vag_graph_replay_is_deterministic(cuda):
    """Call 1 runs eagerly, call 2 captures the CUDA graph, call 3 replays it:
    all three must agree bit for bit."""
    cfg = CFGS["tiny"]
    leaves, x, y = models.gpt_inputs(cfg)
    leaves = [odt.round_bf16(l) for l in leaves]
    r = run_vag(cfg, "bf16", leaves, x, y, calls=3)
    for a, b in zip(r[0], r[1]):
        assert np.array_equal(a, b)
    for a, b in zip(r[0], r[2]):
        assert np.array_equal(a, b)


def test_vag_full_nanogpt_properties(cuda):
    """The full nanoGPT-char workload (B=64, T=256): loss near ln(65) at init,
    every gradient finite and of the right shape, and the per-position
    embedding gradient rows beyond T exactly zero (the slice VJP's pad)."""
    cfg = models.NANOGPT_CHAR
    leaves, x, y = models.gpt_inputs(cfg)
    leaves = [odt.round_bf16(l) for l in leaves]
    (out,) = run_vag(cfg, "bf16", leaves, x, y)
    loss = float(out[0])
    assert abs(loss - np.log(65.0)) < 0.1, loss
    for g, shp in zip(out[1:], models.gpt_leaf_shapes(cfg)):
        assert g.shape == shp
        assert np.isfinite(g).all()
    # positions >= T of wpe get no gradient (pad of the slice VJP)
    assert cfg.seq == cfg.block_size or not out[-2][cfg.seq:].any()
    # the loss itself against the oracle's forward at full size (f32)
    from oracle import ops

    logits = models.gpt_forward_logits(leaves, x, cfg, dtype=np.float32)
    ref = float(ops.cross_entropy(logits, y))
    assert abs(loss - ref) <= TOL_BF16 * abs(ref), (loss, ref)


def test_gpt2_small_shape_matches_oracle(cuda):
    """GPT-2-small shape (12L/12H/768, V=50304, block 1024), bf16, at one
    sequence of 64 tokens (the oracle's fp64 evaluation stays in seconds)."""
    cfg = models.GPTConfig(n_layer=12, n_head=12, n_embd=768, block_size=1024, vocab_size=50304, batch=1, seq=64)
    leaves, x, y = models.gpt_inputs(cfg)
    leaves = [odt.round_bf16(l) for l in leaves]
    (out,) = run_vag(cfg, "bf16", leaves, x, y)
    ref_loss, ref_grads = models.gpt_value_and_grad(leaves, x, y, cfg, dtype=np.float64)
    assert abs(float(out[0]) - ref_loss) <= TOL_BF16 * abs(ref_loss)
    for nm, g, r in zip(models.gpt_leaf_names(cfg), out[1:], ref_grads):
        assert_close(g, r, TOL_BF16, nm)


def test_gpt2_small_shape_at_full_context_matches_oracle(cuda):
    """GPT-2-small widths (12 heads, d 768, V=50304) at the full 1024-token
    context, two layers, one sequence, bf16: attention over 1024 positions
    (8 key tiles per query tile), the 50304-wide cross-entropy and head GEMMs,
    the atomic embedding VJP of a large vocabulary. Oracle evaluated in f32."""
    cfg = models.GPTConfig(n_layer=2, n_head=12, n_embd=768, block_size=1024, vocab_size=50304, batch=1, seq=1024)
    leaves, x, y = models.gpt_inputs(cfg)
    leaves = [odt.round_bf16(l) for l in leaves]
    (out,) = run_vag(cfg, "bf16", leaves, x, y)
    ref_loss, ref_grads = models.gpt_value_and_grad(leaves, x, y, cfg, dtype=np.float32)
    assert abs(float(out[0]) - ref_loss) <= TOL_BF16 * abs(ref_loss), (float(out[0]), ref_loss)
    for nm, g, r in zip(models.gpt_leaf_names(cfg), out[1:], ref_grads):
        assert_close(g, r, TOL_BF16, nm)


def test_vag_reads_resident_parameters_in_place(cuda):
    """Parameters passed as resident device buffers are read where they lie:
    alternating two parameter sets (eager call, graph capture, recaptures on
    every change of addresses), and rewriting one set's contents in place
    between calls, every call returns exactly what a fresh session computes
    for the parameters it was given."""
    from sheaf_b200.runtime import Session

    cfg = CFGS["tiny"]
    la, x, y = models.gpt_inputs(cfg, seed_params=0)
    lb, _, _ = models.gpt_inputs(cfg, seed_params=5)
    la = [odt.round_bf16(l) for l in la]
    lb = [odt.round_bf16(l) for l in lb]
    lc = [odt.round_bf16(l * 0.5) for l in la]  # set A rewritten in place

    def fresh(leaves):
        (out,) = run_vag(cfg, "bf16", leaves, x, y)
        return out

    ref = {"a": fresh(la), "b": fresh(lb), "c": fresh(lc)}
    s = Session(0)
    s.create_gpt_vag("gpt", n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd, block_size=cfg.block_size,
                     vocab_size=cfg.vocab_size, batch=cfg.batch, seq=cfg.seq, elem=BF16)
    ba = [s.upload(l, BF16) for l in la]
    bb = [s.upload(l, BF16) for l in lb]
    ids = [s.upload(x, F32), s.upload(y, F32)]
    rewritten = False
    for which in ("a", "b", "a", "a", "b", "c", "c", "b"):
        if which == "c" and not rewritten:  # same buffers (addresses), new contents
            for buf, l in zip(ba, lc):
                buf.write(odt.f32_to_bf16_bits(l))
            rewritten = True
        bufs = (bb if which == "b" else ba) + ids
        got = [o.to_host() for o in s.call("gpt.value_and_grad", bufs)]
        for g, r in zip(got, ref[which]):
            assert np.array_equal(g, r), which


def test_vag_rejects_bad_inputs(cuda):
    from sheaf_b200.runtime import SheafB200Error, Session

    cfg = CFGS["tiny"]
    s = Session(0)
    s.create_gpt_vag("gpt", n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd, block_size=cfg.block_size,
                     vocab_size=cfg.vocab_size, batch=cfg.batch, seq=cfg.seq, elem=BF16)
    leaves, x, y = models.gpt_inputs(cfg)
    bufs = [s.upload(l, BF16) for l in leaves] + [s.upload(x, F32)]
    with pytest.raises(SheafB200Error) as e:
        s.call("gpt.value_and_grad", bufs)
    assert e.value.code == 3
    with pytest.raises(SheafB200Error) as e:
        s.call("gpt.forward", bufs)
    assert e.value.code == 5
    with pytest.raises(SheafB200Error):
        s.call("nope.value_and_grad", bufs)
