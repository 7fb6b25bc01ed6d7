"""Data-parallel value_and_grad on two GPUs against the oracle.

Each rank runs the fused nanoGPT step on its own half of the batch with the
gradient buckets all-reduced (ncclAvg) over NVLink inside the step; every
rank must return the loss and gradients of the whole batch (the mean over
tokens of equal-sized shards is the mean of the shard means). The eager
first call, the captured second and a replayed third must agree bitwise.
Needs two GPUs; skipped otherwise.
"""
import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import dtype as odt
from oracle import models
from tests.parity import TOL_BF16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu

BF16 = 0x22000010
F32 = 0x21000020
WORLD = 2
FULL = models.GPTConfig(n_layer=2, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=4, seq=64)
# the nanoGPT-char model (6L/6H/384, T=256) at 4 sequences: per-layer
# buckets all-reduced while the side-stream weight-gradient GEMMs run
NANO = models.GPTConfig(batch=4)
CONFIGS = {"tiny": FULL, "nanogpt": NANO}


def _worker(rank, world, uid, kind, q, cfg_name="tiny"):
    try:
        import torch

        from sheaf_b200.runtime import Session

        torch.cuda.set_device(rank)
        c = CONFIGS[cfg_name]
        shard = c.batch // world
        elem = BF16 if kind == "bf16" else F32
        s = Session(rank)
        s.join_group(uid, rank, world)
        s.create_gpt_vag("gpt", n_layer=c.n_layer, n_head=c.n_head, n_embd=c.n_embd, block_size=c.block_size,
                         vocab_size=c.vocab_size, batch=shard, seq=c.seq, elem=elem)
        leaves, x, y = models.gpt_inputs(c)
        rows = slice(rank * shard, (rank + 1) * shard)
        ins = [s.upload(a, elem) for a in leaves] + [s.upload(x[rows], F32), s.upload(y[rows], F32)]
        runs = []
        for _ in range(3):  # eager, capture, replay
            runs.append([o.to_host() for o in s.call("gpt.value_and_grad", ins)])
        s.synchronize()
        s.close()
        q.put((rank, runs, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


def _spawn(target, args_of_rank):
    """Runs one process per rank; returns {rank: result}, failing on any error."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=args_of_rank(r) + (q,)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(WORLD):
        rank, res, err = q.get(timeout=600)
        assert err is None, f"rank {rank}: {err}"
        results[rank] = res
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    return results


@pytest.mark.parametrize("kind,cfg_name", [("bf16", "tiny"), ("f32", "tiny"), ("bf16", "nanogpt")])
def test_dp_value_and_grad_matches_full_batch(kind, cfg_name, cuda):
    import torch

    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    from sheaf_b200.runtime import Session

    uid = Session.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, uid, kind, q, cfg_name)) for r in range(WORLD)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(WORLD):
        rank, runs, err = q.get(timeout=300)
        assert err is None, f"rank {rank}: {err}"
        results[rank] = runs
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0
    c = CONFIGS[cfg_name]
    leaves, x, y = models.gpt_inputs(c)
    bf = kind == "bf16"
    if bf:
        leaves = [odt.round_bf16(a) for a in leaves]
    ref_loss, ref_grads = models.gpt_value_and_grad(leaves, x, y, c, dtype=np.float64)
    tol = TOL_BF16 if bf else TOL_F32
    for rank, runs in results.items():
        for r in runs[1:]:
            for a, b in zip(runs[0], r):
                assert np.array_equal(a, b), f"rank {rank}: replay differs"
        out = runs[-1]
        assert abs(float(out[0]) - ref_loss) <= tol * abs(ref_loss), (rank, float(out[0]), ref_loss)
        for i, (g, e) in enumerate(zip(out[1:], ref_grads)):
            assert_close(g, e, tol, f"rank {rank} grad {i}")
    # both ranks hold the same averaged gradients
    for a, b in zip(results[0][-1], results[1][-1]):
        assert np.array_equal(a, b)


def _front_door_worker(rank, world, uid, rtol, q):
    """Loads the nanoGPT value_and_grad text on a session of the group and
    calls it twice on this rank's shard; `rtol` (if given) overrides this
    rank's first-call tolerance."""
    try:
        import os

        import torch

        from oracle import hlo_emit
        from sheaf_b200.runtime import Session

        if rtol is not None:
            os.environ["SHEAF_B200_VERIFY_RTOL"] = rtol
        torch.cuda.set_device(rank)
        c = FULL
        shard = c.batch // world
        shard_cfg = models.GPTConfig(n_layer=c.n_layer, n_head=c.n_head, n_embd=c.n_embd, block_size=c.block_size,
                                     vocab_size=c.vocab_size, batch=shard, seq=c.seq)
        s = Session(rank)
        s.join_group(uid, rank, world)
        name = s.load_stablehlo(hlo_emit.gpt_vag_module(shard_cfg, "bf16"))
        leaves, x, y = models.gpt_inputs(c)
        rows = slice(rank * shard, (rank + 1) * shard)
        ins = [s.upload(odt.round_bf16(a), BF16) for a in leaves] + [s.upload(x[rows], F32),
                                                                      s.upload(y[rows], F32)]
        runs = [[o.to_host() for o in s.call(f"{name}.value_and_grad", ins)] for _ in range(2)]
        note = s.describe(name)
        s.synchronize()
        s.close()
        q.put((rank, (note, runs), None))
    except Exception as e:
        q.put((rank, None, repr(e)))


@pytest.mark.parametrize("rank1_rtol", [None, "1e-12"])
def test_front_door_group_takes_one_plan(rank1_rtol, cuda):
    """A StableHLO value_and_grad loaded on the sessions of a data-parallel
    group: all ranks take the same plan, decided together on the first call.
    With rank 1's check made to reject (a tolerance below any real
    deviation), rank 0 must fall back with it: both run the generic executor
    with the outputs averaged. Either way every rank returns the full
    batch's loss and gradients."""
    import torch

    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    from sheaf_b200.runtime import Session

    uid = Session.nccl_unique_id()
    res = _spawn(_front_door_worker, lambda r: (r, WORLD, uid, rank1_rtol if r == 1 else None))
    fused = rank1_rtol is None
    for rank, (note, runs) in res.items():
        want = "fused nanoGPT plan, data-parallel" if fused else "generic executor, data-parallel outputs averaged"
        assert want in note, (rank, note)
    leaves, x, y = models.gpt_inputs(FULL)
    leaves = [odt.round_bf16(a) for a in leaves]
    ref_loss, ref_grads = models.gpt_value_and_grad(leaves, x, y, FULL, dtype=np.float64)
    if not fused:
        # the generic executor computes each rank's module op by op in bf16;
        # the group averages those results
        from oracle import hlo_emit, hlo_eval

        shard = FULL.batch // WORLD
        scfg = models.GPTConfig(n_layer=FULL.n_layer, n_head=FULL.n_head, n_embd=FULL.n_embd,
                                block_size=FULL.block_size, vocab_size=FULL.vocab_size, batch=shard, seq=FULL.seq)
        text = hlo_emit.gpt_vag_module(scfg, "bf16")
        per = [hlo_eval.evaluate(text, leaves + [x[r * shard:(r + 1) * shard], y[r * shard:(r + 1) * shard]])
               for r in range(WORLD)]
        avg = [sum(p[i] for p in per) / WORLD for i in range(len(per[0]))]
        ref_loss, ref_grads = float(avg[0]), avg[1:]
    for rank, (note, runs) in res.items():
        for out in runs:
            assert abs(float(out[0]) - ref_loss) <= TOL_BF16 * abs(ref_loss), (rank, float(out[0]), ref_loss)
            for i, (g, e) in enumerate(zip(out[1:], ref_grads)):
                assert_close(g, e, TOL_BF16, f"rank {rank} grad {i}")
    for a, b in zip(res[0][1][-1], res[1][1][-1]):
        assert np.array_equal(a, b)
