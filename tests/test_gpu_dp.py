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


def _worker(rank, world, uid, kind, q):
    try:
        import torch

        from sheaf_b200.runtime import Session

        torch.cuda.set_device(rank)
        c = FULL
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


@pytest.mark.parametrize("kind", ["bf16", "f32"])
def test_dp_value_and_grad_matches_full_batch(kind, cuda):
    import torch

    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    from sheaf_b200.runtime import Session

    uid = Session.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, uid, kind, q)) for r in range(WORLD)]
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
    leaves, x, y = models.gpt_inputs(FULL)
    bf = kind == "bf16"
    if bf:
        leaves = [odt.round_bf16(a) for a in leaves]
    ref_loss, ref_grads = models.gpt_value_and_grad(leaves, x, y, FULL, dtype=np.float64)
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
