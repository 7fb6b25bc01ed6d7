"""Host-side data-parallel plumbing, two gloo ranks on the CPU (no GPU).

bench.py's rank set-up, the broadcast of the 128-byte NCCL group id from rank
0, max-over-ranks timing and barriers; and failure detection: a rank that dies
before a collective turns into an error on the survivor within the process
group's timeout instead of a hang.
"""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    sys.path.insert(0, str(ROOT))
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    import bench

    try:
        if mode == "leave_between_steps":
            from torch.distributed.distributed_c10d import _get_default_store

            import torch

            from sheaf_b200.runtime import announce_departure, departed_ranks

            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=20))
            store = _get_default_store()
            steps = 0
            for step in range(3):
                t = torch.ones(4)
                dist.all_reduce(t)  # the step's collective
                steps += 1
                if rank == 1 and step == 0:
                    announce_departure(store, rank)  # before the boundary barrier
                dist.barrier()  # step boundary
                gone = departed_ranks(store, world)
                if gone:
                    # survivors end the group here (Session.leave_group(abort=True)
                    # on a GPU); nobody enqueues another collective
                    q.put((rank, (steps, gone)))
                    return
            q.put((rank, (steps, [])))
            return
        if mode == "dead_rank":
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=5))
            if rank == 1:
                os._exit(0)  # leaves without joining the collective
            try:
                bench.allmax(1.0, world)
                q.put((rank, "no error"))
            except Exception as e:  # noqa: BLE001
                q.put((rank, "error: " + type(e).__name__))
            return
        w, r, local = bench.dist_setup()
        assert (w, r, local) == (world, rank, rank)
        obj = [bytes(range(128)) if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        t = bench.allmax(float(rank + 1) * 0.5, world)
        bench.barrier(world)
        q.put((rank, (obj[0] == bytes(range(128)), t)))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, "exception: " + repr(e)))


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(2 if mode != "dead_rank" else 1):  # the departing rank reports too
        r, v = q.get(timeout=120)
        results[r] = v
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


def test_group_id_broadcast_and_max_over_ranks():
    res = _run("ok")
    assert res[0] == (True, 1.0) and res[1] == (True, 1.0)


def test_dead_rank_becomes_an_error_not_a_hang():
    res = _run("dead_rank")
    assert res[0].startswith("error"), res


def test_rank_leaves_between_steps_and_survivors_learn_before_the_next_step():
    """A rank that leaves announces it in the store before the step-boundary
    barrier; every rank sees the departure after that barrier, before it
    would enqueue the next step's collective (so no collective waits on the
    missing peer)."""
    res = _run("leave_between_steps")
    assert res[0] == (1, [1]) and res[1] == (1, [1]), res
