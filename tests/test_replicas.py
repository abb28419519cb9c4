"""Host-side multi-GPU plumbing on CPU: utterance sharding, the replica
launcher's failure reporting, and the gloo max-over-ranks timing reduction
(world_size 2).  Failures are made on the host (a raising or exiting
worker); nothing here touches a GPU."""
import os
import socket

import pytest

from qtts_b200 import replicas as R


def test_shard_bounds_partition():
    for total, world in [(512, 8), (512, 3), (7, 4), (1, 2), (64, 1)]:
        seen = []
        for r in range(world):
            lo, hi = R.shard_bounds(total, r, world)
            seen.extend(range(lo, hi))
        assert seen == list(range(total))
    assert R.shard_bounds(512, 3, 8) == (192, 256)
    with pytest.raises(ValueError):
        R.shard_bounds(10, 2, 2)


def work_ok(rank, world, payload):
    lo, hi = R.shard_bounds(payload, rank, world)
    return sum(range(lo, hi))


def work_fail_rank1(rank, world, payload):
    if rank == 1:
        raise RuntimeError("injected failure on rank 1")
    return rank


def work_exit_rank0(rank, world, payload):
    if rank == 0:
        os._exit(3)
    return rank


def test_run_replicas_gathers():
    out = R.run_replicas(3, work_ok, 100, timeout=120)
    assert all(s == "ok" for s, _ in out.values())
    assert sum(v for _, v in out.values()) == sum(range(100))


def test_run_replicas_reports_failure_others_finish():
    out = R.run_replicas(3, work_fail_rank1, None, timeout=120)
    assert out[1][0] == "error" and "injected failure" in out[1][1]
    assert out[0] == ("ok", 0) and out[2] == ("ok", 2)


def test_run_replicas_reports_dead_worker():
    out = R.run_replicas(2, work_exit_rank0, None, timeout=120)
    assert out[0][0] == "lost"
    assert out[1] == ("ok", 1)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _gloo_rank(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        dist.barrier()
        q.put((rank, R.max_over_ranks(1.5 + rank)))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_gloo():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in ps:
        p.join(60)
    assert res == {0: 2.5, 1: 2.5}
