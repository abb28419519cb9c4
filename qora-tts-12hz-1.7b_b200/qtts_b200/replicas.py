"""Independent-utterance sharding across the GPUs of one box (benchmark
config 5: 512 utterances, 64 per GPU, no collective on the data path).

Each rank owns a contiguous block of utterance ids and a full model replica
on its own GPU.  Two launch styles share the sharding:

* ``run_replicas``: one spawned worker process per GPU, results and errors
  returned to the parent over a queue.  A worker that raises or dies is
  reported with its rank; the other workers finish and report normally.
* torchrun / ``torch.distributed`` (bench.py): the process group is used only
  for the start barrier and for taking the max of the per-rank device times
  (``max_over_ranks``), never for model data.
"""
from __future__ import annotations

import multiprocessing as mp
import queue
import time
import traceback
from typing import Any, Callable


def shard_bounds(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous block [lo, hi) of `total` ids owned by `rank`."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    per = (total + world - 1) // world
    lo = min(total, rank * per)
    return lo, min(total, lo + per)


def _worker(rank: int, world: int, fn: Callable, payload: Any, q) -> None:
    try:
        q.put((rank, "ok", fn(rank, world, payload)))
    except BaseException as e:  # report, never hang the parent
        q.put((rank, "error", f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))


def run_replicas(world: int, fn: Callable, payload: Any = None, timeout: float = 600.0) -> dict:
    """Run fn(rank, world, payload) in `world` spawned processes.

    Returns {rank: ("ok", result) | ("error", message) | ("lost", exitcode)}.
    fn must be importable (module-level) so that `spawn` can pickle it.
    """
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, fn, payload, q), daemon=True) for r in range(world)]
    for p in procs:
        p.start()
    out: dict = {}
    deadline = time.time() + timeout
    while len(out) < world and time.time() < deadline:
        try:
            rank, status, val = q.get(timeout=0.2)
            out[rank] = (status, val)
        except queue.Empty:
            for r, p in enumerate(procs):  # a worker that died without reporting
                if r not in out and not p.is_alive() and p.exitcode not in (None, 0):
                    out[r] = ("lost", p.exitcode)
    for r, p in enumerate(procs):
        p.join(timeout=max(0.0, deadline - time.time()))
        if p.is_alive():
            p.terminate()
            p.join(5)
            out.setdefault(r, ("lost", "timeout"))
        elif r not in out:
            out[r] = ("lost", p.exitcode)
    return out


def max_over_ranks(value: float) -> float:
    """Max of a per-rank float over the default process group (gloo or nccl)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
