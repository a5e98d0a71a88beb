"""Host logic of the multi-GPU benchmark, run as two gloo ranks on CPU.

The op itself has no collective: (sequence, head) pairs are independent and
every rank runs its own shard.  What is shared is the harness: the shard
split, the barrier around the timed region, the max-over-ranks of the device
time, and the reference arm that only rank 0 runs.
"""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    import bench

    out = {}
    out["c5"] = bench.shard(bench.CONFIGS["c5"], world, rank)
    out["ns"] = bench.shard(bench.CONFIGS["ns"], world, rank)
    bench.barrier(world)
    out["max"] = bench.max_over_ranks(float(10 * (rank + 1)), world)

    class Args:
        steps, warmup, gpus = 1, 0, world

    # the reference arm: every rank other than 0 returns at once without work
    out["ref_rc"] = bench.run_reference_arm(Args, "ns", out["ns"], world, rank) if rank != 0 else 0
    bench.barrier(world)
    q.put((rank, out))
    dist.destroy_process_group()


def test_two_rank_harness():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in (0, 1):
        r = results[rank]
        # strong scaling (c5): heads split evenly, weak scaling (ns): full shard per rank
        assert r["c5"]["H"] == 32 and r["c5"]["HK"] == 32
        assert r["ns"]["H"] == 32 and r["ns"]["B"] == 4
        assert r["max"] == 20.0
        assert r["ref_rc"] == 0
