"""The multi-process host logic of ``bench.py`` on CPU: two ``gloo`` ranks.

Under torchrun every rank times its own batch and rank 0 reports the slowest
rank's time (max) and the summed work; tensor-parallel ranks share the NCCL
unique id that rank 0 makes.  These helpers run here on the gloo backend,
as they run on NCCL on the GPU box.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import sys
import traceback
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _rank(rank: int, world: int, port: int, queue) -> None:
    try:
        import datetime

        import torch.distributed as dist

        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        import bench

        slowest = bench.rank_reduce(10.0 * (rank + 1), "max")
        total = bench.rank_reduce(float(rank + 1), "sum")
        shared = bench.share_from_rank0(lambda: bytes(range(rank, rank + 8)))
        dist.barrier()
        dist.destroy_process_group()
        queue.put((rank, slowest, total, shared, None))
    except Exception:
        queue.put((rank, None, None, None, traceback.format_exc()))


def test_rank_aggregation_and_id_broadcast_over_gloo():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = 29600 + os.getpid() % 300
    procs = [ctx.Process(target=_rank, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        results = {}
        for _ in procs:
            rank, slowest, total, shared, err = queue.get(timeout=120)
            assert err is None, err
            results[rank] = (slowest, total, shared)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    for rank in (0, 1):
        slowest, total, shared = results[rank]
        assert slowest == 20.0  # the slower rank's time, on every rank
        assert total == 3.0  # work summed over ranks
        assert shared == bytes(range(0, 8))  # rank 0's id everywhere


def test_helpers_without_a_process_group():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.rank_reduce(5.0, "max") == 5.0
    assert bench.share_from_rank0(lambda: b"x") == b"x"
