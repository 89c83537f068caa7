"""Failure detection between tensor-parallel ranks, on the host, without a GPU.

``TpHeartbeat`` makes each rank check in before every forward, so a rank that
fails or stops between forwards is noticed before anything is launched:
  * a rank that raises posts the reason and its peers raise it at once;
  * a rank that silently stops leaves its peers to raise after the deadline;
  * a rank that arrives after its peers gave up raises too (verdicts are
    written once).
Ranks are threads on a ``HashStore`` here, and spawned processes on a
``TCPStore`` (the store the GPU ranks use) in the last tests.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import sys
import threading
import time
import traceback
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from deciax_b200.tp_heartbeat import TpHeartbeat, TpRankMissing  # noqa: E402


def _store():
    import torch.distributed as dist

    return dist.HashStore()


def _run_threads(fns):
    """Run one function per rank in threads; return {rank: result or exception}."""
    out: dict[int, object] = {}

    def wrap(r, fn):
        try:
            out[r] = fn()
        except BaseException as e:  # collected for the assertions
            out[r] = e

    ts = [threading.Thread(target=wrap, args=(r, fn)) for r, fn in enumerate(fns)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(timeout=60)
    assert not any(t.is_alive() for t in ts)
    return out


def test_all_ranks_pass_many_steps_and_old_keys_are_pruned():
    store = _store()
    hbs = [TpHeartbeat(store, r, 3, timeout=10) for r in range(3)]

    def rank(r):
        for _ in range(25):
            hbs[r].arrive()
        return hbs[r].step

    out = _run_threads([lambda r=r: rank(r) for r in range(3)])
    assert out == {0: 25, 1: 25, 2: 25}
    assert not store.check(["clef/tp/0/go"])  # rank 0 deleted the steps every rank is past
    assert store.check(["clef/tp/24/go"])


def test_a_failing_rank_stops_its_peers_at_once():
    store = _store()
    hbs = [TpHeartbeat(store, r, 2, timeout=30) for r in range(2)]

    def rank0():
        for _ in range(5):
            hbs[0].arrive()

    def rank1():
        for i in range(5):
            if i == 3:
                try:
                    raise ValueError("bad batch")
                except ValueError as e:
                    hbs[1].fail(f"{type(e).__name__}: {e}")
                    raise
            hbs[1].arrive()

    t0 = time.monotonic()
    out = _run_threads([rank0, rank1])
    assert time.monotonic() - t0 < 10  # far below the 30 s deadline
    assert isinstance(out[1], ValueError)
    assert isinstance(out[0], TpRankMissing)
    assert "step 3" in str(out[0]) and "rank 1 failed: ValueError: bad batch" in str(out[0])
    assert hbs[0].step == 3


def test_a_silent_rank_is_reported_after_the_deadline():
    store = _store()
    hbs = [TpHeartbeat(store, r, 2, timeout=0.4) for r in range(2)]

    def rank0():
        for _ in range(4):
            hbs[0].arrive()

    def rank1():
        for _ in range(2):  # then stops without a word
            hbs[1].arrive()

    t0 = time.monotonic()
    out = _run_threads([rank0, rank1])
    assert 0.4 <= time.monotonic() - t0 < 10
    assert out[1] is None
    assert isinstance(out[0], TpRankMissing) and "1/2 ranks arrived within 0.4 s" in str(out[0])


def test_a_late_rank_does_not_revive_a_failed_step():
    store = _store()
    a, b = TpHeartbeat(store, 0, 2, timeout=0.2), TpHeartbeat(store, 1, 2, timeout=5)
    with pytest.raises(TpRankMissing):
        a.arrive()
    with pytest.raises(TpRankMissing, match="1/2 ranks arrived"):
        b.arrive()  # completes the count, but the step's verdict already stands


def test_prefixes_keep_models_apart_and_arguments_are_checked():
    store = _store()
    x0, x1 = TpHeartbeat(store, 0, 2, prefix="m1"), TpHeartbeat(store, 1, 2, prefix="m1")
    y0 = TpHeartbeat(store, 0, 2, prefix="m2", timeout=0.2)
    out = _run_threads([x0.arrive, x1.arrive])
    assert out == {0: None, 1: None}
    with pytest.raises(TpRankMissing):
        y0.arrive()
    with pytest.raises(ValueError):
        TpHeartbeat(store, 2, 2)
    with pytest.raises(ValueError):
        TpHeartbeat(store, 0, 2, timeout=0)


def _proc(rank: int, world: int, port: int, mode: str, queue) -> None:
    try:
        sys.path.insert(0, str(ROOT))
        from deciax_b200.tp_heartbeat import TpHeartbeat, TpRankMissing, store_for

        store = store_for(rank, world, port=port, timeout=30)
        hb = TpHeartbeat(store, rank, world, timeout=1.0 if mode == "silent" else 30.0)
        steps = 0
        try:
            for i in range(6):
                if rank == world - 1 and i == 4:
                    if mode == "raise":
                        hb.fail("RuntimeError: injected")
                        queue.put((rank, steps, "injected"))
                        return
                    queue.put((rank, steps, "left"))  # silent: leaves without a word
                    return
                hb.arrive()
                steps += 1
            queue.put((rank, steps, "done"))
        except TpRankMissing as e:
            queue.put((rank, steps, f"missing: {e}"))
        time.sleep(0.5)  # rank 0 hosts the store: keep it up while peers read it
    except Exception:
        queue.put((rank, -1, traceback.format_exc()))


@pytest.mark.parametrize("mode", ["raise", "silent"])
def test_tcp_store_ranks_in_processes(mode):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = 29900 + os.getpid() % 97 + (0 if mode == "raise" else 97)
    procs = [ctx.Process(target=_proc, args=(r, 2, port, mode, queue)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = {}
        for _ in procs:
            rank, steps, what = queue.get(timeout=120)
            got[rank] = (steps, what)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    assert got[1][0] == 4, got
    assert got[0][0] == 4 and got[0][1].startswith("missing: tensor-parallel step 4"), got
    if mode == "raise":
        assert "rank 1 failed: RuntimeError: injected" in got[0][1]
    else:
        assert "1/2 ranks arrived within 1 s" in got[0][1]
