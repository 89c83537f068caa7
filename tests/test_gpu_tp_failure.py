"""Failure detection on the tensor-parallel path, with every failure made on
the host and no collective left in flight:

  * a TP rank that never joins: ``clef_create`` of the rank that did gives up
    after ``tp_timeout`` with CLEF_ENCCL (the half-made NCCL communicator is
    aborted before anything of it reaches a stream) -- one GPU;
  * a TP rank that fails between forwards: through ``TpHeartbeat`` its peer
    raises before launching its next forward, and both ranks close cleanly --
    two GPUs, NVLS off.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import subprocess
import sys
import textwrap
import time
import traceback
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def test_create_fails_when_a_tp_rank_never_joins():
    import torch

    if torch.cuda.device_count() < 1:
        pytest.skip("needs a GPU")
    code = textwrap.dedent(
        """
        import ctypes, sys, time
        sys.path[:0] = [{root!r}, {tests!r}]
        from deciax_b200 import _lib
        from deciax_b200.model import ClefCudaModel
        from test_gpu_tp import _config
        lib = _lib.load()
        nid = ctypes.create_string_buffer(_lib.NCCL_ID_BYTES)
        _lib.check(lib.clef_nccl_unique_id(nid))
        config, head = _config("full")
        t0 = time.monotonic()
        try:
            ClefCudaModel(config, head, dtype="fp32", device=0, tp_rank=0, tp_size=2, nccl_id=nid.raw,
                          max_seq_len=256, tp_timeout=2.0)
        except _lib.ClefError as e:
            print("ERR", time.monotonic() - t0, e)
            sys.exit(0)
        print("created without the peer")
        sys.exit(1)
        """
    ).format(root=str(ROOT), tests=str(ROOT / "tests"))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=240, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    line = [x for x in r.stdout.splitlines() if x.startswith("ERR")][0]
    elapsed = float(line.split()[1])
    assert 2.0 <= elapsed < 60.0, line
    assert f"clef status {3}" in line and "communicator of 2 ranks not formed" in line, line


def _worker(rank: int, world: int, nccl_id: bytes, port: int, queue) -> None:
    try:
        sys.path[:0] = [str(ROOT), str(ROOT / "tests")]
        from gpu_helpers import round_tree
        from test_gpu_tp import _config

        from deciax_b200.model import ClefCudaModel
        from deciax_b200.synthetic import BatchSpec, synthetic_batch, synthetic_weights
        from deciax_b200.tp_heartbeat import TpHeartbeat, TpRankMissing, store_for

        store = store_for(rank, world, port=port, timeout=60)
        hb = TpHeartbeat(store, rank, world, timeout=60.0)
        config, head = _config("full")
        top, layers, hp = synthetic_weights(config, head, seed=5, embed_std=1.0)
        top, layers, hp = round_tree(top, "bf16"), round_tree(layers, "bf16"), round_tree(hp, "bf16")
        model = ClefCudaModel.from_arrays(config, head, top, layers, hp, dtype="bf16", device=rank, tp_rank=rank,
                                          tp_size=world, nccl_id=nccl_id, max_seq_len=256, tp_timeout=60.0,
                                          heartbeat=hb)
        arrays = synthetic_batch(BatchSpec(states=2, seq=128, questions=2, options_per_question=3,
                                           lengths=(128, 70), row_bucket=2), config.vocab_size, seed=6)
        done, outcome = 0, "done"
        for step in range(4):
            if rank == 1 and step == 2:  # the injected failure, between forwards
                try:
                    raise RuntimeError("injected")
                except RuntimeError as e:
                    model.report_failure(e)
                    outcome = "injected"
                    break
            try:
                model.forward(arrays)
            except TpRankMissing as e:
                outcome = f"missing: {e}"
                break
            done += 1
        model.close()  # no collective in flight on either rank
        queue.put((rank, done, outcome, None))
        time.sleep(1.0)  # rank 0 hosts the store
    except Exception:
        queue.put((rank, -1, "", traceback.format_exc()))


def test_peer_failure_between_forwards_stops_the_other_rank(monkeypatch):
    import ctypes

    import torch

    from deciax_b200 import _lib

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    lib = _lib.load()
    nid = ctypes.create_string_buffer(_lib.NCCL_ID_BYTES)
    _lib.check(lib.clef_nccl_unique_id(nid))
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")  # inherited by the spawned ranks
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = 29800 + os.getpid() % 97
    procs = [ctx.Process(target=_worker, args=(r, 2, nid.raw, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in procs:
            rank, done, outcome, err = queue.get(timeout=600)
            assert err is None, err
            got[rank] = (done, outcome)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.terminate()
    assert got[1] == (2, "injected"), got
    assert got[0][0] == 2 and got[0][1].startswith("missing: tensor-parallel step 2"), got
    assert "rank 1 failed: RuntimeError: injected" in got[0][1], got
