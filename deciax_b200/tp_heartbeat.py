"""Host-side arrival check for the tensor-parallel ranks of one Clef model.

Every TP rank runs its own process and its own ``ClefCudaModel``; each
forward carries NCCL collectives that all ranks must join.  A rank that fails
or stops between forwards would leave the others waiting inside a collective.
``TpHeartbeat`` catches that on the host, before any kernel is launched: each
rank checks in on a shared key-value store (a ``torch.distributed`` store) at
the start of every forward and waits, with a deadline, for the others.  A rank
whose own step fails posts the reason, so the others stop at once with it
instead of waiting out the deadline.

The reference serves one process over all devices (JAX sharding,
models/qwen3_5/pallas.py:84-90) and has no counterpart; its server maps any
failure to an HTTP 500 (serve/app.py:261-263), which ``RuntimeError`` here
matches.
"""

from __future__ import annotations

import time
from datetime import timedelta
from typing import Any

_FAILED = "failed:"


class TpRankMissing(RuntimeError):
    """Another tensor-parallel rank did not arrive (or reported a failure)."""


class TpHeartbeat:
    """Check-in of ``size`` ranks on ``store`` before each TP step.

    ``store`` needs ``add``, ``compare_set``, ``check`` and ``get`` (any
    ``torch.distributed.Store``).  Each step's verdict is written once
    (``compare_set`` on an absent key), so a rank that arrives just as another
    gives up cannot turn the failed step back into a go.  ``prefix`` keeps
    several models (or runs) on one store apart.  Steps are counted per rank,
    so every rank must call ``arrive`` once per forward, in the same order.
    """

    def __init__(self, store: Any, rank: int, size: int, *, timeout: float = 300.0, prefix: str = "clef/tp",
                 poll: float = 0.0005) -> None:
        if not 0 <= rank < size:
            raise ValueError(f"bad tensor-parallel rank {rank} of {size}")
        if timeout <= 0:
            raise ValueError("timeout must be positive")
        self.store = store
        self.rank = rank
        self.size = size
        self.timeout = timeout
        self.prefix = prefix
        self.poll = poll
        self.step = 0

    def _key(self, step: int) -> str:
        return f"{self.prefix}/{step}"

    def arrive(self) -> None:
        """Check in for the next step; return once every rank has, else raise
        ``TpRankMissing`` (a peer posted a failure, or the deadline passed)."""
        step = self.step
        key = self._key(step)
        n = self.store.add(key + "/n", 1)
        if n == self.size:
            self._verdict(step, "ok")
        deadline = time.monotonic() + self.timeout
        delay = self.poll
        while True:
            if self.store.check([key + "/go"]):
                state = self.store.get(key + "/go").decode()
                if state.startswith(_FAILED):
                    raise TpRankMissing(f"tensor-parallel step {step}: {state[len(_FAILED):]}")
                self.step = step + 1
                if self.rank == 0 and step > 0:
                    # every rank is past step - 1 once all have arrived here
                    for suffix in ("/n", "/go"):
                        self.store.delete_key(self._key(step - 1) + suffix)
                return
            if time.monotonic() > deadline:
                arrived = self.store.add(key + "/n", 0)
                # tell ranks that arrive later not to wait either
                state = self._verdict(step, f"{_FAILED}{arrived}/{self.size} ranks arrived within {self.timeout:g} s")
                if state == "ok":  # the last rank arrived in the meantime
                    continue
                raise TpRankMissing(f"tensor-parallel step {step}: {state[len(_FAILED):]}")
            time.sleep(delay)
            delay = min(delay * 2, 0.01)

    def fail(self, reason: str) -> None:
        """Post this rank's failure at its current step, so the peers waiting
        there (or arriving later) raise at once with ``reason``."""
        self._verdict(self.step, f"{_FAILED}rank {self.rank} failed: {reason}")

    def _verdict(self, step: int, value: str) -> str:
        """Write the step's verdict unless one is there; return the one that stands."""
        got = self.store.compare_set(self._key(step) + "/go", "", value)
        return got.decode() if isinstance(got, bytes) else str(got)


def store_for(rank: int, size: int, host: str = "127.0.0.1", port: int = 29511, timeout: float = 300.0):
    """A ``torch.distributed.TCPStore`` shared by ``size`` ranks (rank 0 hosts it)."""
    import torch.distributed as dist

    return dist.TCPStore(host, port, size, rank == 0, timedelta(seconds=timeout))
