"""``ClefEngine``: answers a batch of states against one question schema.

Mirrors ``src/deciax/runtime/clef.py:18-40`` (same constructor argument,
``decide_batch`` signature, results in input order, the same ``ValueError``
for ``head_max_len``) with three changes to how the work is scheduled; none
changes a record's answer, because a record's logits do not depend on the
other rows or the padding of its batch:

* the schema is tokenised once per call and the states as one tokenizer batch
  (``SchemaPrompt.encode_states``) instead of one full ``encode`` per state;
* records are grouped by length into batches whose padded size
  (rows x padded length) stays within ``max_batch_tokens``, instead of fixed
  pairs in input order; a batch is padded only to its longest record rounded
  up to 128 tokens (not to a power-of-two bucket) and has no padded rows; the
  cut points minimise a cost model of the padded work (``plan_batches``);
* batches go to every replica at once (data parallelism: one model per GPU,
  each with full weights, no collective), one host thread per replica.  The
  library releases the GIL for the whole forward, so replicas run
  concurrently; while a replica computes, its thread's next batch is already
  collated by a helper thread.

A replica is anything with ``forward(arrays) -> [b, o] logits``, ``name``,
``tokenizer``, ``pad_token_id`` and ``max_token_budget`` (``ClefCudaModel``).
Each replica serves one batch at a time (``forward`` is not re-entrant per
handle); ``decide_batch`` calls may come from several threads.
"""

from __future__ import annotations

import queue
import threading
import time
from collections.abc import Mapping, Sequence
from concurrent.futures import ThreadPoolExecutor
from typing import Any

import numpy as np

from deciax_b200.clef_input import ROW_BUCKETS, Record, SchemaPrompt, collate, decode

DEFAULT_BATCH_TOKENS = 65536
SEQ_ALIGN = 128
# Cost model of one forward, in token-equivalents of linear-layer work (the
# cfg2 clef-flash shape on one B200, where a token of padded work costs
# ~16 us): a fixed cost per batch (launches, head, host collate/decode), a
# floor below which the GPU is not filled, and causal attention's growth with
# the padded length (per token ~ seq / ATTN_TOKENS of the linear work).
BATCH_COST_TOKENS = 256
MIN_BATCH_TOKENS = 4096
ATTN_TOKENS = 24000


def batch_cost(rows: int, seq: int) -> float:
    """Modelled cost of one batch of ``rows`` records padded to ``seq``."""
    padded = rows * seq
    return BATCH_COST_TOKENS + max(padded, MIN_BATCH_TOKENS) + padded * seq / ATTN_TOKENS


def plan_batches(lengths: Sequence[int], max_batch_tokens: int = DEFAULT_BATCH_TOKENS, max_rows: int = ROW_BUCKETS[-1],
                 seq_align: int = SEQ_ALIGN) -> list[tuple[list[int], int]]:
    """Group record indices into (indices, padded length) batches, longest first.

    Records sorted longest first are cut into contiguous runs (with sorted
    lengths the padding-optimal groups are contiguous); a run's padded length
    is its first record rounded up to ``seq_align``, it holds at most
    ``max_rows`` records and ``max_batch_tokens`` padded tokens (a record
    longer than the budget runs alone).  The cut points minimise the summed
    ``batch_cost`` by dynamic programming over (run start, run length), so
    padding is traded against the per-batch cost instead of bounded by a fixed
    length ratio.  The plan depends only on ``lengths``, so tensor-parallel
    ranks that plan the same records run the same batches.
    """
    order = sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))
    n = len(order)
    best = [0.0] + [float("inf")] * n  # best[j]: cost of the first j records
    cut = [0] * (n + 1)
    for i in range(n):  # a run starting at sorted position i
        if best[i] == float("inf"):
            continue
        seq = -(-lengths[order[i]] // seq_align) * seq_align
        cap = max(1, min(max_rows, max_batch_tokens // seq))
        for rows in range(1, min(cap, n - i) + 1):
            c = best[i] + batch_cost(rows, seq)
            if c < best[i + rows]:
                best[i + rows] = c
                cut[i + rows] = i
    batches: list[tuple[list[int], int]] = []
    j = n
    while j > 0:
        i = cut[j]
        batches.append((order[i:j], -(-lengths[order[i]] // seq_align) * seq_align))
        j = i
    return batches[::-1]


class ClefEngine:
    def __init__(self, model: Any, *, replicas: Sequence[Any] | None = None,
                 max_batch_tokens: int = DEFAULT_BATCH_TOKENS, auto_warmup: bool = True) -> None:
        """``auto_warmup=False`` skips the workspace reservation before the
        first forward: the workspace then grows with each new batch shape (the
        cold-start behaviour, for callers that bound device memory themselves
        or that call ``warmup`` at a time of their choosing)."""
        self.model = model
        self.replicas = list(replicas) if replicas else [model]
        if max_batch_tokens < 1:
            raise ValueError("max_batch_tokens must be positive")
        self.max_batch_tokens = max_batch_tokens
        self._locks = [threading.Lock() for _ in self.replicas]
        self._warm = not auto_warmup
        self._warm_lock = threading.Lock()

    def warmup(self) -> None:
        """Reserve every replica's workspace for the largest batch this engine
        forms (``ClefCudaModel.warmup``), so no request allocates device
        memory.  ``decide_batch`` / ``decide_records`` call it once before
        their first forward, so the reference server's warm-up request
        (serve/app.py:385-406, one tiny ``decide``) reaches it."""
        with self._warm_lock:
            if self._warm:
                return
            for replica, lock in zip(self.replicas, self._locks):
                if hasattr(replica, "warmup"):
                    with lock:
                        replica.warmup(max_batch_tokens=self.max_batch_tokens, max_rows=ROW_BUCKETS[-1])
            self._warm = True

    def encode(self, states: Sequence[Any], questions: Mapping[Any, Mapping[str, Any]], max_len: int | None) -> list[Record]:
        model = self.model
        prompt = SchemaPrompt(model.tokenizer, questions)
        return prompt.encode_states(list(states), model.max_token_budget if max_len is None else max_len)

    def decide_batch(self, states: Sequence[Any], questions: Mapping[Any, Mapping[str, Any]], *, max_len: int | None = None,
                     head_max_len: int | None = None) -> list[dict[str, Any]]:
        if head_max_len is not None:
            raise ValueError("Clef has one joint token budget; head_max_len is unsupported")
        return self.decide_records(self.encode(states, questions, max_len), questions)

    def decide_records(self, records: Sequence[Record], questions: Mapping[Any, Mapping[str, Any]],
                       timings: list | None = None) -> list[dict[str, Any]]:
        """Answers for already-encoded records, in input order.  With
        ``timings``, each batch appends (rows, sequence bucket, seconds of its
        forward, host arrays in and logits out)."""
        if not records:
            return []
        self.warmup()
        batches = plan_batches([len(r.ids) for r in records], self.max_batch_tokens)
        results: list[dict[str, Any] | None] = [None] * len(records)
        work: queue.Queue[tuple[list[int], int]] = queue.Queue()
        for b in batches:
            work.put(b)
        errors: list[BaseException] = []
        pad_id, name = self.model.pad_token_id, self.model.name

        def prepare(batch: tuple[list[int], int]) -> tuple[list[int], dict[str, np.ndarray]]:
            idx, seq = batch
            return idx, collate([records[i] for i in idx], pad_id, rows=len(idx), seq_len=seq)

        def serve(k: int) -> None:
            replica, lock = self.replicas[k], self._locks[k]
            with ThreadPoolExecutor(1) as helper:
                pending = None
                while not errors:
                    if pending is None:
                        try:
                            pending = helper.submit(prepare, work.get_nowait())
                        except queue.Empty:
                            return
                    idx, arrays = pending.result()
                    try:
                        pending = helper.submit(prepare, work.get_nowait())
                    except queue.Empty:
                        pending = None
                    with lock:
                        t0 = time.perf_counter()
                        logits = np.asarray(replica.forward(arrays), np.float32)
                        if timings is not None:
                            timings.append((len(idx), arrays["input_ids"].shape[1], time.perf_counter() - t0))
                    for row, i in enumerate(idx):
                        results[i] = decode(records[i], logits[row], questions, name)

        def guarded(k: int) -> None:
            try:
                serve(k)
            except BaseException as e:  # re-raised in the caller's thread
                errors.append(e)

        if len(self.replicas) == 1 or len(batches) == 1:
            serve(0)
        else:
            threads = [threading.Thread(target=guarded, args=(k,), daemon=True) for k in range(len(self.replicas))]
            for t in threads:
                t.start()
            for t in threads:
                t.join()
            if errors:
                raise errors[0]
        return results  # type: ignore[return-value]
