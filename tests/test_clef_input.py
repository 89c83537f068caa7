"""Host side of the Clef path: ``deciax_b200.clef_input`` and ``ClefEngine``.

Pinned to ``golden/clef_input.json`` -- the reference's own ``encode``,
``collate`` and ``decode`` (``src/deciax/models/clef/input.py``) run on the
same tokenizer, states, schemas and logits (``golden/make_input_golden.py``)
-- and to the reference's tests ``tests/clef/test_input.py:17-83``, restated.
"""

from __future__ import annotations

import json
import sys
import threading
import time

import numpy as np
import pytest
from conftest import GOLDEN
from tokenizers import Tokenizer, models, pre_tokenizers

from deciax_b200 import clef_input as I
from deciax_b200.engine import ClefEngine, plan_batches

sys.path.insert(0, str(GOLDEN))
import make_input_golden  # noqa: E402

FIX = json.loads((GOLDEN / "clef_input.json").read_text())
TOK = Tokenizer.from_str(FIX["tokenizer"])
PAD = TOK.token_to_id("<|endoftext|>")


def as_plain(record: I.Record) -> dict:
    return {"ids": list(record.ids), "fields": [
        {"id": f.id, "kind": f.kind, "span": list(f.span), "option_spans": [list(s) for s in f.option_spans],
         "option_ids": list(f.option_ids)} for f in record.fields]}


@pytest.mark.parametrize("case", range(len(FIX["cases"])))
def test_matches_reference_golden(case):
    c = FIX["cases"][case]
    schema = FIX["schemas"][c["schema"]]
    records = [I.encode(TOK, s, schema, c["budget"]) for s in FIX["states"]]
    assert [as_plain(r) for r in records] == c["records"]
    # the batched path (schema tokenised once) gives the same records
    assert I.SchemaPrompt(TOK, schema).encode_states(FIX["states"], c["budget"]) == records
    arrays = I.collate(records, PAD)
    assert set(arrays) == set(c["arrays"])
    for k, v in c["arrays"].items():
        expected = np.asarray(v)
        assert arrays[k].shape == expected.shape, k
        assert arrays[k].dtype == (bool if k.endswith("mask") else np.int32), k
        np.testing.assert_array_equal(arrays[k].astype(np.int32), expected, err_msg=k)
    logits = np.asarray(c["logits"], np.float32)
    decoded = [I.decode(r, logits[i], schema, "clef") for i, r in enumerate(records)]
    assert json.loads(json.dumps(decoded)) == c["decoded"]
    if "too_small" in c:
        with pytest.raises(ValueError) as e:
            I.encode(TOK, "", schema, c["too_small"]["budget"])
        assert str(e.value) == c["too_small"]["error"]


def test_invalid_schemas_match_reference_messages():
    assert len(make_input_golden.INVALID) == len(FIX["invalid"])
    for q, expected in zip(make_input_golden.INVALID, FIX["invalid"], strict=True):
        if expected["error"] is None:
            I.validate_questions(q)
            continue
        with pytest.raises(ValueError) as e:
            I.validate_questions(q)
        assert str(e.value) == expected["error"]


def test_bad_budgets_match_reference_messages():
    values = {"0": 0, "16385": 16385, "True": True, "3.0": 3.0}
    for item in FIX["bad_budgets"]:
        with pytest.raises(ValueError) as e:
            I.encode(TOK, "", FIX["schemas"]["single"], values[item["budget"]])
        assert str(e.value) == item["error"]


# --- tests/clef/test_input.py of the reference, restated ---


@pytest.fixture
def tiny() -> Tokenizer:
    tok = Tokenizer(models.WordLevel({"[UNK]": 0, "hello": 1, "world": 2}, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    return tok


def test_record_spans_options_and_lexical_tokens(tiny):
    questions = {
        "sentiment": {"type": "choice", "criteria": {"z": "world", "a": "hello"}},
        "yes": {"type": "noul"},
        "score": {"type": "score", "criteria": ["hello", "world", "hello world"]},
    }
    records = [I.encode(tiny, s, questions, 512) for s in ("hello", "hello world " * 20)]
    arrays = I.collate(records, 0)
    assert records[0].fields[0].option_ids == ("a", "z")
    assert records[0].fields[1].option_ids == ("true", "false")
    for i, record in enumerate(records):
        j = 0
        for owner, field in enumerate(record.fields):
            assert field.span[0] < field.span[1] < len(record.ids)
            for start, end in field.option_spans:
                ls, le = arrays["lexical_spans"][i, j]
                np.testing.assert_array_equal(record.ids[start:end], arrays["lexical_ids"][i, ls:le])
                assert arrays["option_field"][i, j] == owner
                j += 1
        assert arrays["option_mask"][i].sum() == 7
        result = I.decode(record, np.zeros(8), questions, "clef")
        assert result["answers"]["yes"]["noul"] == 0.5
        assert result["answers"]["score"]["score"] == 1.0
        assert result["usage"]["input_tokens"] == len(record.ids)


def test_truncation_keeps_schema_complete(tiny):
    q = {"x": {"type": "choice", "criteria": {"a": "hello", "b": "world"}}}
    fixed = I.encode(tiny, "", q, 512)
    limit = len(fixed.ids) + 5
    actual = I.encode(tiny, "hello world " * 500, q, limit)
    assert len(actual.ids) == limit
    for a, b in zip(actual.fields, fixed.fields, strict=True):
        assert a.span == (b.span[0] + 5, b.span[1] + 5)
    with pytest.raises(ValueError, match="schema requires"):
        I.encode(tiny, "", q, len(fixed.ids) - 1)


def test_decode_rejects_nonfinite_logits(tiny):
    questions = {"yes": {"type": "noul"}}
    record = I.encode(tiny, "hello", questions, 512)
    with pytest.raises(FloatingPointError, match="non-finite"):
        I.decode(record, np.array([np.nan, 0.0]), questions, "clef")


def test_collate_rejects_more_rows_than_the_largest_bucket(tiny):
    record = I.encode(tiny, "hello", {"yes": {"type": "noul"}}, 512)
    with pytest.raises(ValueError, match="exceeds the largest bucket"):
        I.collate([record] * 65, 0)


# --- engine ---


class FakeReplica:
    """A stand-in model whose logits depend only on each row's own tokens
    (like the real forward, where padding and other rows cannot leak)."""

    name = "clef"
    max_token_budget = I.MAX_TOKENS

    def __init__(self, tokenizer, delay: float = 0.0):
        self.tokenizer = tokenizer
        self.pad_token_id = PAD
        self.delay = delay
        self.calls: list[tuple[int, int]] = []
        self.active = 0
        self.max_active = 0
        self._guard = threading.Lock()

    def forward(self, arrays):
        with self._guard:
            self.active += 1
            self.max_active = max(self.max_active, self.active)
        b, s = arrays["input_ids"].shape
        self.calls.append((b, s))
        time.sleep(self.delay)
        ids = arrays["input_ids"].astype(np.int64)
        sp = arrays["option_spans"]
        lengths = arrays["mask"].sum(1, keepdims=True)
        logits = np.zeros(arrays["option_mask"].shape, np.float32)
        for i in range(b):
            for j in range(sp.shape[1]):
                a, e = sp[i, j]
                logits[i, j] = (ids[i, a:e].sum() % 97) / 13.0 + 0.01 * lengths[i, 0] + 0.1 * j
        with self._guard:
            self.active -= 1
        return np.where(arrays["option_mask"], logits, -1e9).astype(np.float32)


def expected_answers(model, states, questions, max_len=None):
    out = []
    for s in states:
        r = I.encode(model.tokenizer, s, questions, model.max_token_budget if max_len is None else max_len)
        logits = model.forward(I.collate([r], model.pad_token_id))
        out.append(I.decode(r, logits[0], questions, model.name))
    return out


def states(n, seed=0):
    rng = np.random.default_rng(seed)
    words = ["hello", "world", "ticket", "printer", "jammed", "urgent"]
    return [" ".join(rng.choice(words, size=int(rng.integers(1, 400)))) for _ in range(n)]


def test_plan_batches_respects_budget_and_rows():
    lengths = [int(x) for x in np.random.default_rng(3).integers(50, 9000, size=137)]
    batches = plan_batches(lengths, max_batch_tokens=32768)
    assert sorted(i for idx, _ in batches for i in idx) == list(range(137))
    order = sorted(range(137), key=lambda i: (-lengths[i], i))
    assert [i for idx, _ in batches for i in idx] == order  # contiguous runs of the length order
    for idx, seq in batches:
        assert seq % 128 == 0 and max(lengths[i] for i in idx) <= seq < max(lengths[i] for i in idx) + 128
        assert len(idx) * seq <= 32768 or len(idx) == 1
        assert len(idx) <= 64
    assert plan_batches([16384], 1024) == [([0], 16384)]  # one over-budget record runs alone
    assert plan_batches([16384] * 4) == [([0, 1, 2, 3], 16384)]  # the max_len case: one batch
    assert plan_batches([]) == []


def test_plan_batches_minimises_the_cost_model():
    """The cut points are optimal for ``batch_cost``: no single greedy plan
    (any fixed length ratio) and no brute-force split of a small case beats
    them, and on the serving sweep's lognormal lengths the plan pads little."""
    from itertools import combinations

    from deciax_b200.engine import batch_cost

    def cost(batches):
        return sum(batch_cost(len(idx), seq) for idx, seq in batches)

    def greedy(lengths, fill, budget=65536, rows=64):
        order = sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))
        out, pos = [], 0
        while pos < len(order):
            seq = -(-lengths[order[pos]] // 128) * 128
            cap = max(1, min(rows, budget // seq))
            end = pos + 1
            while end < len(order) and end - pos < cap and lengths[order[end]] >= fill * lengths[order[pos]]:
                end += 1
            out.append((order[pos:end], seq))
            pos = end
        return out

    rng = np.random.default_rng(5)
    lengths = [int(x) for x in np.clip(np.round(rng.lognormal(np.log(600), 0.8, 256)), 32, 16384)]
    plan = plan_batches(lengths)
    for fill in (0.0, 0.5, 0.75, 0.85, 0.9, 0.95, 1.0):
        assert cost(plan) <= cost(greedy(lengths, fill)) + 1e-6, fill
    padded = sum(len(idx) * seq for idx, seq in plan)
    assert sum(lengths) / padded > 0.9
    small = [int(x) for x in rng.integers(100, 3000, size=9)]
    order = sorted(range(9), key=lambda i: (-small[i], i))
    best = min(
        cost([(order[a:b], -(-small[order[a]] // 128) * 128) for a, b in zip((0, *cuts), (*cuts, 9))])
        for k in range(9) for cuts in combinations(range(1, 9), k)
    )
    assert abs(cost(plan_batches(small)) - best) < 1e-6


def test_engine_matches_per_record_answers_in_input_order():
    questions = FIX["schemas"]["mixed"]
    model = FakeReplica(TOK)
    ss = states(23) + FIX["states"]
    got = ClefEngine(model, max_batch_tokens=4096).decide_batch(ss, questions)
    assert got == expected_answers(FakeReplica(TOK), ss, questions)
    assert all(s % 128 == 0 for _, s in model.calls)
    assert len(model.calls) < len(ss) // 2  # larger batches than the reference's fixed pairs


class WarmCountingReplica(FakeReplica):
    def __init__(self, tokenizer):
        super().__init__(tokenizer)
        self.warmups: list[dict] = []

    def warmup(self, **kw):
        self.warmups.append(kw)


def test_engine_warms_every_replica_once_before_the_first_forward():
    questions = FIX["schemas"]["reference_test"]
    replicas = [WarmCountingReplica(TOK) for _ in range(2)]
    engine = ClefEngine(replicas[0], replicas=replicas, max_batch_tokens=4096)
    engine.decide_batch(states(3), questions)
    engine.decide_batch(states(5), questions)
    assert [len(r.warmups) for r in replicas] == [1, 1]
    assert replicas[0].warmups[0] == {"max_batch_tokens": 4096, "max_rows": I.ROW_BUCKETS[-1]}
    cold = WarmCountingReplica(TOK)
    ClefEngine(cold, auto_warmup=False).decide_batch(states(3), questions)
    assert cold.warmups == [] and cold.calls  # served without a reservation


def test_engine_data_parallel_replicas_run_concurrently():
    questions = FIX["schemas"]["reference_test"]
    replicas = [FakeReplica(TOK, delay=0.05) for _ in range(4)]
    ss = states(64, seed=1)
    engine = ClefEngine(replicas[0], replicas=replicas, max_batch_tokens=1024)
    got = engine.decide_batch(ss, questions, max_len=600)
    assert got == expected_answers(FakeReplica(TOK), ss, questions, max_len=600)
    assert sum(1 for r in replicas if r.calls) >= 2
    assert all(r.max_active == 1 for r in replicas)  # one batch at a time per replica


def test_engine_errors_follow_the_reference():
    model = FakeReplica(TOK)
    engine = ClefEngine(model)
    with pytest.raises(ValueError, match="head_max_len"):
        engine.decide_batch(["x"], {"q": {"type": "noul"}}, head_max_len=10)
    with pytest.raises(ValueError, match="at least one question"):
        engine.decide_batch(["x"], {})
    assert engine.decide_batch([], {"q": {"type": "noul"}}) == []

    class NaNReplica(FakeReplica):
        def forward(self, arrays):
            return np.full(arrays["option_mask"].shape, np.nan, np.float32)

    replicas = [NaNReplica(TOK), NaNReplica(TOK)]
    with pytest.raises(FloatingPointError, match="non-finite"):
        ClefEngine(replicas[0], replicas=replicas, max_batch_tokens=256).decide_batch(states(9), {"q": {"type": "noul"}})
