"""Host side of the Clef path: question validation, prompt encoding, batch
collation and answer decoding.

Restates ``src/deciax/models/clef/input.py`` of the reference (the serialised
prompt and the span layout are the trained model's contract, so the strings,
the token order and the spans are the reference's), with two changes of form
that keep every output identical:

* the schema half of a prompt depends only on the questions, so
  ``SchemaPrompt`` tokenises it once and ``SchemaPrompt.record`` binds a
  state's tokens to it -- a batch of states sharing one schema (the shape of
  ``decide_batch``) tokenises the schema once instead of once per state;
* ``collate`` fills the padded arrays with NumPy slices per record.

Error behaviour (exception types and messages) follows the reference.
"""

from __future__ import annotations

import json
from collections.abc import Mapping, Sequence
from dataclasses import dataclass
from typing import Any

import numpy as np

# input.py:23-28 (the system prompt and type order are fixed by the trained checkpoint)
SYSTEM_PROMPT = (
    "Read the complete state and schema. Decide every field jointly. Each answer must be exactly one of that field's "
    "allowed options."
)
CLEF_QTYPES = {"noul": 0, "choice": 1, "score": 2}
SEQUENCE_BUCKETS = (128, 256, 512, 1024, 2048, 4096, 8192, 16384)
MAX_TOKENS = SEQUENCE_BUCKETS[-1]
SCHEMA_BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128, 256, 512)
ROW_BUCKETS = (1, 2, 4, 8, 16, 32, 64)  # runtime/buckets.py:14
MAX_QUESTIONS = 64  # protocol/systemone.py:17
MAX_TOTAL_OPTIONS = 512  # protocol/systemone.py:22

NOUL_CRITERIA = {"true": "The proposition is true or the answer is yes.", "false": "The proposition is false or the answer is no."}


def bucket(n: int, buckets: Sequence[int]) -> int:
    """Smallest bucket >= n (runtime/buckets.py:17-22)."""
    for b in sorted(buckets):
        if b >= n:
            return b
    raise ValueError(f"{n} exceeds the largest bucket {max(buckets)}")


def render(value: Any) -> str:
    """Strings verbatim, anything else as compact sorted-key JSON (input.py:31-32)."""
    if isinstance(value, str):
        return value
    return json.dumps(value, ensure_ascii=False, separators=(",", ":"), sort_keys=True)


def options(question: Mapping[str, Any]) -> list[tuple[str, Any]]:
    """(option id, description) in model order (input.py:35-44): noul is
    true/false with default criteria, choice ids sort as strings, score ids
    are the level indices."""
    kind = question["type"]
    if kind == "noul":
        criteria = {**NOUL_CRITERIA, **(question.get("criteria") or {})}
        return [("true", criteria["true"]), ("false", criteria["false"])]
    if kind == "choice":
        return sorted((str(k), v) for k, v in question["criteria"].items())
    return [(str(i), v) for i, v in enumerate(question["criteria"])]


@dataclass(frozen=True)
class Field:
    id: str
    kind: int
    span: tuple[int, int]
    option_spans: tuple[tuple[int, int], ...]
    option_ids: tuple[str, ...]


@dataclass(frozen=True)
class Record:
    ids: tuple[int, ...]
    fields: tuple[Field, ...]


def validate_questions(questions: Mapping[Any, Any]) -> None:
    """input.py:62-88, same checks in the same order and the same messages."""
    if not isinstance(questions, Mapping) or not questions:
        raise ValueError("Clef requires at least one question")
    if len(questions) > MAX_QUESTIONS:
        raise ValueError(f"Clef supports at most {MAX_QUESTIONS} questions per request")
    total = 0
    for qid, q in questions.items():
        if not isinstance(qid, str) or not qid:
            raise ValueError("Clef question ids must be nonempty strings")
        kind = q.get("type") if isinstance(q, Mapping) else None
        if not isinstance(kind, str) or kind not in CLEF_QTYPES:
            raise ValueError(f"{qid}: type must be noul, choice, or score")
        if "labels" in q or "option_order" in q:
            raise ValueError(f"{qid}: Clef does not support labels or option_order")
        criteria = q.get("criteria")
        if kind == "choice" and not (isinstance(criteria, dict) and criteria):
            raise ValueError(f"{qid}: choice criteria must be a nonempty object")
        if kind == "score" and not (isinstance(criteria, list) and criteria):
            raise ValueError(f"{qid}: score criteria must be a nonempty list")
        if kind == "noul" and criteria is not None and not (isinstance(criteria, dict) and set(criteria) <= {"true", "false"}):
            raise ValueError(f"{qid}: noul criteria must use true/false keys")
        total += len(options(q))
    if total > MAX_TOTAL_OPTIONS:
        raise ValueError(f"Clef supports at most {MAX_TOTAL_OPTIONS} total options per request")


def _check_budget(max_length: Any) -> None:
    if isinstance(max_length, bool) or not isinstance(max_length, int) or not 1 <= max_length <= MAX_TOKENS:
        raise ValueError(f"Clef max_len must be between 1 and {MAX_TOKENS}")


class SchemaPrompt:
    """The state-independent parts of a Clef prompt for one question schema.

    Layout (input.py:97-136): ``prefix | state | schema | suffix``.  Field and
    option spans are kept relative to the schema block and shifted by
    ``len(prefix) + len(state)`` when a state is bound.
    """

    def __init__(self, tokenizer: Any, questions: Mapping[str, Any]) -> None:
        validate_questions(questions)
        self.tokenizer = tokenizer
        self.questions = questions
        tok = self.tokens
        schema = tok("\n\nSCHEMA FIELDS:\n")
        fields = []
        for i, (qid, q) in enumerate(questions.items()):
            schema += tok(f"\nFIELD {i + 1}\nID: {qid}\nTYPE: {q['type']}\nINSTRUCTION: ")
            start = len(schema)
            instruction = q.get("instructions")
            schema += tok(qid if instruction in (None, "") else render(instruction))
            span = (start, len(schema))
            schema += tok("\nALLOWED OPTIONS:\n")
            spans, ids = [], []
            for j, (oid, description) in enumerate(options(q)):
                schema += tok(f"OPTION {j + 1}: ")
                start = len(schema)
                semantics = {"option_id": oid} if description is None else {"option_id": oid, "description": description}
                schema += tok(render(semantics))
                spans.append((start, len(schema)))
                ids.append(oid)
                schema += tok("\n")
            schema += tok("END FIELD\n")
            fields.append(Field(qid, CLEF_QTYPES[q["type"]], span, tuple(spans), tuple(ids)))
        self.prefix = tok(f"<|im_start|>system\n{SYSTEM_PROMPT}<|im_end|>\n<|im_start|>user\nSTATE:\n")
        self.suffix = tok("\n<|im_end|>\n<|im_start|>assistant\n<think>\n\n</think>\n\nJOINT SCHEMA DECISIONS:")
        self.schema = schema
        self.fields = tuple(fields)
        self.fixed = len(self.prefix) + len(schema) + len(self.suffix)

    def tokens(self, text: str) -> list[int]:
        return list(self.tokenizer.encode(text, add_special_tokens=False).ids)

    def check(self, max_length: int) -> None:
        _check_budget(max_length)
        if self.fixed > max_length:
            raise ValueError(f"schema requires {self.fixed} tokens before state; maximum is {max_length}")

    def record(self, state_ids: Sequence[int], max_length: int) -> Record:
        """Bind a tokenised state (truncated to the budget left by the schema)."""
        self.check(max_length)
        state_ids = list(state_ids)[: max_length - self.fixed]
        shift = len(self.prefix) + len(state_ids)
        fields = tuple(
            Field(f.id, f.kind, (f.span[0] + shift, f.span[1] + shift), tuple((s + shift, e + shift) for s, e in f.option_spans),
                  f.option_ids)
            for f in self.fields
        )
        return Record(tuple(self.prefix + state_ids + self.schema + self.suffix), fields)

    def encode_states(self, states: Sequence[Any], max_length: int) -> list[Record]:
        """Records for many states; the states are tokenised as one batch."""
        self.check(max_length)
        texts = [render(s) for s in states]
        if hasattr(self.tokenizer, "encode_batch"):
            encoded = self.tokenizer.encode_batch(texts, add_special_tokens=False)
            ids = [e.ids for e in encoded]
        else:
            ids = [self.tokens(t) for t in texts]
        return [self.record(i, max_length) for i in ids]


def encode(tokenizer: Any, state: Any, questions: Mapping[str, Any], max_length: int = MAX_TOKENS) -> Record:
    """One state and its schema as a token record (input.py:91-136)."""
    validate_questions(questions)
    _check_budget(max_length)
    prompt = SchemaPrompt(tokenizer, questions)
    prompt.check(max_length)
    return prompt.record(prompt.tokens(render(state)), max_length)


def collate(records: Sequence[Record], pad_id: int, *, rows: int | None = None, seq_len: int | None = None) -> dict[str, np.ndarray]:
    """Pad records to bucketed shapes; options are flat with explicit field
    ownership and lexical spans index a compact per-row token list
    (input.py:139-182).  ``rows`` / ``seq_len`` override the row and sequence
    buckets (the CUDA model takes any shape; padding never changes a row's
    logits), e.g. to pad only to a multiple of 128 tokens."""
    longest = max(len(r.ids) for r in records)
    b = bucket(len(records), ROW_BUCKETS) if rows is None else rows
    s = bucket(longest, SEQUENCE_BUCKETS) if seq_len is None else seq_len
    if b < len(records) or s < longest:
        raise ValueError("rows / seq_len smaller than the records")
    q = bucket(max(len(r.fields) for r in records), SCHEMA_BUCKETS)
    o = bucket(max(sum(len(f.option_ids) for f in r.fields) for r in records), SCHEMA_BUCKETS)
    option_spans = [[span for f in r.fields for span in f.option_spans] for r in records]
    lex_len = [sum(e - st for st, e in spans) for spans in option_spans]
    lx = bucket(max(lex_len), SEQUENCE_BUCKETS)

    out = {
        "lexical_ids": np.full((b, lx), pad_id, np.int32),
        "lexical_spans": np.zeros((b, o, 2), np.int32),
        "input_ids": np.full((b, s), pad_id, np.int32),
        "mask": np.zeros((b, s), bool),
        "question_spans": np.zeros((b, q, 2), np.int32),
        "question_mask": np.zeros((b, q), bool),
        "types": np.zeros((b, q), np.int32),
        "option_spans": np.zeros((b, o, 2), np.int32),
        "option_mask": np.zeros((b, o), bool),
        "option_field": np.zeros((b, o), np.int32),
    }
    for i, r in enumerate(records):
        ids = np.asarray(r.ids, np.int32)
        n_tok, n_q = len(ids), len(r.fields)
        out["input_ids"][i, :n_tok] = ids
        out["mask"][i, :n_tok] = True
        out["question_spans"][i, :n_q] = [f.span for f in r.fields]
        out["question_mask"][i, :n_q] = True
        out["types"][i, :n_q] = [f.kind for f in r.fields]
        spans = np.asarray(option_spans[i], np.int32).reshape(-1, 2)
        n_o = len(spans)
        out["option_spans"][i, :n_o] = spans
        out["option_mask"][i, :n_o] = True
        out["option_field"][i, :n_o] = np.repeat(np.arange(n_q, dtype=np.int32), [len(f.option_ids) for f in r.fields])
        widths = spans[:, 1] - spans[:, 0]
        ends = np.cumsum(widths, dtype=np.int64)
        out["lexical_spans"][i, :n_o, 0] = ends - widths
        out["lexical_spans"][i, :n_o, 1] = ends
        if n_o:
            out["lexical_ids"][i, : lex_len[i]] = np.concatenate([ids[st:e] for st, e in spans])
    return out


def softmax(z: np.ndarray) -> np.ndarray:
    """protocol/answers.py:44-46 (max-shifted, in the input's dtype)."""
    e = np.exp(z - z.max())
    return e / e.sum()


def decode(record: Record, logits: np.ndarray, questions: Mapping[str, Any], model_name: str) -> dict[str, Any]:
    """Per-field answers from one row of option logits (input.py:185-214):
    noul -> p(true); choice -> argmax in criteria order with its confidence;
    score -> expected level index.  Probabilities are rounded to 4 places."""
    answers: dict[str, Any] = {}
    offset = 0
    for f in record.fields:
        n = len(f.option_ids)
        values = np.asarray(logits[offset : offset + n]).astype(np.float32)
        if not np.isfinite(values).all():
            raise FloatingPointError("non-finite Clef option logits")
        probs = dict(zip(f.option_ids, softmax(values).tolist(), strict=True))
        q = questions[f.id]
        if q["type"] == "noul":
            answer: dict[str, Any] = {"type": "noul", "noul": round(probs["true"], 4)}
        elif q["type"] == "choice":
            keys = [str(k) for k in q["criteria"]]
            chosen = max(keys, key=probs.__getitem__)
            answer = {"type": "choice", "choice": chosen, "confidence": round(probs[chosen], 4),
                      "probabilities": {k: round(probs[k], 4) for k in keys}}
        else:
            keys = list(f.option_ids)
            answer = {
                "type": "score",
                "score": round(sum(i * probs[k] for i, k in enumerate(keys)), 4),
                "confidence": round(max(probs.values()), 4),
                "legend": dict(zip(keys, q["criteria"], strict=True)),
                "probabilities": {k: round(probs[k], 4) for k in keys},
            }
        answers[f.id] = answer
        offset += n
    return {"model": model_name, "answers": answers, "usage": {"input_tokens": len(record.ids), "output_tokens": 0}}
