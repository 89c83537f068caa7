"""Regenerate ``clef_input.json``: known answers of the reference's host-side
Clef input pipeline (``src/deciax/models/clef/input.py:29-214``: question
validation, ``encode``, ``collate`` and ``decode``).

    python tests/golden/make_input_golden.py [REFERENCE_ROOT]

Imports the reference module from REFERENCE_ROOT/src (the reference deciax
checkout: the first argument, else the REFERENCE_ROOT environment variable).
The reference package's ``__init__`` pulls in JAX, which
this machine lacks and which the input module never touches, so the script
registers an empty ``deciax`` package pointing at the sources and a stub
``jax`` module (only used there for type annotations in ``models/base.py``).

The fixture holds the tokenizer (a word-level vocabulary trained here from the
prompt template plus the test states, serialised with ``Tokenizer.to_str()``),
the cases (states, question schemas, token budgets), and for each case the
reference's records, collated arrays and decoded answers for seeded logits,
plus the ``ValueError`` messages of invalid schemas.  The tests only read the
JSON.
"""

from __future__ import annotations

import json
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def reference_root() -> Path:
    """The reference checkout: the first argument, else $REFERENCE_ROOT."""
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT")
    if not root:
        raise SystemExit(f"usage: python {Path(__file__).name} REFERENCE_ROOT (or set REFERENCE_ROOT)")
    return Path(root)


def import_reference(reference: Path):
    src = reference / "src" / "deciax"
    pkg = types.ModuleType("deciax")
    pkg.__path__ = [str(src)]
    sys.modules["deciax"] = pkg
    jax = types.ModuleType("jax")
    jax.Array = object
    sys.modules.setdefault("jax", jax)
    sys.dont_write_bytecode = True
    from deciax.models.clef import input as clef_input

    return clef_input


def tokenizer_for(texts: list[str]):
    from tokenizers import Tokenizer, models, pre_tokenizers, trainers

    tok = Tokenizer(models.WordLevel(unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.train_from_iterator(texts, trainers.WordLevelTrainer(special_tokens=["[UNK]", "<|endoftext|>"]))
    return tok


STATES = [
    "hello",
    "hello world " * 20,
    {"ticket": "Printer on floor 3 is jammed", "priority": 2, "tags": ["hw", "urgent"]},
    "Ünïcödé státe — ‘quoted’ text with 日本語 characters",
    "",
    ["a", 1, None, True, {"nested": {"z": 1, "a": 2}}],
    "long " * 400,
]

SCHEMAS = {
    "reference_test": {
        "sentiment": {"type": "choice", "criteria": {"z": "world", "a": "hello"}},
        "yes": {"type": "noul"},
        "score": {"type": "score", "criteria": ["hello", "world", "hello world"]},
    },
    "mixed": {
        "route": {"type": "choice", "criteria": {"billing": {"team": "finance"}, "10": "numeric key", "2": None, "hardware": "Printers"},
                  "instructions": "Pick the owning team"},
        "escalate": {"type": "noul", "criteria": {"true": "Needs a human now"}, "instructions": {"why": "urgency", "k": [1, 2]}},
        "severity": {"type": "score", "criteria": ["none", {"level": "low"}, "medium", "high", "critical"], "instructions": ""},
        "plain": {"type": "noul", "criteria": None},
    },
    "single": {"x": {"type": "choice", "criteria": {"a": "hello", "b": "world"}}},
}

INVALID = [
    {},
    {"q": {"type": []}},
    {"q": {"type": "score", "criteria": []}},
    {"q": {"type": "noul", "criteria": {"yes": "yes"}}},
    {"q": {"type": "choice", "criteria": {"a": "a"}, "option_order": ["a"]}},
    {"q": {"type": "choice", "criteria": {"a": "a"}, "labels": ["a"]}},
    {"q": {"type": "choice", "criteria": []}},
    {"q": {"type": "score", "criteria": {"a": 1}}},
    {"": {"type": "noul"}},
    {1: {"type": "noul"}},
    {"q": "noul"},
    {"q": {"type": "other"}},
    {f"q{i}": {"type": "noul"} for i in range(65)},
    {f"q{i}": {"type": "score", "criteria": list(range(100))} for i in range(6)},
]


def main() -> None:
    reference = reference_root()
    I = import_reference(reference)

    corpus = [I.SYSTEM_PROMPT, "SCHEMA FIELDS FIELD ID TYPE INSTRUCTION ALLOWED OPTIONS OPTION END STATE JOINT DECISIONS"]
    corpus += [I.render(s) for s in STATES]
    for schema in SCHEMAS.values():
        corpus += [json.dumps(schema)]
        for qid, q in schema.items():
            corpus += [qid] + [I.render({"option_id": k, "description": v}) for k, v in I.options(q)]
    tok = tokenizer_for(corpus)
    rng = np.random.default_rng(41)

    cases = []
    for name, schema in SCHEMAS.items():
        fixed = len(I.encode(tok, "", schema, I.MAX_TOKENS).ids)
        for budget in (I.MAX_TOKENS, fixed + 7, fixed):
            records = [I.encode(tok, s, schema, budget) for s in STATES]
            arrays = I.collate(records, tok.token_to_id("<|endoftext|>"))
            n_opt = sum(len(f.option_ids) for f in records[0].fields)
            logits = rng.normal(0, 2, size=(len(records), arrays["option_mask"].shape[1])).astype(np.float32)
            if name == "mixed":
                logits[0, :n_opt] = 0.0  # ties: choice picks the first key in criteria order
            decoded = [I.decode(r, logits[i], schema, "clef") for i, r in enumerate(records)]
            cases.append({
                "schema": name, "budget": budget, "fixed": fixed,
                "records": [{"ids": list(r.ids), "fields": [
                    {"id": f.id, "kind": f.kind, "span": list(f.span), "option_spans": [list(s) for s in f.option_spans],
                     "option_ids": list(f.option_ids)} for f in r.fields]} for r in records],
                "arrays": {k: v.astype(np.int32).tolist() for k, v in arrays.items()},
                "logits": logits.tolist(),
                "decoded": decoded,
            })
        try:
            I.encode(tok, "", schema, fixed - 1)
        except ValueError as e:
            cases[-1]["too_small"] = {"budget": fixed - 1, "error": str(e)}

    invalid = []
    for q in INVALID:
        try:
            I.validate_questions(q)
            invalid.append({"questions": repr(q), "error": None})
        except ValueError as e:
            invalid.append({"questions": repr(q), "error": str(e)})

    bad_budgets = []
    for b in (0, I.MAX_TOKENS + 1, True, 3.0):
        try:
            I.encode(tok, "", SCHEMAS["single"], b)
        except ValueError as e:
            bad_budgets.append({"budget": repr(b), "error": str(e)})

    out = {
        "generator": "tests/golden/make_input_golden.py",
        "reference": "src/deciax/models/clef/input.py",
        "tokenizer": tok.to_str(),
        "states": STATES,
        "schemas": SCHEMAS,
        "cases": cases,
        "invalid": invalid,
        "bad_budgets": bad_budgets,
    }
    (HERE / "clef_input.json").write_text(json.dumps(out, ensure_ascii=False, separators=(",", ":")))


if __name__ == "__main__":
    main()
