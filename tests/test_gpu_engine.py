"""``ClefEngine`` over ``ClefCudaModel`` replicas: length-grouped batches and
data-parallel replicas give the answers of one-record forwards (the
reference's ``decide_batch`` semantics, ``runtime/clef.py:23-40``)."""

from __future__ import annotations

import json

import numpy as np
import pytest
from conftest import GOLDEN
from gpu_helpers import round_tree
from tokenizers import Tokenizer

from deciax_b200 import clef_input as I
from deciax_b200.config import HeadConfig, TextConfig
from deciax_b200.engine import ClefEngine
from deciax_b200.model import ClefCudaModel
from deciax_b200.synthetic import synthetic_weights

pytestmark = pytest.mark.gpu

FIX = json.loads((GOLDEN / "clef_input.json").read_text())
TOK = Tokenizer.from_str(FIX["tokenizer"])
PAD = TOK.token_to_id("<|endoftext|>")
CONFIG = TextConfig.full_attention(hidden_size=256, intermediate_size=512, num_attention_heads=4, num_key_value_heads=2,
                                   head_dim=64, num_layers=2, vocab_size=512)
HEAD = HeadConfig(heads=4, routing_layers=2, layers=2, width=64, ffn=128)


def replica(device: int, dtype: str = "fp32"):
    top, layers, hp = (round_tree(t, dtype) for t in synthetic_weights(CONFIG, HEAD, 3, embed_std=1.0))
    return ClefCudaModel.from_arrays(CONFIG, HEAD, top, layers, hp, dtype=dtype, device=device, max_seq_len=2048,
                                     tokenizer=TOK, pad_token_id=PAD)


def states(n: int) -> list[str]:
    rng = np.random.default_rng(5)
    words = ["hello", "world", "ticket", "Printer", "jammed", "urgent", "floor", "priority"]
    return [" ".join(rng.choice(words, size=int(rng.integers(1, 700)))) for _ in range(n)] + FIX["states"]


def worst(a, b) -> float:
    """Largest difference between two answer trees (inf on a structural or label mismatch)."""
    if isinstance(a, dict):
        if a.keys() != b.keys():
            return float("inf")
        return max((worst(a[k], b[k]) for k in a), default=0.0)
    if isinstance(a, float):
        return abs(a - b)
    return 0.0 if a == b else float("inf")


def compare(got, want, tol):
    errs = [worst(g, w) for g, w in zip(got, want, strict=True)]
    assert max(errs) <= tol, (max(errs), errs)


def one_by_one(model, ss, questions):
    out = []
    for s in ss:
        r = I.encode(TOK, s, questions, model.max_token_budget)
        out.append(I.decode(r, model.forward(I.collate([r], PAD))[0], questions, model.name))
    return out


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_engine_batches_match_single_record_forwards(dtype):
    """A record's answers do not depend on the batch it runs in: every GEMM
    path is chosen independently of the row count, so the rounded answers
    agree to one step of the 4-place output in both dtypes."""
    model = replica(0, dtype)
    questions = FIX["schemas"]["mixed"]
    ss = states(21)
    got = model.build_engine().decide_batch(ss, questions)
    want = one_by_one(model, ss, questions)
    compare(got, want, 1e-4)


def test_engine_data_parallel_over_gpus():
    import torch

    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    replicas = [replica(d) for d in range(min(n, 4))]
    questions = FIX["schemas"]["reference_test"]
    ss = states(40)
    got = ClefEngine(replicas[0], replicas=replicas, max_batch_tokens=4096).decide_batch(ss, questions)
    want = one_by_one(replicas[0], ss, questions)
    compare(got, want, 1e-4)


def test_requests_after_warmup_allocate_nothing():
    """The engine's warm-up (reached by the first ``decide_batch``, as the
    reference server's warm-up request reaches ``decide``,
    serve/app.py:385-406) reserves the workspace for every batch the engine
    can form, so later requests of any length and schema allocate no device
    memory, no pinned staging and exchange no handles."""
    model = replica(0, "bf16")
    engine = ClefEngine(model, max_batch_tokens=4096)
    engine.decide_batch(["warmup"], {"q": {"type": "noul", "instructions": "Is this a warmup request?"}})
    after_warmup = model.workspace_allocations
    assert after_warmup > 0
    for name in ("mixed", "reference_test"):
        questions = FIX["schemas"][name]
        engine.decide_batch(states(30), questions)  # long and short states, several batch shapes
        engine.decide_batch(FIX["states"][:1], questions)
    assert model.workspace_allocations == after_warmup
    # without the warm-up a larger batch than any before grows the workspace
    cold = replica(0, "bf16")
    r = I.encode(TOK, states(1)[0], FIX["schemas"]["mixed"], cold.max_token_budget)
    cold.forward(I.collate([r], PAD))
    first = cold.workspace_allocations
    cold.forward(I.collate([r] * 4, PAD))
    assert cold.workspace_allocations > first
