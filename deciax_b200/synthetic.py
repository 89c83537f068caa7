"""Seeded synthetic weights and collated batches for benchmarks and tests.

No checkpoint or dataset is available offline, so every measured workload is
random-init weights of the Clef architecture and uniform token ids, shaped
like ``collate``'s output (models/clef/input.py:140-182).

Batch layout (the benchmark configs): each of ``b`` states has ``length``
real tokens (ids uniform over the vocabulary).  Its ``questions`` choice
fields each own an 8-token block at the end of the real tokens: 4 tokens of
question span, then 4 single-token option spans.  Lexical ids are those
option tokens.  ``types`` = 1 (choice), ``option_field`` = question index.
"""

from __future__ import annotations

from dataclasses import dataclass

import ml_dtypes
import numpy as np

from deciax_b200.config import HeadConfig, TextConfig

SEQUENCE_BUCKETS = (128, 256, 512, 1024, 2048, 4096, 8192, 16384)
SCHEMA_BUCKETS = (1, 2, 4, 8, 16, 32, 64, 128, 256, 512)


def bucket(n: int, buckets) -> int:
    for b in buckets:
        if n <= b:
            return b
    raise ValueError(f"{n} exceeds the largest bucket {buckets[-1]}")


def synthetic_weights(config: TextConfig, head: HeadConfig, seed: int, std: float = 0.02, embed_std: float = 0.02,
                      dtype: str = "fp32"):
    """(top, layers, head) dicts of float32 (or bfloat16) arrays, N(0, std).

    Norm weights are N(0, std) too (applied as 1 + w by RMSNorm; LayerNorm
    weights in the head are 1 + N(0, std), biases N(0, std)).
    """
    rng = np.random.default_rng(seed)
    D, F, hq, hkv, d = config.hidden_size, config.intermediate_size, config.num_attention_heads, config.num_key_value_heads, config.head_dim
    V, W, FF = config.vocab_size, head.width, head.ffn
    cast = (lambda a: a.astype(ml_dtypes.bfloat16)) if dtype == "bf16" else (lambda a: a.astype(np.float32))

    def n(*shape, s=std):
        return cast(rng.standard_normal(shape, dtype=np.float32) * np.float32(s))

    emb = n(V, D, s=embed_std)
    top = {"embedding": emb, "lm_head": emb.copy(), "norm": n(D)}
    layers = []
    for kind in config.layer_types:
        if kind == "linear_attention":
            layers.append({
                "input_layernorm.weight": n(D),
                "post_attention_layernorm.weight": n(D),
                **gdn_weights(rng, config, std, cast),
                "mlp.gate_proj.weight": n(F, D),
                "mlp.up_proj.weight": n(F, D),
                "mlp.down_proj.weight": n(D, F),
            })
            continue
        layers.append(
            {
                "input_layernorm.weight": n(D),
                "post_attention_layernorm.weight": n(D),
                "mixer.q_proj.weight": n(hq * 2 * d, D),
                "mixer.k_proj.weight": n(hkv * d, D),
                "mixer.v_proj.weight": n(hkv * d, D),
                "mixer.o_proj.weight": n(D, hq * d),
                "mixer.q_norm.weight": n(d),
                "mixer.k_norm.weight": n(d),
                "mlp.gate_proj.weight": n(F, D),
                "mlp.up_proj.weight": n(F, D),
                "mlp.down_proj.weight": n(D, F),
            }
        )
    return top, layers, _head_weights(rng, D, head, std, cast)


def gdn_weights(rng, config: TextConfig, std: float, cast) -> dict:
    """Gated DeltaNet mixer weights under the split names of
    models/clef/weights.py:43-57.  Projections N(0, std); conv taps N(0, 0.5)
    (the scale of PyTorch's default Conv1d init at width 4); A_log = log of
    U(0.01, 0.3), so per-token decays span slow and fast; dt_bias N(0, 0.5);
    the gated norm's weight (applied as w, not 1 + w) 1 + N(0, 0.1)."""
    D = config.hidden_size
    nh, nv, dh, width = (config.linear_num_key_heads, config.linear_num_value_heads, config.linear_key_head_dim,
                         config.linear_conv_kernel_dim)
    dv = config.linear_value_head_dim

    def n(*shape, s=std):
        return cast(rng.standard_normal(shape, dtype=np.float32) * np.float32(s))

    return {
        "mixer.q.weight": n(nh * dh, D),
        "mixer.k.weight": n(nh * dh, D),
        "mixer.v.weight": n(nv * dv, D),
        "mixer.in_proj_z.weight": n(nv * dv, D),
        "mixer.in_proj_a.weight": n(nv, D),
        "mixer.in_proj_b.weight": n(nv, D),
        "mixer.q.conv": n(nh * dh, width, s=0.5),
        "mixer.k.conv": n(nh * dh, width, s=0.5),
        "mixer.v.conv": n(nv * dv, width, s=0.5),
        "mixer.A_log": cast(np.log(rng.uniform(0.01, 0.3, nv)).astype(np.float32)),
        "mixer.dt_bias": n(nv, s=0.5),
        "mixer.norm.weight": cast((1 + rng.standard_normal(dv) * 0.1).astype(np.float32)),
        "mixer.out_proj.weight": n(D, nv * dv),
    }


def synthetic_head_weights(hidden_size: int, head: HeadConfig, seed: int, std: float = 0.02, dtype: str = "fp32"):
    """Joint-head weights alone (the benchmark builds the backbone on the device)."""
    cast = (lambda a: a.astype(ml_dtypes.bfloat16)) if dtype == "bf16" else (lambda a: a.astype(np.float32))
    return _head_weights(np.random.default_rng(seed), hidden_size, head, std, cast)


def _head_weights(rng, D: int, head: HeadConfig, std: float, cast):
    W, FF = head.width, head.ffn

    def n(*shape, s=std):
        return cast(rng.standard_normal(shape, dtype=np.float32) * np.float32(s))

    hp = {}

    def ln(name, dim):
        hp[name + ".weight"] = cast(1 + rng.standard_normal(dim, dtype=np.float32) * np.float32(std))
        hp[name + ".bias"] = n(dim)

    def mha(name):
        hp[name + ".in_proj_weight"] = n(3 * W, W, s=max(std, W**-0.5))
        hp[name + ".in_proj_bias"] = n(3 * W)
        hp[name + ".out_proj.weight"] = n(W, W, s=max(std, W**-0.5))
        hp[name + ".out_proj.bias"] = n(W)

    ln("hidden_norm", D)
    for k in ("memory_projection", "question_projection", "option_question_projection", "global_projection",
              "option_context_projection", "option_lexical_projection"):
        hp[k + ".weight"] = n(W, D, s=max(std, D**-0.5))
    hp["type_embedding.weight"] = n(3, W)
    for i in range(head.routing_layers):
        p = f"evidence_layers.{i}"
        ln(p + ".query_norm", W)
        ln(p + ".memory_norm", W)
        ln(p + ".feedforward_norm", W)
        mha(p + ".attention")
        hp[p + ".feedforward.0.weight"] = n(FF, W, s=W**-0.5)
        hp[p + ".feedforward.0.bias"] = n(FF)
        hp[p + ".feedforward.3.weight"] = n(W, FF, s=FF**-0.5)
        hp[p + ".feedforward.3.bias"] = n(W)
    ln("option_summary_norm", W)
    for i in range(head.layers):
        p = f"layers.{i}"
        mha(p + ".self_attn")
        mha(p + ".multihead_attn")
        for k in ("norm1", "norm2", "norm3"):
            ln(p + "." + k, W)
        hp[p + ".linear1.weight"] = n(FF, W, s=W**-0.5)
        hp[p + ".linear1.bias"] = n(FF)
        hp[p + ".linear2.weight"] = n(W, FF, s=FF**-0.5)
        hp[p + ".linear2.bias"] = n(W)
    ln("field_norm", W)
    ln("option_norm", W)
    hp["residual_scorer.0.weight"] = n(W, 4 * W, s=(4 * W) ** -0.5)
    hp["residual_scorer.0.bias"] = n(W)
    hp["residual_scorer.3.weight"] = n(1, W, s=W**-0.5)
    hp["residual_scorer.3.bias"] = n(1)
    # The head module's own initial values, as the reference's head fixture
    # holds them (tests/fixtures/clef_head.npz: all three 0, i.e. logit
    # scales exp(0) = 1 and a residual gate of sigmoid(0)).
    hp["prior_logit_scale"] = cast(np.array(0.0, np.float32))
    hp["joint_logit_scale"] = cast(np.array(0.0, np.float32))
    hp["residual_gate"] = cast(np.array(0.0, np.float32))
    return hp


@dataclass(frozen=True)
class BatchSpec:
    states: int
    seq: int  # sequence bucket
    questions: int = 4
    options_per_question: int = 4
    lengths: tuple[int, ...] = ()  # real tokens per state (default: all = seq)
    row_bucket: int = 0  # pad the batch to this many rows (0 = states)


def synthetic_batch(spec: BatchSpec, vocab: int, seed: int) -> dict[str, np.ndarray]:
    """Collated arrays for ``spec`` (see the module docstring for the layout)."""
    rng = np.random.default_rng(seed)
    b = spec.row_bucket or spec.states
    s, nq, no = spec.seq, spec.questions, spec.options_per_question
    lengths = list(spec.lengths) or [s] * spec.states
    if len(lengths) != spec.states:
        raise ValueError("one length per state")
    block = 4 + no
    if min(lengths) < nq * block:
        raise ValueError("states must hold every question block")
    q_b = bucket(nq, SCHEMA_BUCKETS)
    o_b = bucket(nq * no, SCHEMA_BUCKETS)
    lx = bucket(nq * no, SEQUENCE_BUCKETS)
    a = {
        "input_ids": np.zeros((b, s), np.int32),
        "mask": np.zeros((b, s), bool),
        "lexical_ids": np.zeros((b, lx), np.int32),
        "lexical_spans": np.zeros((b, o_b, 2), np.int32),
        "question_spans": np.zeros((b, q_b, 2), np.int32),
        "question_mask": np.zeros((b, q_b), bool),
        "types": np.zeros((b, q_b), np.int32),
        "option_spans": np.zeros((b, o_b, 2), np.int32),
        "option_mask": np.zeros((b, o_b), bool),
        "option_field": np.zeros((b, o_b), np.int32),
    }
    for i, n in enumerate(lengths):
        ids = rng.integers(0, vocab, n, dtype=np.int32)
        a["input_ids"][i, :n] = ids
        a["mask"][i, :n] = True
        start = n - nq * block
        lex = []
        for k in range(nq):
            q0 = start + k * block
            a["question_spans"][i, k] = (q0, q0 + 4)
            a["question_mask"][i, k] = True
            a["types"][i, k] = 1
            for t in range(no):
                j = k * no + t
                pos = q0 + 4 + t
                a["option_spans"][i, j] = (pos, pos + 1)
                a["option_mask"][i, j] = True
                a["option_field"][i, j] = k
                a["lexical_spans"][i, j] = (len(lex), len(lex) + 1)
                lex.append(int(ids[pos]))
        a["lexical_ids"][i, : len(lex)] = lex
    return a


def field_probabilities(logits: np.ndarray, arrays: dict[str, np.ndarray]) -> list[list[np.ndarray]]:
    """Per state, per field: the softmax over that field's options (input.py:185-192)."""
    out = []
    for i in range(logits.shape[0]):
        fields = []
        mask = np.asarray(arrays["option_mask"][i], bool)
        owner = np.asarray(arrays["option_field"][i])
        for f in sorted(set(owner[mask].tolist())):
            v = logits[i][mask & (owner == f)].astype(np.float64)
            e = np.exp(v - v.max())
            fields.append(e / e.sum())
        out.append(fields)
    return out
