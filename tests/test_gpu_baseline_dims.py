"""Parity at the benchmark's own dimensions (clef-flash: hidden 3584, 16 query /
8 key-value heads of 256, gated MLP 14336).

* cfg1, the correctness case: one full-attention layer in FP32 on x ~ N(0, 1)
  of shape [1, 512, 3584] with weights N(0, 0.02) from seed 0 and an all-ones
  mask, at partial rotary 0.25 (the reference default) and 1.0.  The input x
  enters as the embedding table: ``synthetic_weights`` draws the [512, 3584]
  embedding first from seed 0 at std 1.0, and token ids 0..511 select its rows
  in order.  Bar: final hidden states within 1e-4 relative (rtol 1e-4, atol
  1e-4 x max|h|) and logits within 1e-4 of the oracle
  (models/qwen3_5/text.py:70-102, kernels/attention/blocked.py:9-32).
* A two-layer slice of the cfg2 benchmark model in BF16 at S = 2048 (V = 256000,
  the benchmark's joint head), on a full and a ragged state: option
  probabilities within 1e-2 and no argmax flip unless the oracle's top-2 gap
  is below 1e-3.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

from deciax_b200.config import HeadConfig, TextConfig
from deciax_b200.model import ClefCudaModel
from deciax_b200.synthetic import BatchSpec, synthetic_batch, synthetic_weights
from oracle import clef_oracle as O

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
CFG1 = dict(hidden_size=3584, intermediate_size=14336, num_attention_heads=16, num_key_value_heads=8, head_dim=256,
            num_layers=1, vocab_size=512)


@pytest.mark.parametrize("prf", [0.25, 1.0])
def test_cfg1_layer_fp32_matches_oracle(prf):
    config = TextConfig.full_attention(**CFG1, partial_rotary_factor=prf)
    head = HeadConfig(heads=4, routing_layers=1, layers=1, width=64, ffn=128)
    top, layers, hp = synthetic_weights(config, head, seed=0, std=0.02, embed_std=1.0)
    model = ClefCudaModel.from_arrays(config, head, top, layers, hp, dtype="fp32", max_seq_len=512)
    arrays = synthetic_batch(BatchSpec(states=1, seq=512, questions=4, options_per_question=4), 512, seed=0)
    arrays["input_ids"][0] = np.arange(512, dtype=np.int32)  # embedding rows = x, in order
    logits, hidden = model.forward_with_hidden(arrays)
    model.close()
    oc = O.TextConfig(hidden_size=3584, intermediate_size=14336, num_attention_heads=16, num_key_value_heads=8,
                      head_dim=256, partial_rotary_factor=prf)
    exp_logits, exp_hidden = O.forward(top, layers, hp, arrays, oc, O.HeadConfig(heads=4, routing_layers=1, layers=1),
                                       "fp32", return_hidden=True)
    scale = np.abs(exp_hidden).max()
    np.testing.assert_allclose(hidden, exp_hidden, rtol=1e-4, atol=1e-4 * scale)
    m = arrays["option_mask"]
    np.testing.assert_allclose(logits[m], exp_logits[m], rtol=1e-4, atol=1e-4)


def test_cfg2_slice_bf16_probabilities():
    sys.path.insert(0, str(ROOT))
    import bench

    r = bench.cfg2_slice_parity(0, layers=2, lengths=(2048, 1531), seed=12)
    assert r["fields"] == 8
    assert r["max_prob_err"] < 1e-2, r
    assert r["argmax_flips"] == 0, r
    assert r["ok"], r
