"""``ClefCudaModel.from_pretrained`` on a checkpoint directory in the Hub
layout (models/clef/model.py:51-85, weights.py:70-101): backbone shards with
an index, a vision-tower tensor to skip, Gated DeltaNet layers stored with the
fused ``in_proj_qkv`` / ``conv1d`` tensors the library splits, attention
layers under ``self_attn``, and the joint head.  The loaded model must give
bit-identical logits and hidden states to ``from_arrays`` on the same
tensors (split and renamed as weights.py:43-57 does), alone and as
tensor-parallel shards."""

from __future__ import annotations

import numpy as np
import pytest
from checkpoint_helpers import mixed_config, write_checkpoint

from deciax_b200.model import ClefCudaModel
from deciax_b200.synthetic import BatchSpec, synthetic_batch, synthetic_weights

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["bf16", "fp32"])
def test_from_pretrained_matches_from_arrays(tmp_path, dtype):
    config, head = mixed_config()
    top, layers, hp = synthetic_weights(config, head, seed=21, embed_std=1.0, dtype="bf16")
    extra = {"model.visual.blocks.0.attn.qkv.weight": np.ones((8, 8), np.float32)}
    d = write_checkpoint(tmp_path / "clef", config, head, top, layers, hp, shards=3, extra=extra)
    loaded = ClefCudaModel.from_pretrained(d, dtype=dtype, max_seq_len=256)
    assert loaded.pad_token_id == 1 and loaded.tokenizer.token_to_id("<|endoftext|>") == 1
    direct = ClefCudaModel.from_arrays(config, head, top, layers, hp, dtype=dtype, max_seq_len=256)
    arrays = synthetic_batch(BatchSpec(states=3, seq=256, questions=2, options_per_question=3, lengths=(256, 130, 40),
                                       row_bucket=4), config.vocab_size, seed=22)
    a_logits, a_hidden = loaded.forward_with_hidden(arrays)
    b_logits, b_hidden = direct.forward_with_hidden(arrays)
    np.testing.assert_array_equal(a_logits, b_logits)
    valid = arrays["mask"]
    np.testing.assert_array_equal(a_hidden[valid], b_hidden[valid])
    assert np.isfinite(a_logits[arrays["option_mask"]]).all()
    loaded.close()
    direct.close()


def test_bad_tensor_shape_in_checkpoint_is_value_error(tmp_path):
    config, head = mixed_config()
    top, layers, hp = synthetic_weights(config, head, seed=23, dtype="bf16")
    layers[1] = dict(layers[1])
    layers[1]["mlp.up_proj.weight"] = layers[1]["mlp.up_proj.weight"][:-1]  # one row short
    d = write_checkpoint(tmp_path / "clef", config, head, top, layers, hp)
    with pytest.raises(ValueError, match="shape mismatch for layers.1.mlp.up_proj.weight"):
        ClefCudaModel.from_pretrained(d, dtype="bf16", max_seq_len=256)
