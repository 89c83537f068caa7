"""Tensor parallelism across GPUs: every rank holds a shard (attention heads,
Gated DeltaNet key/value heads and MLP columns split as
models/clef/weights.py:60-67), o-proj / out_proj and down-proj partial sums
are all-reduced in FP32 over NCCL before the cast (qwen3_5/pallas.py:
66-69,121), and rank 0's logits must match the single-GPU oracle.

Runs one spawned process per GPU; skipped with fewer than two GPUs.
"""

from __future__ import annotations

import multiprocessing as mp
import traceback

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _config(kind: str):
    from deciax_b200.config import HeadConfig, TextConfig

    head = HeadConfig(heads=4, routing_layers=1, layers=1, width=64, ffn=128)
    if kind == "mixed":  # Gated DeltaNet layers shard by key/value heads (qwen3_5/pallas.py:84-90)
        return TextConfig(
            hidden_size=512, intermediate_size=3072, num_attention_heads=4, num_key_value_heads=2, head_dim=256,
            linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=64, linear_value_head_dim=64,
            linear_conv_kernel_dim=4, layer_types=("linear_attention", "full_attention"), rms_norm_eps=1e-6,
            rope_theta=10000.0, partial_rotary_factor=0.25, vocab_size=300), head
    # intermediate 3072: at TP=2 the down-proj (K = 1536) runs the fused GEMM + peer reduction in
    # bf16, the o-proj (K = 512) the unfused pull kernel
    return TextConfig.full_attention(hidden_size=512, intermediate_size=3072, num_attention_heads=4, num_key_value_heads=2,
                                     head_dim=256, num_layers=2, vocab_size=300), head


def _worker(rank, world, nccl_id, dtype, kind, queue):
    try:
        import sys
        from pathlib import Path

        root = Path(__file__).resolve().parents[1]
        sys.path[:0] = [str(root), str(root / "tests")]
        from gpu_helpers import round_tree

        from deciax_b200.model import ClefCudaModel
        from deciax_b200.synthetic import BatchSpec, synthetic_batch, synthetic_weights

        config, head = _config(kind)
        top, layers, hp = synthetic_weights(config, head, seed=5, embed_std=1.0)
        top, layers, hp = round_tree(top, dtype), round_tree(layers, dtype), round_tree(hp, dtype)
        model = ClefCudaModel.from_arrays(config, head, top, layers, hp, dtype=dtype, device=rank, tp_rank=rank,
                                          tp_size=world, nccl_id=nccl_id, max_seq_len=256)
        arrays = synthetic_batch(BatchSpec(states=3, seq=256, questions=2, options_per_question=3,
                                           lengths=(256, 130, 40), row_bucket=4), config.vocab_size, seed=6)
        logits, hidden = model.forward_with_hidden(arrays)
        queue.put((rank, logits, hidden, None))
        model.close()
    except Exception:  # report instead of hanging the parent
        queue.put((rank, None, None, traceback.format_exc()))


def _run_tp(world: int, dtype: str, kind: str = "full"):
    import torch

    from deciax_b200 import _lib

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import ctypes

    lib = _lib.load()
    nid = ctypes.create_string_buffer(_lib.NCCL_ID_BYTES)
    _lib.check(lib.clef_nccl_unique_id(nid))
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, nid.raw, dtype, kind, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, logits, hidden, err = queue.get(timeout=600)
            assert err is None, err
            results[rank] = (logits, hidden)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():  # a peer that died leaves the other blocked in NCCL init
                p.terminate()
    return results


def _oracle(dtype, kind: str = "full"):
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parent))
    from gpu_helpers import oracle_config, oracle_head, round_tree

    from deciax_b200.synthetic import BatchSpec, synthetic_batch, synthetic_weights
    from oracle import clef_oracle as O

    config, head = _config(kind)
    top, layers, hp = synthetic_weights(config, head, seed=5, embed_std=1.0)
    top, layers, hp = round_tree(top, dtype), round_tree(layers, dtype), round_tree(hp, dtype)
    arrays = synthetic_batch(BatchSpec(states=3, seq=256, questions=2, options_per_question=3,
                                       lengths=(256, 130, 40), row_bucket=4), config.vocab_size, seed=6)
    logits, hidden = O.forward(top, layers, hp, arrays, oracle_config(config), oracle_head(head), dtype, return_hidden=True)
    return arrays, logits, hidden


@pytest.mark.parametrize("kind", ["full", "mixed"])
def test_tp2_fp32_matches_oracle(kind):
    results = _run_tp(2, "fp32", kind)
    arrays, exp_logits, exp_hidden = _oracle("fp32", kind)
    valid = arrays["mask"]
    scale = np.abs(exp_hidden[valid]).max()
    for rank, (logits, hidden) in results.items():
        np.testing.assert_allclose(hidden[valid], exp_hidden[valid], rtol=1e-4, atol=1e-4 * scale)
        m = arrays["option_mask"]
        np.testing.assert_allclose(logits[m], exp_logits[m], rtol=1e-4, atol=1e-4)
    np.testing.assert_array_equal(results[0][0], results[1][0])  # every rank ends with the same logits


@pytest.mark.parametrize("kind", ["full", "mixed"])
def test_tp2_bf16_probabilities(kind):
    from gpu_helpers import probs_close

    results = _run_tp(2, "bf16", kind)
    arrays, exp_logits, exp_hidden = _oracle("bf16", kind)
    err, flips = probs_close(results[0][0], exp_logits, arrays)
    assert err < 1e-2 and flips == 0, (err, flips)
    # bf16 TP runs the fused GEMM + peer reduction: each owner writes its rows
    # into every rank's residual stream, so both ranks hold the same bits
    np.testing.assert_array_equal(results[0][1], results[1][1])
    valid = arrays["mask"]
    got, exp = results[0][1][valid], exp_hidden[valid]
    scale = np.abs(exp).max()
    assert np.abs(got - exp).max() < 3e-2 * scale and np.abs(got - exp).mean() < 2e-3 * scale
