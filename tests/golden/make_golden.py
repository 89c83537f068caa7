"""Regenerate the golden fixtures that pin the CPU oracle.

    python tests/golden/make_golden.py [REFERENCE_ROOT]

Writes, next to this script:

* ``clef_head.npz`` / ``clef_head.json`` -- the reference deciax repository's
  own joint-head fixture (``tests/fixtures/clef_head.npz``: Cloudflare's torch
  ``JointSchemaHead`` outputs, seed 131), copied byte for byte from
  REFERENCE_ROOT (the first argument, else the REFERENCE_ROOT environment
  variable).  The reference test
  ``tests/clef/test_head.py:11-29`` compares against it at atol 3e-6 / rtol 3e-5.
* ``qwen35_backbone_mixed.npz`` -- Transformers ``Qwen3_5TextModel`` at the
  configuration of the reference test ``tests/test_qwen3_5.py:43-87`` (three
  Gated DeltaNet layers + one full-attention layer, partial rotary 0.5, seed
  21, ids [2, 130] with row 1 padded from 99): weights, inputs and the final
  hidden state.
* ``qwen35_backbone_full.npz`` -- the same model class with every layer
  ``full_attention`` (the layer kind the CUDA library runs), partial rotary
  0.25 and RoPE theta 10000, seed 22.

Needs torch and transformers (>= 5.5 with Qwen3.5) on the machine that runs
it; the tests only read the .npz files.
"""

from __future__ import annotations

import hashlib
import json
import shutil
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def reference_root() -> Path:
    """The reference checkout: the first argument, else $REFERENCE_ROOT."""
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT")
    if not root:
        raise SystemExit(f"usage: python {Path(__file__).name} REFERENCE_ROOT (or set REFERENCE_ROOT)")
    return Path(root)


def copy_head_fixture(reference: Path) -> None:
    src = reference / "tests" / "fixtures"
    for name in ("clef_head.npz", "clef_head.json"):
        shutil.copyfile(src / name, HERE / name)


def backbone_fixture(name: str, seed: int, layer_types: list[str], rope: dict, ids_shape=(2, 130), pad_from: int = 99, **dims) -> None:
    import torch
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from transformers.models.qwen3_5.modeling_qwen3_5 import Qwen3_5TextModel

    torch.manual_seed(seed)
    c = Qwen3_5TextConfig(num_hidden_layers=len(layer_types), layer_types=layer_types, rope_parameters=rope, **dims)
    c._attn_implementation = "eager"
    model = Qwen3_5TextModel(c).eval()
    # Perturb every norm weight so the (1 + w) RMSNorm scaling and the gated
    # norm's plain w scaling both see non-trivial weights.
    with torch.no_grad():
        for key, value in model.state_dict().items():
            if key.endswith("norm.weight") and value.ndim == 1:
                value.add_(torch.randn_like(value) * 0.1)
    ids = torch.randint(0, c.vocab_size, ids_shape)
    mask = torch.ones_like(ids)
    mask[1, pad_from:] = 0
    with torch.no_grad():
        expected = model(ids, attention_mask=mask, use_cache=False).last_hidden_state.numpy()
        embedded = model.embed_tokens(ids).numpy()

    saved = {"ids": ids.numpy().astype(np.int32), "mask": mask.numpy().astype(bool), "embedded": embedded, "expected": expected}
    saved.update({"param." + k: v.numpy() for k, v in model.state_dict().items()})
    meta = {k: v for k, v in c.to_dict().items() if isinstance(v, (int, float, str, list, dict, bool)) or v is None}
    saved["config_json"] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
    np.savez_compressed(HERE / f"{name}.npz", **saved)


DIMS = dict(
    vocab_size=100,
    hidden_size=32,
    intermediate_size=64,
    num_attention_heads=4,
    num_key_value_heads=2,
    head_dim=8,
    linear_num_key_heads=2,
    linear_num_value_heads=6,
    linear_key_head_dim=8,
    linear_value_head_dim=8,
    linear_conv_kernel_dim=4,
)


if __name__ == "__main__":
    reference = reference_root()
    copy_head_fixture(reference)
    backbone_fixture(
        "qwen35_backbone_mixed",
        21,
        ["linear_attention"] * 3 + ["full_attention"],
        {"rope_type": "default", "rope_theta": 10000000.0, "partial_rotary_factor": 0.5, "mrope_section": [1, 1, 0], "mrope_interleaved": True},
        **DIMS,
    )
    backbone_fixture(
        "qwen35_backbone_full",
        22,
        ["full_attention"] * 2,
        {"rope_type": "default", "rope_theta": 10000.0, "partial_rotary_factor": 0.25, "mrope_section": [1, 1, 0], "mrope_interleaved": True},
        **{**DIMS, "head_dim": 16},
    )
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size, hashlib.sha256(f.read_bytes()).hexdigest()[:16])
