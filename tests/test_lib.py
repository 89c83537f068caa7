"""CPU checks of the C-ABI boundary: the library builds, loads and exports
every entry point ``include/clef_b200.h`` declares; host-side argument
handling maps errors the way the reference does (ValueError = HTTP 422)."""

from __future__ import annotations

import ctypes
import re
import subprocess

import numpy as np
import pytest
from conftest import ROOT

from deciax_b200 import _lib
from deciax_b200.build import LIB, build
from deciax_b200.config import HeadConfig, TextConfig
from deciax_b200.model import batch_struct
from deciax_b200.synthetic import BatchSpec, synthetic_batch


def declared_functions() -> set[str]:
    text = (ROOT / "include" / "clef_b200.h").read_text()
    return set(re.findall(r"^(?:int|const char\*)\s+(clef_\w+)\(", text, flags=re.M))


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def test_header_and_binding_agree():
    assert declared_functions() == set(_lib.EXPORTS)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = declared_functions() - exported
    assert not missing, missing
    for name in declared_functions():
        assert hasattr(lib, name)


def test_library_links_torch_nccl(lib):
    out = subprocess.run(["ldd", str(LIB)], capture_output=True, text=True, check=True).stdout
    nccl = [line for line in out.splitlines() if "libnccl" in line]
    assert nccl and "nvidia/nccl" in nccl[0]


def test_build_targets_sm100a_only():
    from deciax_b200 import build as b

    assert b.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_error_paths_without_gpu(lib):
    """With no usable device, create fails with a status and a message (never a crash)."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("checks the no-GPU path")
    cfg = _lib.ClefConfigC(hidden_size=32, intermediate_size=64, num_attention_heads=2, num_key_value_heads=1, head_dim=16,
                           num_layers=1, vocab_size=10, rms_norm_eps=1e-6, rope_theta=1e4, partial_rotary_factor=0.25,
                           max_seq_len=128, head_width=16, head_heads=2, head_routing_layers=1, head_layers=1, head_ffn=32)
    h = ctypes.c_void_p()
    st = lib.clef_create(ctypes.byref(cfg), 0, 0, 1, None, _lib.DTYPE_BF16, ctypes.byref(h))
    assert st == _lib.CLEF_ECUDA
    assert lib.clef_last_error(None)


def test_config_validation_is_value_error(lib):
    cfg = _lib.ClefConfigC(hidden_size=32, intermediate_size=64, num_attention_heads=3, num_key_value_heads=2, head_dim=16,
                           num_layers=1, vocab_size=10, rms_norm_eps=1e-6, rope_theta=1e4, partial_rotary_factor=0.25,
                           max_seq_len=128, head_width=16, head_heads=2, head_routing_layers=1, head_layers=1, head_ffn=32)
    h = ctypes.c_void_p()
    st = lib.clef_create(ctypes.byref(cfg), 0, 0, 1, None, _lib.DTYPE_BF16, ctypes.byref(h))
    assert st == _lib.CLEF_EINVAL
    with pytest.raises(ValueError, match="key head groups"):
        _lib.check(st)


def test_op_argument_checks_are_value_errors(lib):
    st = lib.clef_op_gemm(_lib.DTYPE_BF16, 0, 128, 128, 30, 16, 16, 16, 128, None, None, 0, None)
    assert st == _lib.CLEF_EINVAL
    st = lib.clef_op_attention(_lib.DTYPE_BF16, None, None, None, 1, 1, 1, 1, 64, 0.0, 0, None)
    assert st == _lib.CLEF_EINVAL


def test_text_config_mirrors_reference_validation():
    with pytest.raises(ValueError, match="partial rotary"):
        TextConfig.full_attention(hidden_size=32, intermediate_size=64, num_attention_heads=2, num_key_value_heads=1,
                                  head_dim=2, num_layers=1, vocab_size=10, partial_rotary_factor=0.25)
    raw = {"hidden_size": 32, "intermediate_size": 64, "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 8,
           "linear_num_key_heads": 2, "linear_num_value_heads": 4, "linear_key_head_dim": 8, "linear_value_head_dim": 8,
           "linear_conv_kernel_dim": 4, "rms_norm_eps": 1e-6, "num_hidden_layers": 2, "vocab_size": 100,
           "layer_types": ["linear_attention", "full_attention"], "rope_parameters": {"rope_theta": 1e7}}
    c = TextConfig.from_dict({"text_config": raw})
    assert c.partial_rotary_factor == 0.25 and c.vocab_size == 100
    with pytest.raises(ValueError):
        TextConfig.from_dict({**raw, "attn_output_gate": False})
    with pytest.raises(ValueError):
        TextConfig.from_dict({**raw, "num_hidden_layers": 3})


def test_batch_struct_checks_shapes():
    arrays = synthetic_batch(BatchSpec(states=2, seq=128), 50, seed=0)
    keep: list = []
    c = batch_struct(arrays, keep)
    assert (c.b, c.s, c.lx, c.o, c.q) == (2, 128, 128, 16, 4)
    bad = dict(arrays)
    bad["types"] = bad["types"][:, :2]
    with pytest.raises(ValueError):
        batch_struct(bad, [])


def test_synthetic_batch_layout():
    spec = BatchSpec(states=3, seq=256, questions=2, options_per_question=3, lengths=(256, 100, 30), row_bucket=4)
    a = synthetic_batch(spec, 1000, seed=1)
    assert a["mask"].sum(1).tolist() == [256, 100, 30, 0]
    for i, n in enumerate([256, 100, 30]):
        spans = a["option_spans"][i][a["option_mask"][i]]
        assert spans.max() <= n
        lex = a["lexical_ids"][i][: len(spans)]
        np.testing.assert_array_equal(lex, a["input_ids"][i][spans[:, 0]])
    assert not a["option_mask"][3].any()


def test_head_config_fields():
    h = HeadConfig(heads=4, routing_layers=2, layers=2, width=256, ffn=512)
    assert h.width % h.heads == 0
