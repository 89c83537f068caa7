"""ctypes binding of ``libclef_b200.so`` (declared in ``include/clef_b200.h``).

The library is the product path; there is no fallback.  ``load()`` raises if
the shared object has not been built.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libclef_b200.so"

CLEF_OK, CLEF_EINVAL, CLEF_ECUDA, CLEF_ENCCL, CLEF_EDEVICE, CLEF_ESTATE = range(6)
DTYPE_F32, DTYPE_BF16 = 0, 1
LAYER_FULL, LAYER_LINEAR = 0, 1
DEBUG_POISON = 1  # CLEF_DEBUG_POISON
NCCL_ID_BYTES = 128

EXPORTS = (
    "clef_nccl_unique_id",
    "clef_create",
    "clef_upload",
    "clef_upload_device",
    "clef_finalize",
    "clef_forward",
    "clef_forward_head",
    "clef_forward_device",
    "clef_reserve",
    "clef_workspace_allocations",
    "clef_check_status",
    "clef_set_timing",
    "clef_timing_report",
    "clef_last_launch_count",
    "clef_set_debug",
    "clef_destroy",
    "clef_last_error",
    "clef_op_gemm",
    "clef_op_gemm_qkv",
    "clef_op_rmsnorm",
    "clef_op_qk_norm_rope",
    "clef_op_qk_norm_rope_noalloc",
    "clef_op_attention",
    "clef_op_gdn_core",
)


class ClefConfigC(ctypes.Structure):
    _fields_ = [
        ("hidden_size", ctypes.c_int32),
        ("intermediate_size", ctypes.c_int32),
        ("num_attention_heads", ctypes.c_int32),
        ("num_key_value_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("num_layers", ctypes.c_int32),
        ("layer_types", ctypes.POINTER(ctypes.c_int32)),
        ("vocab_size", ctypes.c_int32),
        ("rms_norm_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("partial_rotary_factor", ctypes.c_float),
        ("max_seq_len", ctypes.c_int32),
        ("head_width", ctypes.c_int32),
        ("head_heads", ctypes.c_int32),
        ("head_routing_layers", ctypes.c_int32),
        ("head_layers", ctypes.c_int32),
        ("head_ffn", ctypes.c_int32),
        ("attn_softcap", ctypes.c_float),
        ("layer_window", ctypes.POINTER(ctypes.c_int32)),
        ("embed_scale", ctypes.c_float),
        ("linear_num_key_heads", ctypes.c_int32),
        ("linear_num_value_heads", ctypes.c_int32),
        ("linear_key_head_dim", ctypes.c_int32),
        ("linear_value_head_dim", ctypes.c_int32),
        ("linear_conv_kernel_dim", ctypes.c_int32),
        ("tp_timeout_ms", ctypes.c_int32),
    ]


class ClefBatchC(ctypes.Structure):
    _fields_ = [
        ("b", ctypes.c_int32),
        ("s", ctypes.c_int32),
        ("lx", ctypes.c_int32),
        ("o", ctypes.c_int32),
        ("q", ctypes.c_int32),
        ("input_ids", ctypes.c_void_p),
        ("mask", ctypes.c_void_p),
        ("lexical_ids", ctypes.c_void_p),
        ("lexical_spans", ctypes.c_void_p),
        ("question_spans", ctypes.c_void_p),
        ("question_mask", ctypes.c_void_p),
        ("types", ctypes.c_void_p),
        ("option_spans", ctypes.c_void_p),
        ("option_mask", ctypes.c_void_p),
        ("option_field", ctypes.c_void_p),
    ]


BATCH_KEYS = (
    "input_ids",
    "mask",
    "lexical_ids",
    "lexical_spans",
    "question_spans",
    "question_mask",
    "types",
    "option_spans",
    "option_mask",
    "option_field",
)


class ClefError(RuntimeError):
    """A CUDA, NCCL or device-side failure inside the library."""


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the shared library, declaring every entry point's signature."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built; run `python -m deciax_b200.build`")
        lib = ctypes.CDLL(str(LIB_PATH))
        vp, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        sigs = {
            "clef_nccl_unique_id": [ctypes.c_char_p],
            "clef_create": [ctypes.POINTER(ClefConfigC), i32, i32, i32, ctypes.c_char_p, i32, ctypes.POINTER(vp)],
            "clef_upload": [vp, ctypes.c_char_p, vp, i32, ctypes.POINTER(ctypes.c_int64), i32],
            "clef_upload_device": [vp, ctypes.c_char_p, vp, i32, ctypes.POINTER(ctypes.c_int64), i32],
            "clef_set_timing": [vp, i32],
            "clef_set_debug": [vp, i32],
            "clef_timing_report": [vp, i32, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_int)],
            "clef_finalize": [vp],
            "clef_forward": [vp, ctypes.POINTER(ClefBatchC), vp, vp],
            "clef_forward_head": [vp, ctypes.POINTER(ClefBatchC), vp, vp],
            "clef_forward_device": [vp, ctypes.POINTER(ClefBatchC), vp, vp],
            "clef_reserve": [vp, i32, i32, i32, i32, i32],
            "clef_workspace_allocations": [vp, ctypes.POINTER(ctypes.c_int64)],
            "clef_check_status": [vp],
            "clef_last_launch_count": [vp],
            "clef_destroy": [vp],
            "clef_op_gemm": [i32, i32, i32, i32, i32, vp, vp, vp, i32, vp, vp, i32, vp],
            "clef_op_gemm_qkv": [vp, vp, vp, i32, i32, i32, i32, i32, f32, f32, i32, vp, vp, f32, vp],
            "clef_op_rmsnorm": [i32, vp, vp, vp, i32, i32, f32, vp],
            "clef_op_qk_norm_rope": [i32, vp, i32, i32, i32, i32, i32, f32, f32, vp, vp, f32, vp],
            "clef_op_qk_norm_rope_noalloc": [i32, vp, i32, i32, i32, i32, i32, f32, f32, vp, vp, f32, vp],
            "clef_op_attention": [i32, vp, vp, vp, i32, i32, i32, i32, i32, f32, i32, vp],
            "clef_op_gdn_core": [i32, vp, i32, vp, i32, vp, vp, vp, vp, i32, i32, i32, i32, i32, f32, vp],
        }
        for name, args in sigs.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        lib.clef_last_error.argtypes = [vp]
        lib.clef_last_error.restype = ctypes.c_char_p
        _lib = lib
        return lib


def check(status: int, handle=None) -> None:
    """Map a CLEF_E* status to the reference's exception types.

    CLEF_EINVAL -> ValueError (the server's 422, serve/app.py:259-260);
    everything else -> ClefError, a RuntimeError (500).
    """
    if status == CLEF_OK:
        return
    msg = load().clef_last_error(handle).decode(errors="replace")
    if status == CLEF_EINVAL:
        raise ValueError(msg)
    raise ClefError(f"clef status {status}: {msg}")
