"""``ClefCudaModel``: the ``impl="cuda"`` counterpart of the reference ``ClefModel``.

Mirrors ``src/deciax/models/clef/model.py:30-102``: the same attributes used
by callers (``name``, ``tokenizer``, ``pad_token_id``, ``max_token_budget``,
``build_engine()``) and ``forward(arrays) -> [b, o] float32`` over the dict
``collate`` returns.  Every step of the forward runs inside
``libclef_b200.so``; this module only moves host arrays across the C ABI.
"""

from __future__ import annotations

import ctypes
import json
import struct
from collections.abc import Mapping, Sequence
from pathlib import Path
from typing import Any

import ml_dtypes
import numpy as np

from deciax_b200 import _lib
from deciax_b200.clef_input import MAX_TOKENS, SEQUENCE_BUCKETS
from deciax_b200.config import HeadConfig, KernelFlags, TextConfig

INT_KEYS = ("input_ids", "lexical_ids", "lexical_spans", "question_spans", "types", "option_spans", "option_field")
BOOL_KEYS = ("mask", "question_mask", "option_mask")


def _host_tensor(array: Any) -> tuple[np.ndarray, int]:
    """A C-contiguous host array and its CLEF_DTYPE (bf16 is passed as raw bits)."""
    a = np.asarray(array)
    if a.dtype == ml_dtypes.bfloat16:
        return np.ascontiguousarray(a).view(np.uint16), _lib.DTYPE_BF16
    return np.ascontiguousarray(a, dtype=np.float32), _lib.DTYPE_F32


def batch_struct(arrays: Mapping[str, Any], keep: list) -> _lib.ClefBatchC:
    """ClefBatch over host numpy arrays (kept alive through ``keep``)."""
    ids = np.ascontiguousarray(arrays["input_ids"], np.int32)
    b, s = ids.shape
    lx = np.asarray(arrays["lexical_ids"]).shape[1]
    o = np.asarray(arrays["option_mask"]).shape[1]
    q = np.asarray(arrays["question_mask"]).shape[1]
    expect = {
        "input_ids": (b, s), "mask": (b, s), "lexical_ids": (b, lx), "lexical_spans": (b, o, 2),
        "question_spans": (b, q, 2), "question_mask": (b, q), "types": (b, q), "option_spans": (b, o, 2),
        "option_mask": (b, o), "option_field": (b, o),
    }
    c = _lib.ClefBatchC(b=b, s=s, lx=lx, o=o, q=q)
    for key in _lib.BATCH_KEYS:
        if key in BOOL_KEYS:
            a = np.ascontiguousarray(np.asarray(arrays[key]).astype(np.uint8))
        else:
            a = np.ascontiguousarray(arrays[key], np.int32)
        if a.shape != expect[key]:
            raise ValueError(f"{key}: expected shape {expect[key]}, got {a.shape}")
        keep.append(a)
        setattr(c, key, a.ctypes.data)
    return c


class ClefCudaModel:
    """One Clef model on one GPU (one tensor-parallel rank)."""

    max_token_budget = MAX_TOKENS

    def __init__(
        self,
        config: TextConfig,
        head_config: HeadConfig,
        *,
        dtype: str = "bf16",
        device: int = 0,
        tp_rank: int = 0,
        tp_size: int = 1,
        nccl_id: bytes | None = None,
        max_seq_len: int = MAX_TOKENS,
        flags: KernelFlags = KernelFlags(),
        name: str = "clef",
        tokenizer: Any = None,
        pad_token_id: int = 0,
        tp_timeout: float = 300.0,
        heartbeat: Any = None,
    ) -> None:
        """``tp_timeout`` (seconds, 0 = no limit) bounds the library's host
        waits for the other TP ranks: communicator creation and each host
        forward.  ``heartbeat`` (a ``TpHeartbeat``) makes each forward check
        in with the other ranks before launching anything."""
        if dtype not in ("bf16", "fp32"):
            raise ValueError("Clef CUDA dtype must be 'bf16' or 'fp32'")
        if not config.vocab_size:
            raise ValueError("TextConfig.vocab_size is required by the CUDA implementation")
        self.name = name
        self.config = config
        self.head_config = head_config
        self.dtype = dtype
        self.device = device
        self.tokenizer = tokenizer
        self.pad_token_id = pad_token_id
        self.heartbeat = heartbeat
        # records are encoded so that their sequence bucket fits the library's max_seq_len
        fits = [b for b in SEQUENCE_BUCKETS if b <= max_seq_len]
        self.max_token_budget = fits[-1] if fits else max_seq_len
        self._lib = _lib.load()
        n = len(config.layer_types)
        self._types = (ctypes.c_int32 * n)(*[_lib.LAYER_LINEAR if t == "linear_attention" else _lib.LAYER_FULL for t in config.layer_types])
        window = list(flags.layer_window) or [0] * n
        if len(window) != n:
            raise ValueError("layer_window needs one entry per layer")
        self._window = (ctypes.c_int32 * n)(*window)
        cfg = _lib.ClefConfigC(
            hidden_size=config.hidden_size,
            intermediate_size=config.intermediate_size,
            num_attention_heads=config.num_attention_heads,
            num_key_value_heads=config.num_key_value_heads,
            head_dim=config.head_dim,
            num_layers=n,
            layer_types=self._types,
            vocab_size=config.vocab_size,
            rms_norm_eps=config.rms_norm_eps,
            rope_theta=config.rope_theta,
            partial_rotary_factor=config.partial_rotary_factor,
            max_seq_len=max_seq_len,
            head_width=head_config.width,
            head_heads=head_config.heads,
            head_routing_layers=head_config.routing_layers,
            head_layers=head_config.layers,
            head_ffn=head_config.ffn,
            attn_softcap=flags.attn_softcap,
            layer_window=self._window,
            embed_scale=flags.embed_scale,
            linear_num_key_heads=config.linear_num_key_heads,
            linear_num_value_heads=config.linear_num_value_heads,
            linear_key_head_dim=config.linear_key_head_dim,
            linear_value_head_dim=config.linear_value_head_dim,
            linear_conv_kernel_dim=config.linear_conv_kernel_dim,
            tp_timeout_ms=int(round(tp_timeout * 1000)),
        )
        handle = ctypes.c_void_p()
        dt = _lib.DTYPE_BF16 if dtype == "bf16" else _lib.DTYPE_F32
        status = self._lib.clef_create(ctypes.byref(cfg), device, tp_rank, tp_size, nccl_id, dt, ctypes.byref(handle))
        _lib.check(status, None)
        self._handle = handle

    # ------------------------------------------------------------------ weights

    def upload(self, name: str, array: Any) -> None:
        a, dt = _host_tensor(array)
        shape = (ctypes.c_int64 * max(a.ndim, 1))(*a.shape)
        _lib.check(self._lib.clef_upload(self._handle, name.encode(), a.ctypes.data, dt, shape, a.ndim), self._handle)

    def upload_device(self, name: str, tensor: Any) -> None:
        """Upload from a CUDA tensor on this model's GPU, already in the compute dtype."""
        import torch

        want = torch.bfloat16 if self.dtype == "bf16" else torch.float32
        if tensor.dtype != want or not tensor.is_cuda or not tensor.is_contiguous():
            raise ValueError(f"{name}: device uploads need a contiguous CUDA {want} tensor")
        shape = (ctypes.c_int64 * max(tensor.dim(), 1))(*tensor.shape)
        dt = _lib.DTYPE_BF16 if self.dtype == "bf16" else _lib.DTYPE_F32
        _lib.check(self._lib.clef_upload_device(self._handle, name.encode(), tensor.data_ptr(), dt, shape, tensor.dim()), self._handle)

    def finalize(self) -> None:
        _lib.check(self._lib.clef_finalize(self._handle), self._handle)

    TIMING_CATEGORIES = ("embed", "rmsnorm", "gemm_qkv", "qk_norm_rope", "attention", "gemm_o", "gemm_gate_up", "gemm_down",
                         "allreduce", "residual_add", "head", "other", "gdn")

    def set_timing(self, enable: bool) -> None:
        _lib.check(self._lib.clef_set_timing(self._handle, int(enable)), self._handle)

    def set_debug(self, poison: bool = False) -> None:
        """Debug switches: ``poison`` fills the forward's scratch buffers with
        NaN bytes before every forward (reads of unwritten memory show up)."""
        _lib.check(self._lib.clef_set_debug(self._handle, _lib.DEBUG_POISON if poison else 0), self._handle)

    def timing_report(self) -> dict[str, tuple[float, int]]:
        """{category: (device ms, launches)} since the last report (see include/clef_b200.h)."""
        n = len(self.TIMING_CATEGORIES)
        ms = (ctypes.c_float * n)()
        cnt = (ctypes.c_int * n)()
        _lib.check(self._lib.clef_timing_report(self._handle, n, ms, cnt), self._handle)
        return {c: (float(ms[i]), int(cnt[i])) for i, c in enumerate(self.TIMING_CATEGORIES)}

    @classmethod
    def from_arrays(
        cls,
        config: TextConfig,
        head_config: HeadConfig,
        top: Mapping[str, Any],
        layers: Sequence[Mapping[str, Any]],
        head: Mapping[str, Any],
        **kwargs: Any,
    ) -> "ClefCudaModel":
        """Build from in-memory weights: ``top`` (embedding, lm_head, norm),
        per-layer dicts keyed as after ``weights.layer_weights`` renames
        (``mixer.q_proj.weight`` ...), and the joint-head state dict."""
        m = cls(config, head_config, **kwargs)
        for k in ("embedding", "lm_head", "norm"):
            m.upload(k, top[k])
        for i, p in enumerate(layers):
            for k, v in p.items():
                m.upload(f"layers.{i}.{k}", v)
        for k, v in head.items():
            m.upload("head." + k, v)
        m.finalize()
        return m

    @classmethod
    def from_pretrained(cls, path: str | Path, dtype: str = "bf16", name: str = "clef", **kwargs: Any) -> "ClefCudaModel":
        """Load a Clef checkpoint directory (config.json, tokenizer.json,
        model*.safetensors, joint_head_config.json, joint_head.safetensors) as
        ``ClefModel.__init__`` does (models/clef/model.py:51-85, weights.py:70-101)."""
        from tokenizers import Tokenizer

        path = Path(path)
        raw = json.loads((path / "config.json").read_text())
        config = TextConfig.from_dict(raw)
        if not config.vocab_size:
            config = TextConfig(**{**config.__dict__, "vocab_size": int(raw.get("text_config", raw)["vocab_size"])})
        tokenizer = Tokenizer.from_file(str(path / "tokenizer.json"))
        pad_id = tokenizer.token_to_id("<|endoftext|>")
        if pad_id is None:
            raise ValueError("missing pad token")
        head_cfg = json.loads((path / "joint_head_config.json").read_text())
        head = dict(safetensors_tensors(path / "joint_head.safetensors"))
        hc = HeadConfig(
            heads=head_cfg["heads"],
            routing_layers=head_cfg["routing_layers"],
            layers=head_cfg["layers"],
            width=int(head["memory_projection.weight"].shape[0]),
            ffn=int(head["evidence_layers.0.feedforward.0.weight"].shape[0]) if head_cfg["routing_layers"] else int(head["layers.0.linear1.weight"].shape[0]),
        )
        m = cls(config, hc, dtype=dtype, name=name, tokenizer=tokenizer, pad_token_id=pad_id, **kwargs)
        index = json.loads((path / "model.safetensors.index.json").read_text())["weight_map"]
        for filename in sorted(set(index.values())):
            for key, value in safetensors_tensors(path / filename):
                if key.startswith("model.visual."):
                    continue
                if key == "lm_head.weight":
                    m.upload("lm_head", value)
                elif key == "model.language_model.embed_tokens.weight":
                    m.upload("embedding", value)
                elif key == "model.language_model.norm.weight":
                    m.upload("norm", value)
                elif key.startswith("model.language_model.layers."):
                    _, _, _, number, rest = key.split(".", 4)
                    rest = rest.replace("linear_attn.", "mixer.").replace("self_attn.", "mixer.")
                    m.upload(f"layers.{number}.{rest}", value)
                else:
                    raise ValueError(f"unexpected backbone tensor: {key}")
        for k, v in head.items():
            m.upload("head." + k, v)
        m.finalize()
        return m

    # ------------------------------------------------------------------ forward

    def forward(self, arrays: Mapping[str, Any]) -> np.ndarray:
        """Option logits [b, o] float32 for one collated batch (model.py:92-102)."""
        return self._forward(arrays, hidden=False)[0]

    def forward_with_hidden(self, arrays: Mapping[str, Any]) -> tuple[np.ndarray, np.ndarray]:
        """Logits and the final-normed hidden states [b, s, hidden] (float32)."""
        logits, hidden = self._forward(arrays, hidden=True)
        assert hidden is not None
        return logits, hidden

    def forward_head(self, arrays: Mapping[str, Any], hidden: Any) -> np.ndarray:
        """Lexical means + joint head on given final-normed hidden states [b, s, D]."""
        keep: list = []
        c = batch_struct(arrays, keep)
        h = np.ascontiguousarray(hidden, np.float32)
        if h.shape != (c.b, c.s, self.config.hidden_size):
            raise ValueError(f"hidden must be [{c.b}, {c.s}, {self.config.hidden_size}], got {h.shape}")
        out = np.empty((c.b, c.o), np.float32)
        _lib.check(self._lib.clef_forward_head(self._handle, ctypes.byref(c), h.ctypes.data, out.ctypes.data), self._handle)
        return out

    def _forward(self, arrays: Mapping[str, Any], hidden: bool) -> tuple[np.ndarray, np.ndarray | None]:
        keep: list = []
        try:
            c = batch_struct(arrays, keep)
        except Exception as e:
            self.report_failure(e)
            raise
        out = np.empty((c.b, c.o), np.float32)
        hid = np.empty((c.b, c.s, self.config.hidden_size), np.float32) if hidden else None
        if self.heartbeat is not None:
            self.heartbeat.arrive()
        status = self._lib.clef_forward(self._handle, ctypes.byref(c), out.ctypes.data, hid.ctypes.data if hid is not None else None)
        if status != _lib.CLEF_OK:
            self.report_failure(RuntimeError(f"clef_forward status {status}"))
        _lib.check(status, self._handle)
        return out, hid

    def report_failure(self, e: BaseException) -> None:
        """Tell the other TP ranks (through the heartbeat) that this rank's
        next forward will not come."""
        if self.heartbeat is not None:
            self.heartbeat.fail(f"{type(e).__name__}: {e}")

    def forward_device(self, tensors: Mapping[str, Any], out: Any, stream: int | None = None) -> None:
        """Enqueue a forward over device-resident tensors (torch CUDA tensors:
        int32 arrays, uint8 masks) writing float32 logits into ``out``."""
        ids = tensors["input_ids"]
        c = _lib.ClefBatchC(
            b=ids.shape[0], s=ids.shape[1], lx=tensors["lexical_ids"].shape[1], o=tensors["option_mask"].shape[1],
            q=tensors["question_mask"].shape[1],
        )
        for key in _lib.BATCH_KEYS:
            setattr(c, key, tensors[key].data_ptr())
        if self.heartbeat is not None:
            self.heartbeat.arrive()
        status = self._lib.clef_forward_device(self._handle, ctypes.byref(c), out.data_ptr(), stream)
        _lib.check(status, self._handle)

    def reserve(self, b: int, s: int, lx: int, o: int, q: int) -> None:
        _lib.check(self._lib.clef_reserve(self._handle, b, s, lx, o, q), self._handle)

    def check_status(self) -> None:
        _lib.check(self._lib.clef_check_status(self._handle), self._handle)

    @property
    def last_launch_count(self) -> int:
        return int(self._lib.clef_last_launch_count(self._handle))

    def build_engine(self):
        from deciax_b200.engine import ClefEngine

        return ClefEngine(self)

    def close(self) -> None:
        if getattr(self, "_handle", None):
            self._lib.clef_destroy(self._handle)
            self._handle = None

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


def safetensors_tensors(path: Path):
    """Yield (name, array) from a safetensors file via memmap; BF16 as ml_dtypes.

    The file format is an 8-byte little-endian header length, a JSON header
    of {name: {dtype, shape, data_offsets}}, then the raw data.
    """
    with open(path, "rb") as f:
        size = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(size))
    types = {"BF16": ml_dtypes.bfloat16, "F32": np.float32, "F16": np.float16}
    for key, entry in header.items():
        if key == "__metadata__":
            continue
        start, end = entry["data_offsets"]
        arr = np.memmap(path, mode="r", dtype=types[entry["dtype"]], offset=8 + size + start, shape=tuple(entry["shape"]))
        if entry["dtype"] == "F16":
            arr = np.asarray(arr, np.float32)
        yield key, arr
