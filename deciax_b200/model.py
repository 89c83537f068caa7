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
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import ml_dtypes
import numpy as np

from deciax_b200 import _lib
from deciax_b200.clef_input import (MAX_QUESTIONS, MAX_TOKENS, MAX_TOTAL_OPTIONS, ROW_BUCKETS, SCHEMA_BUCKETS,
                                    SEQUENCE_BUCKETS, bucket)
from deciax_b200.config import HeadConfig, KernelFlags, TextConfig
from deciax_b200.engine import DEFAULT_BATCH_TOKENS

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
        model*.safetensors with their index, joint_head_config.json,
        joint_head.safetensors) as ``ClefModel.__init__`` does
        (models/clef/model.py:51-85, weights.py:70-101).  The directory is
        validated on the host first (``read_checkpoint``); the library then
        keeps each tensor's tensor-parallel shard as it arrives, splitting the
        Gated DeltaNet layers' fused ``in_proj_qkv`` / ``conv1d`` tensors."""
        plan = read_checkpoint(path)
        m = cls(plan.config, plan.head_config, dtype=dtype, name=name, tokenizer=plan.tokenizer,
                pad_token_id=plan.pad_token_id, **kwargs)
        for filename, names in plan.backbone.items():
            for key, value in safetensors_tensors(filename):
                if key in names:
                    m.upload(names[key], value)
        for key, value in safetensors_tensors(plan.head_file):
            m.upload("head." + key, value)
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

    def warmup(self, max_batch_tokens: int = DEFAULT_BATCH_TOKENS, max_rows: int = ROW_BUCKETS[-1],
               max_options: int = MAX_TOTAL_OPTIONS, max_questions: int = MAX_QUESTIONS) -> None:
        """Reserve the workspace for every batch a ``ClefEngine`` can form
        under these limits, so that no later forward allocates (device
        buffers, pinned staging, or -- under TP, where every rank must call
        this with the same limits -- the exchange of peer-memory handles).

        The engine's batches hold at most ``max_rows`` records padded to at
        most ``max_token_budget`` tokens, with rows x padded length within
        ``max_batch_tokens``; options and questions are bounded by the
        protocol's limits (protocol/systemone.py:17,22).  Every workspace
        term grows with one of rows x length, rows x options, rows x
        questions or rows x lexical tokens (at most rows x length), so two
        reservations cover them all: the longest records at the most rows
        the token budget allows, and the most rows at the length the budget
        then allows.  The reference server's warm-up request
        (serve/app.py:385-406) compiles one small shape; this reserves the
        whole admitted range."""
        s_max = self.max_token_budget
        o = bucket(max_options, SCHEMA_BUCKETS)
        q = bucket(max_questions, SCHEMA_BUCKETS)
        long_rows = max(1, min(max_rows, max_batch_tokens // s_max))
        many_seq = max(1, min(s_max, max_batch_tokens // max_rows))
        for b, s in ((long_rows, s_max), (max_rows, many_seq)):
            self.reserve(b, s, bucket(s, SEQUENCE_BUCKETS), o, q)

    @property
    def workspace_allocations(self) -> int:
        """Workspace growths since creation (see ``clef_workspace_allocations``)."""
        n = ctypes.c_int64()
        _lib.check(self._lib.clef_workspace_allocations(self._handle, ctypes.byref(n)), self._handle)
        return int(n.value)

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


SAFETENSORS_TYPES = {"BF16": ml_dtypes.bfloat16, "F32": np.float32, "F16": np.float16}


def safetensors_header(path: Path) -> tuple[int, dict[str, Any]]:
    """(header length, {name: {dtype, shape, data_offsets}}) of a safetensors
    file, checked the way the reference has ``safe_open`` check it before
    mapping (weights.py:26-31): a supported dtype, offsets inside the data
    section and a byte size that matches the shape."""
    path = Path(path)
    total = path.stat().st_size
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise ValueError(f"{path.name}: not a safetensors file")
        size = struct.unpack("<Q", raw)[0]
        if 8 + size > total:
            raise ValueError(f"{path.name}: header runs past the end of the file")
        try:
            header = json.loads(f.read(size))
        except json.JSONDecodeError as e:
            raise ValueError(f"{path.name}: unreadable header ({e})") from None
    data = total - 8 - size
    for key, entry in header.items():
        if key == "__metadata__":
            continue
        if entry.get("dtype") not in SAFETENSORS_TYPES:
            raise ValueError(f"{path.name}: {key} has unsupported dtype {entry.get('dtype')!r}")
        start, end = entry["data_offsets"]
        nbytes = int(np.prod(entry["shape"], dtype=np.int64)) * np.dtype(SAFETENSORS_TYPES[entry["dtype"]]).itemsize
        if not 0 <= start <= end <= data or end - start != nbytes:
            raise ValueError(f"{path.name}: {key} has invalid data offsets")
    return size, header


def safetensors_tensors(path: Path):
    """Yield (name, array) from a safetensors file via memmap; BF16 as ml_dtypes
    (models/clef/weights.py:26-40).

    The file format is an 8-byte little-endian header length, a JSON header
    of {name: {dtype, shape, data_offsets}}, then the raw data.
    """
    size, header = safetensors_header(path)
    for key, entry in header.items():
        if key == "__metadata__":
            continue
        start, _ = entry["data_offsets"]
        arr = np.memmap(path, mode="r", dtype=SAFETENSORS_TYPES[entry["dtype"]], offset=8 + size + start,
                        shape=tuple(entry["shape"]))
        if entry["dtype"] == "F16":
            arr = np.asarray(arr, np.float32)
        yield key, arr


@dataclass(frozen=True)
class CheckpointPlan:
    """What ``from_pretrained`` will load, read from headers only."""

    config: TextConfig
    head_config: HeadConfig
    tokenizer: Any
    pad_token_id: int
    backbone: dict[Path, dict[str, str]]  # shard file -> {checkpoint key: library upload name}
    head_file: Path


def backbone_name(key: str, num_layers: int) -> str | None:
    """The library's upload name for a backbone checkpoint key, or None for a
    key the reference skips (the vision tower); the renames of
    models/clef/weights.py:43-45,84-93.  Gated DeltaNet layers keep their
    fused ``in_proj_qkv`` / ``conv1d`` names: the library splits them into the
    q, k, v parts of weights.py:46-55 as it shards."""
    if key.startswith("model.visual."):
        return None
    if key == "lm_head.weight":
        return "lm_head"
    if key == "model.language_model.embed_tokens.weight":
        return "embedding"
    if key == "model.language_model.norm.weight":
        return "norm"
    if key.startswith("model.language_model.layers."):
        parts = key.split(".", 4)
        if len(parts) == 5 and parts[3].isdigit() and int(parts[3]) < num_layers:
            rest = parts[4].replace("linear_attn.", "mixer.").replace("self_attn.", "mixer.")
            return f"layers.{int(parts[3])}.{rest}"
    raise ValueError(f"unexpected backbone tensor: {key}")


def read_checkpoint(path: str | Path) -> CheckpointPlan:
    """Validate a Clef checkpoint directory on the host, before any device
    work, with the reference's rejections (models/clef/model.py:51-57,
    weights.py:70-101): the ``config.json`` checks of ``TextConfig.from_dict``,
    a tokenizer without ``<|endoftext|>`` ("missing pad token"), an unexpected
    backbone key, and a text checkpoint without its embedding, lm_head, final
    norm or any tensor of some layer ("incomplete Clef text checkpoint")."""
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
    n = len(config.layer_types)
    index = json.loads((path / "model.safetensors.index.json").read_text())["weight_map"]
    backbone: dict[Path, dict[str, str]] = {}
    top, layers = set(), [0] * n
    for filename in sorted(set(index.values())):
        names = backbone.setdefault(path / filename, {})
        for key in safetensors_header(path / filename)[1]:
            if key == "__metadata__":
                continue
            upload = backbone_name(key, n)
            if upload is None:
                continue
            names[key] = upload
            if upload.startswith("layers."):
                layers[int(upload.split(".")[1])] += 1
            else:
                top.add(upload)
    if top != {"lm_head", "embedding", "norm"} or not all(layers):
        raise ValueError("incomplete Clef text checkpoint")
    head_cfg = json.loads((path / "joint_head_config.json").read_text())
    head_file = path / "joint_head.safetensors"
    shapes = {k: v["shape"] for k, v in safetensors_header(head_file)[1].items() if k != "__metadata__"}
    if "memory_projection.weight" not in shapes:
        raise ValueError("missing joint head tensor: memory_projection.weight")
    ffn_key = "evidence_layers.0.feedforward.0.weight" if head_cfg["routing_layers"] else "layers.0.linear1.weight"
    if ffn_key not in shapes:
        raise ValueError(f"missing joint head tensor: {ffn_key}")
    hc = HeadConfig(heads=head_cfg["heads"], routing_layers=head_cfg["routing_layers"], layers=head_cfg["layers"],
                    width=int(shapes["memory_projection.weight"][0]), ffn=int(shapes[ffn_key][0]))
    return CheckpointPlan(config, hc, tokenizer, pad_id, backbone, head_file)
