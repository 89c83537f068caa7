"""Clef prefill-and-score benchmark on B200 (the BASELINE ``configs[1]`` workload).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Workload ("cfg2"): a clef-flash-shaped model -- 42 full-attention Qwen3.5
layers, hidden 3584, 16 query / 8 key-value heads of 256, gated-MLP 14336,
vocab 256000, lm_head = a copy of the embedding -- in BF16 with random
N(0, 0.02) weights (seed 1), and the joint schema head (width 256, 4 heads,
2 routing + 2 field layers; its real dims are not published).  One step is
one full forward of 8 states x 2048 tokens (uniform token ids) carrying 4
choice questions x 4 options each, from token ids to option logits.

Output: one JSON line.  ``value`` = prefill tokens/s with the batch already
resident in HBM, timed with CUDA events on the launching stream over exactly
K steps (max over ranks).  ``e2e`` = the same metric through the public host
API (``ClefCudaModel.forward`` -> ``clef_forward``), which copies the collated
host arrays in and the logits out every step.  ``roofline`` = the dominant
kernel (the gate/up GEMM with the fused SwiGLU epilogue) timed live by CUDA
events inside the timed region.  ``cpu_baseline`` = the CPU oracle (FP32,
the reference's impl="auto" arithmetic) on a bounded sample, extrapolated.

With torchrun (N > 1) every rank holds a full replica and runs its own batch
(data parallel, no collective on the data path): ``value`` scales "weak".
The same line then carries ``tp``: cfg2 tensor-parallel over the N ranks
(heads and MLP columns sharded, FP32 partials of o-proj and down-proj summed
over NVLink peer memory), one shared batch per step (strong scaling), with
its per-category device time split into GEMM, attention, reduction and
barrier; and ``tp_parity``: a TP=N check of small sharded models against the
CPU oracle, run before anything is timed.  At N = 1 the line carries
``parity``: a two-layer slice of the cfg2 model (same dims, BF16, one
2048-token state) against the CPU oracle, also outside the timed region.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "prefill tokens/s and decisions/s, clef-flash/clef BF16, 1/2/4/8 B200"
UNIT = "tokens/s"
CFG2 = dict(hidden_size=3584, intermediate_size=14336, num_attention_heads=16, num_key_value_heads=8, head_dim=256,
            num_layers=42, vocab_size=256000)
HEAD = dict(heads=4, routing_layers=2, layers=2, width=256, ffn=512)
STATES, SEQ, QUESTIONS, OPTIONS = 8, 2048, 4, 4
WEIGHT_SEED, WEIGHT_STD = 1, 0.02


def workload_config(n_gpus: int) -> dict:
    return {
        "workload": "cfg2: clef-flash-shaped prefill+scoring, 42 full-attention layers (D3584, 16q/8kv x256, F14336, "
        "V256000), joint head W256/4 heads/2+2 layers; 8 states x 2048 tokens, 4 choice x 4 options per state",
        "model": "clef-flash-shaped, random init N(0,0.02) seed 1",
        "global_batch": STATES * n_gpus,
        "seq_len": SEQ,
        "parallelism": f"dp{n_gpus}" if n_gpus > 1 else "single",
        "l2": "inputs larger than L2: every step streams 21 GB of weights and >1 GB of activations",
    }


def algorithmic_flops(c, lengths) -> tuple[float, float, float]:
    """(linear FLOPs, attention FLOPs, gate/up FLOPs) for one batch, real tokens only."""
    D, F, hq, hkv, d, L = c["hidden_size"], c["intermediate_size"], c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"], c["num_layers"]
    tokens = sum(lengths)
    linear = 2.0 * D * (2 * hq * d + 2 * hkv * d + hq * d + 3 * F) * tokens * L
    attention = sum(2.0 * hq * d * n * (n + 1) for n in lengths) * L
    return linear, attention, 2.0 * D * 2 * F


def rank_reduce(value: float, op: str = "max") -> float:
    """``value`` reduced over the ranks of the default process group ("max" or
    "sum"; the value itself without one).  On the group's own device: CUDA
    for NCCL, the host for gloo."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return value
    device = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return float(t.item())


def share_from_rank0(make):
    """The object rank 0 builds with ``make()`` (e.g. an NCCL unique id), on every rank."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return make()
    obj = [make() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()) | {"source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------


class ClockSampler:
    FIELDS = ("clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.sw_power_cap",
              "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown")

    def __init__(self, device: int) -> None:
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={','.join(self.FIELDS)}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self) -> None:
        assert self.proc and self.proc.stdout
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc) -> None:
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) != len(self.FIELDS):
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), parts[3:]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ("sw_power_cap", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown")
        reasons = sorted({n for _, _, flags in rows for n, f in zip(names, flags) if f.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# model on the device
# ---------------------------------------------------------------------------


def build_model(device: int, max_seq_len: int = SEQ, cfg: dict | None = None, tp_rank: int = 0, tp_size: int = 1,
                nccl_id: bytes | None = None):
    """cfg2 (or ``cfg``) in BF16: backbone weights drawn on the GPU (torch RNG,
    the same full tensors on every tensor-parallel rank, which keeps its
    shard), head from NumPy."""
    import torch

    from deciax_b200.build import build as build_lib
    from deciax_b200.config import HeadConfig, TextConfig
    from deciax_b200.model import ClefCudaModel
    from deciax_b200.synthetic import synthetic_head_weights

    build_lib()
    cfg = cfg or CFG2
    config = TextConfig.full_attention(**cfg)
    head = HeadConfig(**HEAD)
    model = ClefCudaModel(config, head, dtype="bf16", device=device, max_seq_len=max_seq_len, tp_rank=tp_rank,
                          tp_size=tp_size, nccl_id=nccl_id)
    gen = torch.Generator(device=f"cuda:{device}")
    gen.manual_seed(WEIGHT_SEED)
    D, F, hq, hkv, d, V = (cfg[k] for k in ("hidden_size", "intermediate_size", "num_attention_heads", "num_key_value_heads", "head_dim", "vocab_size"))

    def randn(*shape):
        t = torch.empty(shape, dtype=torch.bfloat16, device=f"cuda:{device}")
        return t.normal_(0.0, WEIGHT_STD, generator=gen)

    emb = randn(V, D)
    model.upload_device("embedding", emb)
    model.upload_device("lm_head", emb)  # "tied" = the same array written twice
    del emb
    model.upload_device("norm", randn(D))
    shapes = {
        "input_layernorm.weight": (D,), "post_attention_layernorm.weight": (D,), "mixer.q_proj.weight": (hq * 2 * d, D),
        "mixer.k_proj.weight": (hkv * d, D), "mixer.v_proj.weight": (hkv * d, D), "mixer.o_proj.weight": (D, hq * d),
        "mixer.q_norm.weight": (d,), "mixer.k_norm.weight": (d,), "mlp.gate_proj.weight": (F, D),
        "mlp.up_proj.weight": (F, D), "mlp.down_proj.weight": (D, F),
    }
    for i in range(cfg["num_layers"]):
        for name, shape in shapes.items():
            model.upload_device(f"layers.{i}.{name}", randn(*shape))
    for k, v in synthetic_head_weights(D, head, seed=WEIGHT_SEED, std=WEIGHT_STD, dtype="bf16").items():
        model.upload("head." + k, v)
    model.finalize()
    torch.cuda.synchronize(device)
    return model


def make_batch(seed: int) -> dict[str, np.ndarray]:
    from deciax_b200.synthetic import BatchSpec, synthetic_batch

    return synthetic_batch(BatchSpec(states=STATES, seq=SEQ, questions=QUESTIONS, options_per_question=OPTIONS),
                           CFG2["vocab_size"], seed)


# ---------------------------------------------------------------------------
# parity checks outside the timed region (the CPU oracle is the checker)
# ---------------------------------------------------------------------------

PARITY_SEED = 11


def probability_agreement(actual: np.ndarray, expected: np.ndarray, arrays) -> tuple[float, int, int]:
    """(max abs option-probability error, fields whose argmax differs while the
    expected top-2 gap is at least 1e-3, fields compared): the north star's
    BF16 bar (probabilities within 1e-2, identical choices unless the
    reference's top-2 gap is below 1e-3), on the per-field softmax of
    models/clef/input.py:185-192."""
    from deciax_b200.synthetic import field_probabilities

    err, flips, fields = 0.0, 0, 0
    for fa, fe in zip(field_probabilities(actual, arrays), field_probabilities(expected, arrays)):
        for a, e in zip(fa, fe):
            fields += 1
            err = max(err, float(np.abs(a - e).max()))
            if a.argmax() != e.argmax():
                top = np.sort(e)[::-1]
                if len(top) < 2 or top[0] - top[1] >= 1e-3:
                    flips += 1
    return err, flips, fields


def cfg2_slice_parity(device: int, layers: int = 2, lengths: tuple[int, ...] = (SEQ,), seed: int = PARITY_SEED,
                      oracle_floor: bool = True) -> dict:
    """The CUDA forward against the CPU oracle on a slice of the bench
    workload: ``layers`` decoder layers at cfg2's dims (D3584, 16q/8kv x 256,
    F14336, V256000), BF16, the bench's joint head, states of ``lengths``
    real tokens in the 2048 bucket with 4 choice x 4 options each.

    Weights are drawn on the GPU as ``build_model`` draws them (torch RNG,
    N(0, 0.02)), uploaded, and copied back for the oracle; the oracle gets
    only the embedding rows the batch uses (ids remapped), which gathers the
    same vectors.  Runs outside any timed region.  With ``oracle_floor`` the
    oracle runs a second time with float64 accumulation in its linear layers;
    the probability distance between its two runs is reported beside the
    CUDA path's, as the drift expected between two faithful BF16
    implementations at these dims."""
    import torch

    from deciax_b200.config import HeadConfig, TextConfig
    from deciax_b200.model import ClefCudaModel
    from deciax_b200.synthetic import BatchSpec, synthetic_batch, synthetic_head_weights
    from oracle import clef_oracle as O

    t0 = time.perf_counter()
    cfg = dict(CFG2, num_layers=layers)
    config = TextConfig.full_attention(**cfg)
    head = HeadConfig(**HEAD)
    D, F, hq, hkv, d, V = (cfg[k] for k in ("hidden_size", "intermediate_size", "num_attention_heads", "num_key_value_heads", "head_dim", "vocab_size"))
    model = ClefCudaModel(config, head, dtype="bf16", device=device, max_seq_len=SEQ)
    gen = torch.Generator(device=f"cuda:{device}")
    gen.manual_seed(seed)

    def randn(*shape):
        return torch.empty(shape, dtype=torch.bfloat16, device=f"cuda:{device}").normal_(0.0, WEIGHT_STD, generator=gen)

    def host(t) -> np.ndarray:
        return t.float().cpu().numpy()

    arrays = synthetic_batch(BatchSpec(states=len(lengths), seq=SEQ, questions=QUESTIONS, options_per_question=OPTIONS,
                                       lengths=tuple(lengths)), V, seed)
    used = np.unique(np.concatenate([arrays["input_ids"].ravel(), arrays["lexical_ids"].ravel()]))
    emb = randn(V, D)
    model.upload_device("embedding", emb)
    model.upload_device("lm_head", emb)
    table = host(emb[torch.from_numpy(used.astype(np.int64)).to(emb.device)])
    del emb
    norm = randn(D)
    model.upload_device("norm", norm)
    top = {"embedding": table, "lm_head": table, "norm": host(norm)}
    shapes = {
        "input_layernorm.weight": (D,), "post_attention_layernorm.weight": (D,), "mixer.q_proj.weight": (hq * 2 * d, D),
        "mixer.k_proj.weight": (hkv * d, D), "mixer.v_proj.weight": (hkv * d, D), "mixer.o_proj.weight": (D, hq * d),
        "mixer.q_norm.weight": (d,), "mixer.k_norm.weight": (d,), "mlp.gate_proj.weight": (F, D),
        "mlp.up_proj.weight": (F, D), "mlp.down_proj.weight": (D, F),
    }
    host_layers = []
    for i in range(layers):
        p = {}
        for name, shape in shapes.items():
            w = randn(*shape)
            model.upload_device(f"layers.{i}.{name}", w)
            p[name] = host(w)
        host_layers.append(p)
    hp = synthetic_head_weights(D, head, seed=seed, std=WEIGHT_STD, dtype="bf16")
    for k, v in hp.items():
        model.upload("head." + k, v)
    model.finalize()
    logits, hidden = model.forward_with_hidden(arrays)
    model.close()
    torch.cuda.empty_cache()
    t1 = time.perf_counter()
    oracle_arrays = dict(arrays)
    oracle_arrays["input_ids"] = np.searchsorted(used, arrays["input_ids"]).astype(np.int32)
    oracle_arrays["lexical_ids"] = np.searchsorted(used, arrays["lexical_ids"]).astype(np.int32)
    oc = O.TextConfig(hidden_size=D, intermediate_size=F, num_attention_heads=hq, num_key_value_heads=hkv, head_dim=d,
                      layer_types=config.layer_types)
    hp32 = {k: np.asarray(v, np.float32) for k, v in hp.items()}
    expected, exp_hidden = O.forward(top, host_layers, hp32, oracle_arrays, oc,
                                     O.HeadConfig(heads=HEAD["heads"], routing_layers=HEAD["routing_layers"],
                                                  layers=HEAD["layers"]), "bf16", return_hidden=True)
    t2 = time.perf_counter()
    err, flips, fields = probability_agreement(logits, expected, arrays)
    valid = arrays["mask"]
    diff = np.abs(hidden[valid] - exp_hidden[valid]) / np.abs(exp_hidden[valid]).max()
    floor = None
    if oracle_floor:
        # the same restatement with float64 accumulation in every linear layer:
        # how far two faithful implementations drift apart on this case
        with O.matmul_accumulation(np.float64):
            alt = O.forward(top, host_layers, hp32, oracle_arrays, oc,
                            O.HeadConfig(heads=HEAD["heads"], routing_layers=HEAD["routing_layers"], layers=HEAD["layers"]),
                            "bf16")
        floor = probability_agreement(alt, expected, arrays)[0]
    return {
        "case": f"cfg2 dims, {layers} layers, BF16, {len(lengths)} state(s) of {list(lengths)} tokens (bucket {SEQ}), "
        f"{QUESTIONS} choice x {OPTIONS} options, weights seed {seed}",
        "max_prob_err": err, "argmax_flips": flips, "fields": fields, "prob_tol": 1e-2,
        "oracle_fp64_accumulation_prob_err": floor,
        "hidden_err_max_rel": float(diff.max()), "hidden_err_mean_rel": float(diff.mean()),
        "ok": bool(err < 1e-2 and flips == 0 and np.isfinite(logits[arrays["option_mask"]]).all()),
        "gpu_seconds": round(t1 - t0, 2), "oracle_seconds": round(t2 - t1, 2),
    }


# ---------------------------------------------------------------------------
# CPU baseline: the oracle (FP32) on a bounded sample
# ---------------------------------------------------------------------------


def cpu_sample(repeats: int = 1) -> dict:
    """One decoder layer + the joint head for one 2048-token state, FP32 NumPy,
    extrapolated to the 42-layer model: tokens/s = 2048 / (42 t_layer + t_head)."""
    from deciax_b200.config import HeadConfig
    from deciax_b200.synthetic import synthetic_head_weights
    from oracle import clef_oracle as O

    rng = np.random.default_rng(0)
    D, F, hq, hkv, d = (CFG2[k] for k in ("hidden_size", "intermediate_size", "num_attention_heads", "num_key_value_heads", "head_dim"))

    def n(*shape):
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(WEIGHT_STD)

    p = {"input_layernorm.weight": n(D), "post_attention_layernorm.weight": n(D), "mixer.q_proj.weight": n(hq * 2 * d, D),
         "mixer.k_proj.weight": n(hkv * d, D), "mixer.v_proj.weight": n(hkv * d, D), "mixer.o_proj.weight": n(D, hq * d),
         "mixer.q_norm.weight": n(d), "mixer.k_norm.weight": n(d), "mlp.gate_proj.weight": n(F, D),
         "mlp.up_proj.weight": n(F, D), "mlp.down_proj.weight": n(D, F)}
    c = O.TextConfig(hidden_size=D, intermediate_size=F, num_attention_heads=hq, num_key_value_heads=hkv, head_dim=d)
    hp = synthetic_head_weights(D, HeadConfig(**HEAD), seed=1)
    arrays = {k: v[:1] for k, v in make_batch(seed=0).items()}
    x = rng.standard_normal((1, SEQ, D), dtype=np.float32)
    lex = rng.standard_normal((1, arrays["option_mask"].shape[1], D), dtype=np.float32)
    t_layer = t_head = 0.0
    for _ in range(repeats):
        t0 = time.perf_counter()
        h = O.layer(p, x, arrays["mask"], c, linear_attention=False, dtype="fp32")
        t1 = time.perf_counter()
        O.head_forward(hp, h, lex, arrays, heads=HEAD["heads"], routing_layers=HEAD["routing_layers"], layers=HEAD["layers"], dtype="fp32")
        t2 = time.perf_counter()
        t_layer += t1 - t0
        t_head += t2 - t1
    t_layer /= repeats
    t_head /= repeats
    per_state = CFG2["num_layers"] * t_layer + t_head
    return {"value": SEQ / per_state, "unit": UNIT, "cores": len(os.sched_getaffinity(0)), "kind": "port",
            "sample": f"oracle FP32 NumPy: 1 decoder layer ({t_layer:.2f} s) + joint head ({t_head:.2f} s) on one "
            f"2048-token state, extrapolated to 42 layers ({per_state:.1f} s per state); embedding gather excluded",
            "seconds": t_layer + t_head}


def reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    for _ in range(args.warmup):
        cpu_sample()
    samples = [cpu_sample() for _ in range(args.steps)]
    value = statistics.mean(s["value"] for s in samples)
    cb = dict(samples[-1])
    cb["value"] = value
    cb.pop("seconds", None)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * statistics.mean(s["seconds"] for s in samples),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": workload_config(args.gpus), "cpu_baseline": cb,
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference CPU path = the NumPy restatement of deciax's impl=\"auto\" Clef forward (JAX is not installed)",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------


TP_PREFLIGHT_BATCH = dict(states=3, seq=256, questions=2, options_per_question=3, lengths=(256, 130, 40), row_bucket=4)


def tp_preflight_config(kind: str):
    """Small models that shard at TP = 2, 4 and 8 (16 query / 8 key-value
    heads; Gated DeltaNet 8 key / 16 value heads).  Intermediate 12288 makes
    the down-proj run the fused GEMM + peer reduction at every tp in BF16
    (K tp / (tp - 1) >= 1536), the o-proj fused at TP=2 and unfused at 4 and 8."""
    from deciax_b200.config import HeadConfig, TextConfig

    head = HeadConfig(heads=4, routing_layers=1, layers=1, width=64, ffn=128)
    dims = dict(hidden_size=1024, intermediate_size=12288, num_attention_heads=16, num_key_value_heads=8, head_dim=128)
    if kind == "mixed":
        return TextConfig(**dims, linear_num_key_heads=8, linear_num_value_heads=16, linear_key_head_dim=64,
                          linear_value_head_dim=64, linear_conv_kernel_dim=4,
                          layer_types=("linear_attention", "full_attention"), rms_norm_eps=1e-6, rope_theta=10000.0,
                          partial_rotary_factor=0.25, vocab_size=1000), head
    return TextConfig.full_attention(**dims, num_layers=2, vocab_size=1000), head


def tp_preflight(rank: int, world: int, local: int) -> dict | None:
    """TP = world parity before the timed region: each small model of
    ``tp_preflight_config`` in FP32 and BF16, sharded over the ranks, runs one
    forward of a ragged 3-state batch; rank 0 checks its logits and hidden
    states against the CPU oracle (FP32: hidden within 1e-4 relative, logits
    within 1e-4; BF16: option probabilities within 1e-2, no argmax flip)
    and that every rank ends with the same bits.  Returns the summary on
    rank 0, None elsewhere."""
    import torch.distributed as dist

    from deciax_b200.model import ClefCudaModel
    from deciax_b200.synthetic import BatchSpec, synthetic_batch, synthetic_weights

    cases, ok = {}, True
    for kind in ("full", "mixed"):
        for dtype in ("fp32", "bf16"):
            config, head = tp_preflight_config(kind)
            top, layers, hp = synthetic_weights(config, head, seed=5, embed_std=1.0, dtype=dtype)
            nccl_id = share_from_rank0(nccl_unique_id)
            model = ClefCudaModel.from_arrays(config, head, top, layers, hp, dtype=dtype, device=local, tp_rank=rank,
                                              tp_size=world, nccl_id=nccl_id, max_seq_len=256, tp_timeout=300.0)
            arrays = synthetic_batch(BatchSpec(**TP_PREFLIGHT_BATCH), config.vocab_size, seed=6)
            logits, hidden = model.forward_with_hidden(arrays)
            model.close()
            gathered = [None] * world
            dist.all_gather_object(gathered, (logits, hidden))
            if rank != 0:
                continue
            from oracle import clef_oracle as O

            f32 = lambda t: {k: np.asarray(v, np.float32) for k, v in t.items()}  # noqa: E731
            oc = O.TextConfig(
                hidden_size=config.hidden_size, intermediate_size=config.intermediate_size,
                num_attention_heads=config.num_attention_heads, num_key_value_heads=config.num_key_value_heads,
                head_dim=config.head_dim, layer_types=config.layer_types, linear_num_key_heads=config.linear_num_key_heads,
                linear_num_value_heads=config.linear_num_value_heads, linear_key_head_dim=config.linear_key_head_dim,
                linear_value_head_dim=config.linear_value_head_dim, linear_conv_kernel_dim=config.linear_conv_kernel_dim)
            exp_logits, exp_hidden = O.forward(f32(top), [f32(p) for p in layers], f32(hp), arrays, oc,
                                               O.HeadConfig(heads=head.heads, routing_layers=head.routing_layers,
                                                            layers=head.layers), dtype, return_hidden=True)
            valid, m = arrays["mask"], arrays["option_mask"]
            same = all(np.array_equal(g[0], logits) and np.array_equal(g[1][valid], hidden[valid]) for g in gathered)
            entry = {"ranks_identical": bool(same)}
            if dtype == "fp32":
                scale = float(np.abs(exp_hidden[valid]).max())
                h_ratio = float((np.abs(hidden[valid] - exp_hidden[valid]) / (1e-4 * scale + 1e-4 * np.abs(exp_hidden[valid]))).max())
                l_ratio = float((np.abs(logits[m] - exp_logits[m]) / (1e-4 + 1e-4 * np.abs(exp_logits[m]))).max())
                entry |= {"hidden_err_over_tol": h_ratio, "logit_err_over_tol": l_ratio, "tol": "rtol 1e-4, atol 1e-4 x max|h|"}
                entry["ok"] = bool(h_ratio <= 1 and l_ratio <= 1 and same)
            else:
                err, flips, fields = probability_agreement(logits, exp_logits, arrays)
                entry |= {"max_prob_err": err, "argmax_flips": flips, "fields": fields, "tol": 1e-2}
                entry["ok"] = bool(err < 1e-2 and flips == 0 and same)
            cases[f"{kind}-{dtype}"] = entry
            ok &= entry["ok"]
    if rank != 0:
        return None
    return {"tp": world, "case": "D1024, 16q/8kv x128, F12288, 2 layers (full: 2 full-attention; mixed: Gated DeltaNet "
            "8 key/16 value heads x64 + full attention); 3 states of 256/130/40 tokens in 4 rows", "cases": cases, "ok": ok}


def device_batch(arrays):
    """The collated arrays as CUDA tensors (int32; masks as uint8)."""
    import torch

    from deciax_b200 import _lib

    return {k: torch.from_numpy(np.ascontiguousarray(arrays[k]).astype(np.uint8 if arrays[k].dtype == bool else np.int32)).cuda()
            for k in _lib.BATCH_KEYS}


def timed_forwards(model, tensors, out, stream, steps: int, warmup: int, local: int, dist) -> tuple[float, dict, dict]:
    """W untimed forwards, then exactly K forwards between a barrier and a
    device synchronisation on both sides, timed with CUDA events on the
    launching stream (the library enqueues on it); returns (ms for the K
    forwards, per-category timeline, clocks sampled during them)."""
    import torch

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(warmup):
        model.forward_device(tensors, out, stream.cuda_stream)
    torch.cuda.synchronize()
    model.check_status()
    barrier()
    model.set_timing(True)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(steps):
            model.forward_device(tensors, out, stream.cuda_stream)
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    elapsed_ms = start.elapsed_time(end)
    timing = model.timing_report()
    model.set_timing(False)
    model.check_status()
    return elapsed_ms, timing, clocks.summary()


def tp_arm(args, rank: int, world: int, local: int, dist) -> dict:
    """cfg2 tensor-parallel over the ``world`` ranks (heads and MLP columns
    sharded, the o-proj and down-proj FP32 partials reduced over NVLink peer
    memory), every rank running the same 8 x 2048 batch: strong scaling, the
    group's tokens/s.  Returns the ``tp`` object of the bench line."""
    import torch

    from deciax_b200.synthetic import field_probabilities

    model = build_model(local, tp_rank=rank, tp_size=world, nccl_id=share_from_rank0(nccl_unique_id))
    arrays = make_batch(seed=100)
    tensors = device_batch(arrays)
    out = torch.empty(arrays["option_mask"].shape, dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    elapsed_ms, timing, clocks = timed_forwards(model, tensors, out, stream, args.steps, args.warmup, local, dist)
    logits = out.cpu().numpy()
    launches = model.last_launch_count * args.steps
    model.close()
    if not np.isfinite(logits[arrays["option_mask"]]).all():
        raise SystemExit("non-finite logits (tensor parallel)")
    ms = rank_reduce(elapsed_ms, "max") / args.steps
    tokens = STATES * SEQ
    linear, attention, _ = algorithmic_flops(CFG2, [SEQ] * STATES)
    peaks = measured_peaks()
    per = {k: ms_ / args.steps for k, (ms_, n) in timing.items() if n}
    gemm = sum(per.get(k, 0.0) for k in ("gemm_qkv", "gemm_o", "gemm_gate_up", "gemm_down"))
    decisions = sum(len(f) for f in field_probabilities(logits, arrays))
    return {
        "tp": world, "value": tokens / (ms / 1e3), "unit": UNIT, "ms_per_step": ms, "scaling": "strong",
        "decisions_per_s": decisions / (ms / 1e3),
        "tensor_frac": {"achieved_tflops": (linear + attention) / (ms / 1e3) / 1e12,
                        "frac_of_measured_burst_x_gpus": (linear + attention) / (ms / 1e3) / 1e12 / (peaks["bf16_tflops"] * world)},
        "kernel_ms_per_step_rank0": {k: round(v, 3) for k, v in per.items()},
        "split_ms_per_step_rank0": {
            "gemm_incl_fused_reduction": round(gemm, 3), "attention": round(per.get("attention", 0.0), 3),
            "reduction_unfused": round(per.get("residual_add", 0.0), 3), "barrier": round(per.get("allreduce", 0.0), 3),
            "other": round(sum(per.values()) - gemm - per.get("attention", 0.0) - per.get("residual_add", 0.0)
                           - per.get("allreduce", 0.0), 3)},
        "gpu_launches_rank0": launches, "clocks_rank0": clocks,
        "layout": "Hq/tp query and Hkv/tp key-value heads, F/tp MLP columns per rank; FP32 partials of o-proj and "
        "down-proj summed over NVLink peer memory (fused into the down-proj GEMM; o-proj fused when K tp/(tp-1) >= 1536)",
    }


def gpu_arm(args) -> None:
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))

    from deciax_b200 import _lib
    from deciax_b200.build import build as build_lib
    from deciax_b200.synthetic import field_probabilities

    build_lib()
    tp_parity = tp_preflight(rank, world, local) if world > 1 and not args.no_tp else None

    # --- data parallel: every rank a full replica with its own batch ---
    cfg = dict(CFG2, num_layers=args.layers)  # --layers: a shorter stack for profiling captures only
    model = build_model(local, cfg=cfg)
    arrays = make_batch(seed=100 + rank)
    tensors = device_batch(arrays)
    out = torch.empty(arrays["option_mask"].shape, dtype=torch.float32, device="cuda")
    # A real stream: the library enqueues on it and the CUDA events are
    # recorded on it.  (torch's default stream is the legacy NULL stream, for
    # which the library would use its own stream instead.)
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    elapsed_ms, timing, clocks = timed_forwards(model, tensors, out, stream, args.steps, args.warmup, local, dist)
    launches = model.last_launch_count * args.steps
    logits_dev = out.cpu().numpy()
    if not np.isfinite(logits_dev[arrays["option_mask"]]).all():
        raise SystemExit("non-finite logits")

    def barrier():
        if dist:
            dist.barrier()

    # --- end to end through the host API ---
    h2d = sum(int(np.asarray(arrays[k]).size * (1 if arrays[k].dtype == bool else 4)) for k in _lib.BATCH_KEYS)
    d2h = int(np.asarray(arrays["option_mask"]).size * 4)
    model.forward(arrays)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        logits = model.forward(arrays)
    e2e_s = time.perf_counter() - t0
    barrier()
    model.close()
    decisions = sum(len(f) for f in field_probabilities(logits, arrays))

    elapsed_ms = rank_reduce(elapsed_ms, "max")
    e2e_s = rank_reduce(e2e_s, "max")
    tokens = STATES * SEQ
    value = world * tokens * args.steps / (elapsed_ms / 1e3)
    e2e_value = world * tokens * args.steps / e2e_s
    linear, attention, gu_flops_per_token = algorithmic_flops(cfg, [SEQ] * STATES)
    peaks = measured_peaks()
    step_s = elapsed_ms / 1e3 / args.steps
    gu_ms, gu_n = timing["gemm_gate_up"]
    gu_avg_s = gu_ms / 1e3 / max(gu_n, 1)
    gu_flops = gu_flops_per_token * tokens
    achieved = gu_flops / gu_avg_s / 1e12
    peak = peaks["bf16_tflops_sustained"]
    total_ms = sum(ms for ms, _ in timing.values())
    shares = {k: round(ms / total_ms, 4) for k, (ms, _) in timing.items() if ms > 0}
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (random-init weights, uniform token ids)",
        "config": workload_config(world) | ({"layers_override": args.layers} if args.layers != CFG2["num_layers"] else {}),
        "decisions_per_s": world * decisions * args.steps / (elapsed_ms / 1e3),
        "tensor_frac": {"flops_per_step": linear + attention, "achieved_tflops": (linear + attention) / step_s / 1e12,
                        "frac_of_measured_burst": (linear + attention) / step_s / 1e12 / peaks["bf16_tflops"],
                        "frac_of_measured_sustained": (linear + attention) / step_s / 1e12 / peaks["bf16_tflops_sustained"],
                        "peak_source": peaks["source"]},
        "roofline": {"kernel": "gemm_gate_up (tcgen05, fused SwiGLU epilogue)", "bound": "tensor", "achieved": achieved,
                     "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "peak_kind": f"bf16_tflops_sustained of {peaks['source']} (kernel timed inside a long step)",
                     "flops_per_launch": gu_flops, "avg_launch_ms": gu_avg_s * 1e3, "traffic": traffic_per_launch()},
        "kernel_ms_per_step": {k: round(ms / args.steps, 3) for k, (ms, _) in timing.items() if ms > 0},
        "timeline_ms_per_step": total_ms / args.steps,  # cross-check of ms_per_step from the per-launch events
        "kernel_share": shares,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if world > 1 and not args.no_tp:
        line["tp"] = tp_arm(args, rank, world, local, dist)
        line["tp_parity"] = tp_parity
    if world == 1 and not args.no_parity:
        line["parity"] = cfg2_slice_parity(local)
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_sample(repeats=4)
        cb.pop("seconds", None)
        line["cpu_baseline"] = cb
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def gemm_arm(args) -> None:
    """BASELINE configs[2] ("cfg3"): the fused-QKV and fused gated-MLP GEMMs at
    M=16384 through the kernel-level C ABI, reported as TFLOP/s.

    x [16384, 3584] ~ N(0,1); W_qkv [8192, 3584] ((16+2x8)x256 rows, no gate,
    as BASELINE states), W_gate|up packed [28672, 3584], W_down [3584, 14336],
    all N(0, 0.02), seed 2, BF16.  One step = QKV GEMM + gate/up GEMM with the
    SwiGLU epilogue + down GEMM with the residual epilogue.
    """
    import torch

    from deciax_b200 import _lib
    from deciax_b200.build import build as build_lib

    build_lib()
    lib = _lib.load()
    torch.cuda.set_device(0)
    gen = torch.Generator(device="cuda:0")
    gen.manual_seed(2)
    M, D, F, NQ = 16384, 3584, 14336, (16 + 2 * 8) * 256

    def randn(*shape, std):
        return torch.empty(shape, dtype=torch.bfloat16, device="cuda").normal_(0.0, std, generator=gen)

    x = randn(M, D, std=1.0)
    w_qkv = randn(NQ, D, std=WEIGHT_STD)
    w_gu = randn(2 * F, D, std=WEIGHT_STD)
    w_down = randn(D, F, std=WEIGHT_STD)
    qkv = torch.empty((M, NQ), dtype=torch.bfloat16, device="cuda")
    act = torch.empty((M, F), dtype=torch.bfloat16, device="cuda")
    y = torch.empty((M, D), dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    sp = stream.cuda_stream
    B = _lib.DTYPE_BF16
    events = []

    def step(timed: bool) -> None:
        calls = [(0, M, NQ, D, x, w_qkv, qkv, NQ, None, 0), (1, M, 2 * F, D, x, w_gu, act, F, None, 0),
                 (2, M, D, F, act, w_down, y, D, y, D)]
        for epi, m, n, k, a, b, out, ldo, res, ldr in calls:
            if timed:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
            _lib.check(lib.clef_op_gemm(B, epi, m, n, k, a.data_ptr(), b.data_ptr(), out.data_ptr(), ldo, None,
                                        res.data_ptr() if res is not None else None, ldr, sp))
            if timed:
                e1.record(stream)
                events.append((epi, e0, e1))

    for _ in range(args.warmup):
        step(False)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            step(True)
        end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    flops = {0: 2.0 * M * D * NQ, 1: 2.0 * M * D * 2 * F, 2: 2.0 * M * F * D}
    per = {0: [], 1: [], 2: []}
    for epi, e0, e1 in events:
        per[epi].append(e0.elapsed_time(e1))
    total = sum(flops.values())
    peaks = measured_peaks()
    names = {0: "qkv", 1: "gate_up_swiglu", 2: "down_residual"}
    kern = {names[e]: {"ms": statistics.mean(v), "tflops": flops[e] / (statistics.mean(v) / 1e3) / 1e12} for e, v in per.items()}
    value = total * args.steps / (ms / 1e3) / 1e12
    print(json.dumps({
        "metric": "cfg3 fused QKV + gated-MLP GEMM throughput (M=16384, BF16)", "value": value, "unit": "TFLOP/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "cfg3: x[16384,3584] N(0,1); W_qkv[8192,3584], W_gate|up[28672,3584], W_down[3584,14336] "
                   "N(0,0.02) seed 2", "l2": "operands larger than L2 (1.3 GB per step)"},
        "kernels": kern, "frac_of_measured_burst": value / peaks["bf16_tflops"],
        "frac_of_measured_sustained": value / peaks["bf16_tflops_sustained"], "gpu_launches": 3 * args.steps,
        "clocks": clocks.summary(),
    }), flush=True)


def attention_arm(args) -> None:
    """One attention layer alone: causal GQA over a packed projection with the
    sigmoid gate, through clef_op_attention; TFLOP/s counts causal pairs only.
    ``attention``: cfg2's layer (8 x 2048 tokens, 16 query / 8 key-value heads
    of 256); ``attention4``: cfg4's (16 x 8192 tokens, 32 / 16 heads of 128)."""
    import torch

    from deciax_b200 import _lib
    from deciax_b200.build import build as build_lib

    build_lib()
    lib = _lib.load()
    torch.cuda.set_device(0)
    gen = torch.Generator(device="cuda:0")
    gen.manual_seed(3)
    if args.workload == "attention4":
        B, S, H, HK, Dh = CFG4_BATCH["states"], CFG4_BATCH["seq"], CFG4["num_attention_heads"], CFG4["num_key_value_heads"], CFG4["head_dim"]
        label = "cfg4 attention layer throughput (B16 S8192 32q/16kv x128, causal, gated)"
    else:
        B, S, H, HK, Dh = STATES, SEQ, CFG2["num_attention_heads"], CFG2["num_key_value_heads"], CFG2["head_dim"]
        label = "cfg2 attention layer throughput (B8 S2048 16q/8kv x256, causal, gated)"
    n = H * 2 * Dh + 2 * HK * Dh
    qkv = torch.empty((B * S, n), dtype=torch.bfloat16, device="cuda").normal_(0.0, 1.0, generator=gen)
    mask = torch.ones((B, S), dtype=torch.uint8, device="cuda")
    out = torch.empty((B * S, H * Dh), dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()

    def run():
        _lib.check(lib.clef_op_attention(_lib.DTYPE_BF16, qkv.data_ptr(), mask.data_ptr(), out.data_ptr(), B, S, H, HK, Dh,
                                         0.0, 0, stream.cuda_stream))

    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        run()
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    flops = 2.0 * H * Dh * S * (S + 1) * B
    peaks = measured_peaks()
    print(json.dumps({"metric": label,
                      "value": flops / (ms / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms, "steps": args.steps,
                      "warmup": args.warmup, "frac_of_measured_burst": flops / (ms / 1e3) / 1e12 / peaks["bf16_tflops"],
                      "dtype": "bf16", "data": "synthetic", "gpu_launches": args.steps}), flush=True)


CFG5 = {"states": 256, "median": 600, "sigma": 0.8, "min": 32, "max": 16384, "seed": 5, "long": 4}


def serving_records(lengths, vocab: int, seed: int):
    """Encoded records of the given lengths (uniform token ids) whose last 32
    tokens hold 4 choice fields: 4 tokens of question span, then 4
    single-token options each (the cfg2 layout), and the matching schema."""
    from deciax_b200.clef_input import Field, Record

    rng = np.random.default_rng(seed)
    questions = {f"q{k}": {"type": "choice", "criteria": {c: f"option {c}" for c in "abcd"}} for k in range(QUESTIONS)}
    records = []
    for n in lengths:
        ids = rng.integers(0, vocab, size=int(n), dtype=np.int64)
        fields = []
        for k in range(QUESTIONS):
            off = int(n) - 8 * QUESTIONS + 8 * k
            fields.append(Field(f"q{k}", 1, (off, off + 4), tuple((off + 4 + j, off + 5 + j) for j in range(OPTIONS)),
                                tuple("abcd")))
        records.append(Record(tuple(int(i) for i in ids), tuple(fields)))
    return records, questions


def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id from the library (made on rank 0, then shared)."""
    from deciax_b200 import _lib

    buf = ctypes.create_string_buffer(_lib.NCCL_ID_BYTES)
    _lib.check(_lib.load().clef_nccl_unique_id(buf))
    return buf.raw


def serving_arm(args) -> None:
    """BASELINE cfg5: decide_batch of 256 states with lognormal lengths (median
    600, sigma 0.8, clipped to [32, 16384], seed 5), 4 choice x 4 options
    each, through ClefEngine (length-grouped batches, host arrays in, answers
    out), plus the max_len case of 4 x 16384 tokens.  Under torchrun each rank
    (one GPU, a full replica) serves every N-th state: data parallel, max over
    ranks.  With --serving-tp the N ranks instead form one tensor-parallel
    model and every rank runs every batch (the engine's batch plan depends only
    on the records, so the ranks stay in step); rank 0's answers count.
    Reports decisions/s and p50/p99 per-batch latency."""
    import torch

    from deciax_b200.engine import ClefEngine

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=torch.device("cuda", local))
    c = CFG5
    tp = world if args.serving_tp and world > 1 else 1
    rng = np.random.default_rng(c["seed"])
    lengths = np.clip(np.round(rng.lognormal(np.log(c["median"]), c["sigma"], c["states"])), c["min"], c["max"]).astype(int)
    longs, _ = serving_records([c["max"]] * c["long"], CFG2["vocab_size"], seed=20)
    if tp > 1:
        sweep, questions = serving_records(lengths, CFG2["vocab_size"], seed=10)
        model = build_model(local, max_seq_len=c["max"], tp_rank=rank, tp_size=tp, nccl_id=share_from_rank0(nccl_unique_id))
    else:
        sweep, questions = serving_records(lengths[rank::world], CFG2["vocab_size"], seed=10 + rank)
        longs = longs[rank::world]
        model = build_model(local, max_seq_len=c["max"])

    def run(records, timings=None, eng=None):
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        answers = (eng or engine).decide_records(records, questions, timings) if records else []
        elapsed = time.perf_counter() - t0
        return answers, elapsed

    def pct(vals, q):
        return float(np.percentile(np.asarray(vals) * 1e3, q)) if vals else 0.0

    def first_sweep(m, warm: bool) -> dict:
        """The first sweep a fresh model serves: after ClefEngine.warmup (the
        server's warm-up request) or cold, its workspace growing with each new
        batch shape."""
        eng = ClefEngine(m, auto_warmup=warm)
        warm_s = 0.0
        if warm:
            if dist:
                dist.barrier()
            t0 = time.perf_counter()
            eng.warmup()
            warm_s = time.perf_counter() - t0
        before = m.workspace_allocations
        timings = []
        _, s = run(sweep, timings, eng)
        return {"warmup_seconds": rank_reduce(warm_s, "max"), "sweep_seconds": rank_reduce(s, "max"),
                "batch_latency_ms": {"p50": rank_reduce(pct([t for *_, t in timings], 50), "max"),
                                     "p99": rank_reduce(pct([t for *_, t in timings], 99), "max"),
                                     "max": rank_reduce(pct([t for *_, t in timings], 100), "max")},
                "workspace_allocations_during_sweep": int(rank_reduce(float(m.workspace_allocations - before), "max"))}

    # a second, fresh model serves its first sweep cold, then is released
    if tp > 1:
        cold_model = build_model(local, max_seq_len=c["max"], tp_rank=rank, tp_size=tp,
                                 nccl_id=share_from_rank0(nccl_unique_id))
    else:
        cold_model = build_model(local, max_seq_len=c["max"])
    cold = first_sweep(cold_model, warm=False)
    cold_model.close()
    del cold_model
    warmed = first_sweep(model, warm=True)
    engine = ClefEngine(model)

    for _ in range(args.warmup):
        run(sweep)
        run(longs)
    sweep_t, long_t, timings, long_timings = [], [], [], []
    for _ in range(args.steps):
        answers, t = run(sweep, timings)
        sweep_t.append(t)
        _, t = run(longs, long_timings)
        long_t.append(t)
    assert all(len(a["answers"]) == QUESTIONS for a in answers)

    agg = rank_reduce

    sweep_s = agg(statistics.mean(sweep_t), "max")
    long_s = agg(statistics.mean(long_t), "max")
    count = "max" if tp > 1 else "sum"  # TP ranks serve the same states; DP ranks disjoint ones
    decisions = agg(float(len(sweep) * QUESTIONS), count)
    tokens = agg(float(sum(len(r.ids) for r in sweep)), count)
    p50, p99 = agg(pct([t for *_, t in timings], 50), "max"), agg(pct([t for *_, t in timings], 99), "max")
    lp50 = agg(pct([t for *_, t in long_timings], 50), "max")
    if dist:
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({
            "metric": "cfg5 serving sweep: decisions/s (decide_batch of 256 lognormal-length states)",
            "value": decisions / sweep_s, "unit": "decisions/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
            "data": "synthetic (random-init weights, uniform token ids, lognormal lengths)",
            "config": {"workload": "cfg5", "states": c["states"], "lengths": "lognormal(log 600, 0.8) clipped [32, 16384], seed 5",
                       "total_tokens": int(lengths.sum()),
                       "parallelism": f"tp{tp}" if tp > 1 else (f"dp{world}" if world > 1 else "single"),
                       "batching": "ClefEngine length-grouped, max_batch_tokens 65536"},
            "prefill_tokens_per_s": tokens / sweep_s, "sweep_seconds": sweep_s,
            "batch_latency_ms": {"p50": p50, "p99": p99, "batches_per_rank": len(timings) // max(args.steps, 1)},
            "first_sweep": {"after_warmup": warmed, "cold": cold},
            "max_len_case": {"states": c["long"], "tokens_per_state": c["max"], "seconds": long_s,
                             "decisions_per_s": c["long"] * QUESTIONS / long_s, "batch_latency_ms_p50": lp50},
            "timing": "host wall clock around ClefEngine.decide_records (collate, H2D, forward, D2H, decode)",
        }), flush=True)


def rmsnorm_arm(args) -> None:
    """cfg2's RMSNorm alone (the memory-bound kernel run 85 times per step):
    [16384, 3584] bf16 in and out (235 MB, larger than L2), through
    clef_op_rmsnorm; achieved GB/s = (read + write bytes) / time."""
    import torch

    from deciax_b200 import _lib
    from deciax_b200.build import build as build_lib

    build_lib()
    lib = _lib.load()
    torch.cuda.set_device(0)
    rows, dim = STATES * SEQ, CFG2["hidden_size"]
    gen = torch.Generator(device="cuda:0")
    gen.manual_seed(6)
    x = torch.empty((rows, dim), dtype=torch.bfloat16, device="cuda").normal_(0.0, 1.0, generator=gen)
    w = torch.empty(dim, dtype=torch.bfloat16, device="cuda").normal_(0.0, 0.02, generator=gen)
    out = torch.empty_like(x)
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()

    def run():
        _lib.check(lib.clef_op_rmsnorm(_lib.DTYPE_BF16, x.data_ptr(), w.data_ptr(), out.data_ptr(), rows, dim,
                                       ctypes.c_float(1e-6), stream.cuda_stream))

    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(args.steps):
        run()
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    moved = 2 * rows * dim * 2 + dim * 2
    peaks = measured_peaks()
    print(json.dumps({"metric": "cfg2 RMSNorm bandwidth ([16384, 3584] bf16)", "value": moved / (ms / 1e3) / 1e9,
                      "unit": "GB/s", "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup,
                      "frac_of_measured_hbm": moved / (ms / 1e3) / 1e9 / peaks["hbm_gbs"], "bytes_per_launch": moved,
                      "dtype": "bf16", "data": "synthetic", "gpu_launches": args.steps}), flush=True)


CFG4 = dict(hidden_size=4608, intermediate_size=36864, num_attention_heads=32, num_key_value_heads=16, head_dim=128,
            num_layers=46, vocab_size=256000)
CFG4_BATCH = {"states": 16, "seq": 8192, "choice": (8, 24), "score": (24, 8), "noul": 32}


def mixed_records(states: int, length: int, vocab: int, seed: int):
    """cfg4 records: per state `length` uniform token ids ending in 64 fields
    (8 choice x 24 options, 24 score x 8 levels, 32 noul x 2 = 448 options);
    each field is 4 tokens of question span followed by one token per option."""
    from deciax_b200.clef_input import Field, Record

    rng = np.random.default_rng(seed)
    c = CFG4_BATCH
    kinds = [(1, c["choice"][1])] * c["choice"][0] + [(2, c["score"][1])] * c["score"][0] + [(0, 2)] * c["noul"]
    schema = sum(4 + n for _, n in kinds)
    records = []
    for _ in range(states):
        ids = rng.integers(0, vocab, size=length, dtype=np.int64)
        off, fields = length - schema, []
        for k, (kind, n) in enumerate(kinds):
            oids = ("true", "false") if kind == 0 else tuple(str(j) for j in range(n))
            fields.append(Field(f"f{k}", kind, (off, off + 4), tuple((off + 4 + j, off + 5 + j) for j in range(n)), oids))
            off += 4 + n
        records.append(Record(tuple(int(i) for i in ids), tuple(fields)))
    return records


def cfg4_arm(args) -> None:
    """BASELINE cfg4: the clef-shaped 27B model (46 layers, hidden 4608, 32 q /
    16 kv heads of 128, MLP 36864, vocab 256000), BF16, tensor-parallel over
    the N ranks of torchrun (heads and MLP columns sharded; the o-proj and
    down-proj partials summed in FP32 across ranks over NVLink peer memory
    inside the projection kernel), one batch of 16 states x 8192 tokens per
    step (64 fields, 448 options per state).  Strong scaling: the work per
    step is fixed; value = the group's tokens/s."""
    import torch

    from deciax_b200 import _lib
    from deciax_b200.clef_input import collate

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    nccl_id = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=torch.device("cuda", local))
        nccl_id = share_from_rank0(nccl_unique_id)
    c = CFG4_BATCH
    model = build_model(local, max_seq_len=c["seq"], cfg=CFG4, tp_rank=rank, tp_size=world, nccl_id=nccl_id)
    arrays = collate(mixed_records(c["states"], c["seq"], CFG4["vocab_size"], seed=31), 0)
    tensors = {k: torch.from_numpy(np.ascontiguousarray(arrays[k]).astype(np.uint8 if arrays[k].dtype == bool else np.int32)).cuda()
               for k in _lib.BATCH_KEYS}
    out = torch.empty(arrays["option_mask"].shape, dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()

    def barrier():
        if dist:
            dist.barrier()
            torch.cuda.synchronize()

    for _ in range(args.warmup):
        model.forward_device(tensors, out, stream.cuda_stream)
    torch.cuda.synchronize()
    model.check_status()
    barrier()
    model.set_timing(True)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            model.forward_device(tensors, out, stream.cuda_stream)
        end.record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = start.elapsed_time(end) / args.steps
    timing = model.timing_report()
    model.set_timing(False)
    model.check_status()
    logits = out.cpu().numpy()
    if not np.isfinite(logits[arrays["option_mask"]]).all():
        raise SystemExit("non-finite logits")
    ms = rank_reduce(ms, "max")
    tokens = c["states"] * c["seq"]
    linear, attention, _ = algorithmic_flops(CFG4, [c["seq"]] * c["states"])
    flops = linear + attention
    peaks = measured_peaks()
    if rank == 0:
        print(json.dumps({
            "metric": "cfg4 27B-shaped prefill+scoring tokens/s (tensor parallel)", "value": tokens / (ms / 1e3),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "dtype": "bf16",
            "data": "synthetic (random-init weights, uniform token ids)",
            "config": {"workload": "cfg4: 46 layers, D4608, 32q/16kv x128, F36864, V256000; 16 x 8192 tokens; 64 fields / 448 "
                       "options per state (8 choice x 24, 24 score x 8, 32 noul)", "parallelism": f"tp{world}"},
            "decisions_per_s": c["states"] * 64 / (ms / 1e3),
            "tensor_frac": {"flops_per_step": flops, "achieved_tflops": flops / (ms / 1e3) / 1e12,
                            "frac_of_measured_burst_x_gpus": flops / (ms / 1e3) / 1e12 / (peaks["bf16_tflops"] * world)},
            "kernel_ms_per_step_rank0": {k: round(v[0] / args.steps, 3) for k, v in timing.items() if v[1]},
            "clocks": clocks.summary(), "gpu_launches": model.last_launch_count * args.steps,
        }), flush=True)
    if dist:
        model.close()
        dist.destroy_process_group()


GDN = {"states": 8, "seq": 2048, "key_heads": 16, "value_heads": 32, "head_dim": 128, "conv": 4}


def gdn_flops(c: dict) -> float:
    """Algorithmic FLOPs of the chunked delta rule (64-token chunks) per
    launch: per chunk and value head, k k^T and q k^T (2 C^2 dk each), the
    triangular solve on dk + dv right-hand columns (C^2 (dk + dv)), X_k S,
    (q e^g) S and the state update (2 C dk dv each), and (q k^T) value
    (2 C^2 dv); the conv, norms and gates are O(C d) and not counted."""
    C, dk, dv = 64, c["head_dim"], c["head_dim"]
    per_chunk = 2 * C * C * dk * 2 + C * C * (dk + dv) + 3 * 2 * C * dk * dv + 2 * C * C * dv
    chunks = -(-c["seq"] // C)
    return float(per_chunk * chunks * c["value_heads"] * c["states"])


def gdn_arm(args) -> None:
    """The Gated DeltaNet core (conv, chunked delta rule, gated norm) of one
    linear_attention layer, through clef_op_gdn_core at Qwen3.5-style dims
    (16 key / 32 value heads of 128, conv 4) on 8 x 2048 tokens, BF16 I/O."""
    import torch

    from deciax_b200 import _lib
    from deciax_b200.build import build as build_lib

    build_lib()
    lib = _lib.load()
    torch.cuda.set_device(0)
    c = GDN
    B, S, nh, nv, dh = c["states"], c["seq"], c["key_heads"], c["value_heads"], c["head_dim"]
    n = 2 * nh * dh + 2 * nv * dh + 2 * nv
    gen = torch.Generator(device="cuda:0")
    gen.manual_seed(4)
    proj = torch.empty((B * S, n), dtype=torch.bfloat16, device="cuda").normal_(0.0, 1.0, generator=gen)
    conv = torch.empty((2 * nh * dh + nv * dh, c["conv"]), dtype=torch.bfloat16, device="cuda").normal_(0.0, 0.5,
                                                                                                     generator=gen)
    a_log = torch.empty(nv, device="cuda").uniform_(0.01, 0.3, generator=gen).log().to(torch.bfloat16)
    dt_bias = torch.zeros(nv, dtype=torch.bfloat16, device="cuda")
    norm_w = torch.ones(dh, dtype=torch.bfloat16, device="cuda")
    out = torch.empty((B * S, nv * dh), dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()

    def run():
        _lib.check(lib.clef_op_gdn_core(_lib.DTYPE_BF16, proj.data_ptr(), n, conv.data_ptr(), c["conv"], a_log.data_ptr(),
                                        dt_bias.data_ptr(), norm_w.data_ptr(), out.data_ptr(), B, S, nh, nv, dh,
                                        ctypes.c_float(1e-6), stream.cuda_stream))

    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            run()
        end.record(stream)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    flops = gdn_flops(c)
    clk = clocks.summary()
    # FP32 CUDA-core peak at the sampled clock: 148 SMs x 128 FP32 lanes x 2 FLOP per FMA
    fp32_peak = 148 * 128 * 2 * clk["sm_mhz"] * 1e6 / 1e12 if clk.get("sm_mhz") else None
    moved = proj.numel() * 2 + out.numel() * 2
    print(json.dumps({"metric": "Gated DeltaNet core throughput (B8 S2048, 16 key / 32 value heads x128)",
                      "value": flops / (ms / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms, "steps": args.steps,
                      "warmup": args.warmup, "dtype": "bf16 I/O, fp32 recurrence", "data": "synthetic",
                      "flops_per_launch": flops, "frac_of_fp32_cuda_core_peak_at_sampled_clock":
                      (flops / (ms / 1e3) / 1e12 / fp32_peak) if fp32_peak else None,
                      "hbm_bytes_per_launch": moved, "achieved_gbs": moved / (ms / 1e3) / 1e9, "clocks": clk,
                      "gpu_launches": 3 * args.steps}), flush=True)


def traffic_per_launch():
    """DRAM bytes per gate/up launch from the committed ncu summary, if present."""
    p = ROOT / "profiles" / "gemm_gate_up_m16384.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_full_launch:"):
            return float(line.split(":", 1)[1].split()[0])
    return None


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("cuda", "reference"), default="cuda")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="N=1: skip the cfg2-slice parity check against the oracle")
    ap.add_argument("--no-tp", action="store_true", help="N>1: skip the TP=N preflight and timed run")
    ap.add_argument("--layers", type=int, default=CFG2["num_layers"],
                    help="cfg2 with fewer decoder layers: a small case for ncu captures of single kernels (not a bench line)")
    ap.add_argument("--serving-tp", action="store_true",
                    help="cfg5 under torchrun: one tensor-parallel model over the N GPUs instead of N replicas")
    ap.add_argument("--workload", choices=("cfg2", "cfg3", "cfg4", "cfg5", "attention", "attention4", "gdn", "rmsnorm"), default="cfg2",
                    help="cfg2 = the full prefill+scoring step (default); cfg3 = the GEMM microbenchmark; "
                    "cfg5 = the serving sweep through ClefEngine; attention = cfg2's attention layer alone; "
                    "gdn = one Gated DeltaNet core; rmsnorm = cfg2's RMSNorm alone; cfg4 = the 27B-shaped model, "
                    "tensor parallel over the torchrun ranks")
    args = ap.parse_args()
    if args.impl == "reference":
        reference_arm(args)
    elif args.workload == "cfg3":
        gemm_arm(args)
    elif args.workload in ("attention", "attention4"):
        attention_arm(args)
    elif args.workload == "gdn":
        gdn_arm(args)
    elif args.workload == "cfg5":
        serving_arm(args)
    elif args.workload == "rmsnorm":
        rmsnorm_arm(args)
    elif args.workload == "cfg4":
        cfg4_arm(args)
    else:
        gpu_arm(args)


if __name__ == "__main__":
    main()
