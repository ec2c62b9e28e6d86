"""Typed configuration: YAML in, dataclasses out, unknown keys rejected.

Schema parity: every section, key and default of the reference's
``packbalance/config.py:20-137`` is accepted here with the same meaning, so a
reference YAML file loads unchanged.  Keys added by this framework are grouped at
the end of each dataclass and default to behaviour that matches the reference.
Strict loading (unknown sections / keys are errors) follows ``config.py:147-179``.
"""

from __future__ import annotations

import dataclasses
import math
from dataclasses import asdict, dataclass, field, fields
from pathlib import Path
from typing import Any

import yaml

# "sm100" selects the native varlen attention kernel explicitly; "auto" picks it on
# CUDA tensors and the eager per-document oracle on CPU tensors.  "flex" is kept as
# an accepted value for reference configs and means the same as "auto" here.
ATTENTION_BACKENDS = ("auto", "flex", "eager", "sm100")
PACKING_MODES = ("pad", "pack_random", "pack_ffd", "isoflop")
SCHEDULES = ("balanced", "random")
TOKEN_DISTRIBUTIONS = ("uniform", "zipf")
COMM_BACKENDS = ("auto", "fused", "nccl")
DTYPES = ("bf16", "fp16", "fp32")


@dataclass
class ModelConfig:
    vocab_size: int = 49152
    d_model: int = 512
    n_layers: int = 8
    n_heads: int = 8
    n_kv_heads: int = 2
    d_ff: int = 1536
    max_seq_len: int = 2048
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    tie_embeddings: bool = True
    dropout: float = 0.0
    attention_backend: str = "auto"
    compile_attention: bool = True
    use_fused_rmsnorm: bool = True
    use_fused_swiglu: bool = True
    use_fused_ce: bool = True
    ce_chunk_size: int = 1024
    z_loss_coeff: float = 0.0
    gradient_checkpointing: bool = False
    init_std: float = 0.02

    def __post_init__(self) -> None:
        if self.attention_backend not in ATTENTION_BACKENDS:
            raise ValueError(f"attention_backend must be one of {ATTENTION_BACKENDS}")
        if self.d_model % self.n_heads != 0:
            raise ValueError("d_model must be divisible by n_heads")
        if self.n_heads % self.n_kv_heads != 0:
            raise ValueError("n_heads must be divisible by n_kv_heads")
        if self.d_ff <= 0 or self.n_layers <= 0:
            raise ValueError("d_ff and n_layers must be positive")
        if self.head_dim % 2:
            raise ValueError("head_dim must be even for RoPE")
        if self.ce_chunk_size <= 0:
            raise ValueError("ce_chunk_size must be positive")

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    @property
    def d_kv(self) -> int:
        return self.n_kv_heads * self.head_dim


@dataclass
class DataConfig:
    dataset: str = "synthetic"
    data_dir: str = "data/synthetic"
    tokenizer: str = "HuggingFaceTB/SmolLM-135M"
    seq_len: int = 2048
    mode: str = "isoflop"
    schedule: str = "balanced"
    pad_batch_size: int = 8
    max_docs: int | None = None
    num_workers: int = 4
    prefetch_factor: int = 4
    pin_memory: bool = True
    persistent_workers: bool = True
    val_fraction: float = 0.01
    seed: int = 42
    pad_token_id: int = 0
    eos_token_id: int = 0
    min_doc_len: int = 8
    max_doc_len: int = 2048
    synthetic_num_docs: int = 20000
    synthetic_mu: float = 5.5
    synthetic_sigma: float = 1.0
    synthetic_min_len: int = 16
    synthetic_max_len: int = 4096
    synthetic_vocab_size: int = 49152
    isoflop_iterations: int = 8
    drop_last: bool = True
    # --- additions (synthetic generators of the B200 benchmark configs) ---
    # Median document length; when set it overrides ``synthetic_mu`` (mu = ln median).
    synthetic_median: float | None = None
    # "uniform": ids uniform in [synthetic_token_min, vocab); "zipf": Zipf(s) ranks
    # mapped onto the same id range.
    synthetic_token_dist: str = "uniform"
    synthetic_zipf_s: float = 1.1
    synthetic_token_min: int = 0
    # False: last token of every document is overwritten by EOS (reference
    # behaviour, ``prepare.py:69-70``).  True: EOS is appended after the length drawn.
    synthetic_append_eos: bool = False
    # Fraction of documents replaced by one document of exactly ``seq_len`` tokens
    # (the adversarial single-document packs of the long-context config).
    synthetic_long_doc_frac: float = 0.0

    def __post_init__(self) -> None:
        if self.mode not in PACKING_MODES:
            raise ValueError(f"mode must be one of {PACKING_MODES}")
        if self.schedule not in SCHEDULES:
            raise ValueError(f"schedule must be one of {SCHEDULES}")
        if self.seq_len <= 0:
            raise ValueError("seq_len must be positive")
        if self.synthetic_token_dist not in TOKEN_DISTRIBUTIONS:
            raise ValueError(f"synthetic_token_dist must be one of {TOKEN_DISTRIBUTIONS}")
        if not 0.0 <= self.synthetic_long_doc_frac <= 1.0:
            raise ValueError("synthetic_long_doc_frac must be in [0, 1]")

    @property
    def lognormal_mu(self) -> float:
        if self.synthetic_median is not None:
            return math.log(self.synthetic_median)
        return self.synthetic_mu


@dataclass
class TrainConfig:
    output_dir: str = "artifacts/run"
    seed: int = 42
    max_steps: int = 2000
    grad_accum: int = 4
    lr: float = 3e-4
    min_lr: float = 3e-5
    warmup_steps: int = 100
    weight_decay: float = 0.1
    beta1: float = 0.9
    beta2: float = 0.95
    grad_clip: float = 1.0
    dtype: str = "bf16"
    log_interval: int = 10
    eval_interval: int = 0
    eval_steps: int = 20
    save_interval: int = 500
    keep_last: int = 2
    resume: bool = False
    fsdp: bool = False
    compile: bool = False
    profile: bool = False
    profile_steps: int = 5
    profile_warmup: int = 2
    gpu_hourly_cost: float = 2.0
    peak_tflops: float = 0.0
    deterministic: bool = False
    bucket_cap_mb: int = 25
    find_unused_parameters: bool = False
    # --- additions ---
    # Gradient all-reduce / reduce-scatter transport: "fused" = this framework's
    # peer-memory kernels, "nccl" = torch.distributed collectives, "auto" = fused
    # on CUDA when peer memory can be set up, else nccl (gloo on CPU).
    comm_backend: str = "auto"
    # Process-group timeout; a rank that stops answering ends its peers' next
    # collective with an error instead of a hang.
    pg_timeout_s: float = 300.0
    # Run the step's grad_accum packs of one rank as ONE forward/backward over their
    # concatenation (document masking keeps packs independent).  The loss and the
    # gradient are those of the microbatch loop; only the launch count changes.
    fuse_microbatches: bool = True
    # Capture the native single-GPU / data-parallel step in a CUDA graph and replay it
    # (inputs copied into static buffers); steps with a new input shape run eagerly.
    cuda_graphs: bool = True
    # Skip the optimizer step when the gradient norm is not finite.
    skip_nonfinite_steps: bool = True
    # Data type on the wire of the fused gradient all-reduce: "fp32" (the reference's
    # precision), or "bf16" (half the NVLink bytes; every sum in fp32, each rank's input
    # and the average rounded to bf16, identical on every rank).
    grad_reduce_dtype: str = "fp32"
    # Native sharded engine (fsdp on CUDA): 0 keeps every unit's gathered bf16 weights
    # for the whole step (2 B/param per rank, no second all-gather); K >= 2 rotates the
    # decoder layers' gathered weights through K windows of one layer, fetched again for
    # the backward pass one layer ahead (the reference's FSDP2 resharding after forward);
    # -1 (auto) keeps them when they take at most a quarter of the device's memory, else
    # uses two windows.
    fsdp_weight_windows: int = -1

    def __post_init__(self) -> None:
        if self.dtype not in DTYPES:
            raise ValueError("dtype must be bf16, fp16, or fp32")
        if self.max_steps <= 0:
            raise ValueError("max_steps must be positive")
        if self.grad_accum <= 0:
            raise ValueError("grad_accum must be positive")
        if self.comm_backend not in COMM_BACKENDS:
            raise ValueError(f"comm_backend must be one of {COMM_BACKENDS}")
        if self.keep_last < 0:
            raise ValueError("keep_last must be >= 0")
        if self.grad_reduce_dtype not in ("fp32", "bf16"):
            raise ValueError("grad_reduce_dtype must be fp32 or bf16")
        if self.fsdp_weight_windows < -1 or self.fsdp_weight_windows == 1:
            raise ValueError("fsdp_weight_windows must be -1 (auto), 0 or at least 2")


@dataclass
class PackBalanceConfig:
    model: ModelConfig = field(default_factory=ModelConfig)
    data: DataConfig = field(default_factory=DataConfig)
    train: TrainConfig = field(default_factory=TrainConfig)


_SECTIONS = {"model": ModelConfig, "data": DataConfig, "train": TrainConfig}


def _section(cls: type, values: Any, where: str) -> Any:
    if values is None:
        values = {}
    if not isinstance(values, dict):
        raise TypeError(f"{where} must be a mapping, got {type(values).__name__}")
    allowed = {f.name for f in fields(cls)}
    extra = sorted(set(values) - allowed)
    if extra:
        raise ValueError(f"unknown {where} keys: {extra}")
    return cls(**values)


def load_config(path: str | Path) -> PackBalanceConfig:
    """Parse a YAML file; unknown sections or keys raise ``ValueError``."""
    with open(path, encoding="utf-8") as fh:
        raw = yaml.safe_load(fh) or {}
    return config_from_dict(raw)


def config_from_dict(raw: dict[str, Any]) -> PackBalanceConfig:
    if not isinstance(raw, dict):
        raise TypeError("config root must be a mapping")
    extra = sorted(set(raw) - set(_SECTIONS))
    if extra:
        raise ValueError(f"unknown config sections: {extra}")
    parts = {name: _section(cls, raw.get(name), name) for name, cls in _SECTIONS.items()}
    return PackBalanceConfig(**parts)


def apply_overrides(config: PackBalanceConfig, items: list[str]) -> PackBalanceConfig:
    """``section.key=value`` overrides (value parsed as YAML: ``2``, ``true``, ``bf16``),
    validated like a config file."""
    raw = asdict(config)
    for item in items:
        key, sep, value = item.partition("=")
        section, dot, name = key.partition(".")
        if not sep or not dot or section not in _SECTIONS:
            raise ValueError(f"override {item!r}: expected section.key=value")
        if name not in raw[section]:
            raise ValueError(f"unknown {section} key in override: {name}")
        parsed = yaml.safe_load(value)
        old = raw[section][name]
        if isinstance(old, float) and isinstance(parsed, (int, str)) and not isinstance(parsed, bool):
            try:  # YAML reads "3e-4" as a string and "2" as an int
                parsed = float(parsed)
            except ValueError as exc:
                raise ValueError(f"override {item!r}: {section}.{name} takes a number") from exc
        raw[section][name] = parsed
    return config_from_dict(raw)


def save_config(config: PackBalanceConfig, path: str | Path) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, "w", encoding="utf-8") as fh:
        yaml.safe_dump(asdict(config), fh, sort_keys=False)


def config_to_dict(config: PackBalanceConfig) -> dict[str, Any]:
    return asdict(config)


def replace_section(config: PackBalanceConfig, **sections: Any) -> PackBalanceConfig:
    """Return a copy with whole sections swapped (benches clone configs this way)."""
    return dataclasses.replace(config, **sections)
