"""Shared helpers: seeding, rank queries, formatting, timers, rank-0 JSONL logging and
a background checkpoint writer.

Public names mirror the reference's ``packbalance/utils.py:18-227`` (same
signatures, same console format for the logger) so callers can switch imports.
Additions: :class:`DeviceTimer` (CUDA-event timing on the launching stream) and
:func:`all_reduce_max` (max over ranks, the aggregation every multi-GPU number in
this framework uses).
"""

from __future__ import annotations

import contextlib
import json
import os
import random
import threading
import time
from pathlib import Path
from typing import Any

import numpy as np
import torch
import torch.distributed as dist

_CONSOLE_KEYS = (
    "loss",
    "lr",
    "grad_norm",
    "tokens_per_sec",
    "step_ms",
    "data_ms",
    "gpu_mem_gb",
    "mfu",
    "usd_per_b_tokens",
)


def seed_everything(seed: int, deterministic: bool = False) -> None:
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
    if deterministic:
        torch.backends.cudnn.deterministic = True
        torch.backends.cudnn.benchmark = False


def _pg_ready() -> bool:
    return dist.is_available() and dist.is_initialized()


def get_rank() -> int:
    return dist.get_rank() if _pg_ready() else int(os.environ.get("RANK", "0"))


def get_world_size() -> int:
    return dist.get_world_size() if _pg_ready() else int(os.environ.get("WORLD_SIZE", "1"))


def get_local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK", "0"))


def is_distributed() -> bool:
    return get_world_size() > 1


def is_main_process() -> bool:
    return get_rank() == 0


def barrier() -> None:
    if _pg_ready():
        dist.barrier()


def human_int(n: float) -> str:
    for suffix, scale in (("T", 1e12), ("B", 1e9), ("M", 1e6), ("K", 1e3)):
        if abs(n) >= scale:
            return f"{n / scale:.2f}{suffix}"
    return f"{n:.0f}"


def human_bytes(n: float) -> str:
    units = ("B", "KiB", "MiB", "GiB", "TiB")
    for i, unit in enumerate(units):
        if abs(n) < 1024 or i == len(units) - 1:
            return f"{n:.1f}{unit}"
        n /= 1024
    return f"{n:.1f}TiB"


def format_duration(seconds: float) -> str:
    total = max(0, int(seconds))
    hours, rest = divmod(total, 3600)
    minutes, secs = divmod(rest, 60)
    if hours:
        return f"{hours}h{minutes:02d}m{secs:02d}s"
    if minutes:
        return f"{minutes}m{secs:02d}s"
    return f"{secs}s"


def ensure_dir(path: str | Path) -> Path:
    p = Path(path)
    p.mkdir(parents=True, exist_ok=True)
    return p


def _cuda_sync() -> None:
    if torch.cuda.is_available():
        torch.cuda.synchronize()


class CudaTimer:
    """Wall-clock timer with a device synchronize at both ends (reference API)."""

    def __init__(self, enabled: bool = True) -> None:
        self.enabled = enabled
        self.elapsed_ms = 0.0
        self._t0 = 0.0

    def __enter__(self) -> CudaTimer:
        if self.enabled:
            _cuda_sync()
            self._t0 = time.perf_counter()
        return self

    def __exit__(self, *exc: object) -> None:
        if self.enabled:
            _cuda_sync()
            self.elapsed_ms = (time.perf_counter() - self._t0) * 1e3


class DeviceTimer:
    """CUDA-event timer on the current stream; falls back to wall clock on CPU.

    ``elapsed_ms`` is valid after ``__exit__`` (which synchronizes the end event).
    """

    def __init__(self, device: torch.device | None = None) -> None:
        self.device = device if device is not None else torch.device("cpu")
        self.elapsed_ms = 0.0
        self._cuda = self.device.type == "cuda"
        if self._cuda:
            self._start = torch.cuda.Event(enable_timing=True)
            self._end = torch.cuda.Event(enable_timing=True)

    def __enter__(self) -> DeviceTimer:
        if self._cuda:
            self._start.record()
        else:
            self._t0 = time.perf_counter()
        return self

    def __exit__(self, *exc: object) -> None:
        if self._cuda:
            self._end.record()
            self._end.synchronize()
            self.elapsed_ms = float(self._start.elapsed_time(self._end))
        else:
            self.elapsed_ms = (time.perf_counter() - self._t0) * 1e3


@contextlib.contextmanager
def nullcontext():
    yield None


def elapsed_ms(fn) -> float:
    _cuda_sync()
    t0 = time.perf_counter()
    fn()
    _cuda_sync()
    return (time.perf_counter() - t0) * 1e3


def all_reduce_max(value: float, device: torch.device | None = None) -> float:
    """Max of a host scalar over all ranks (identity without a process group)."""
    if not _pg_ready():
        return float(value)
    dev = device if device is not None else torch.device("cpu")
    if dist.get_backend() == "nccl" and dev.type != "cuda":
        dev = torch.device("cuda", torch.cuda.current_device())
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_gather_floats(values: list[float], device: torch.device | None = None) -> list[list[float]]:
    """Gather an equal-length float list from every rank -> [world][len]."""
    if not _pg_ready():
        return [list(values)]
    dev = device if device is not None else torch.device("cpu")
    if dist.get_backend() == "nccl" and dev.type != "cuda":
        dev = torch.device("cuda", torch.cuda.current_device())
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [o.tolist() for o in out]


class JsonlLogger:
    """Rank-0 JSONL metrics file plus a readable console line per step record.

    The file is truncated when the logger is created; console output matches the
    reference logger (``utils.py:127-165``).
    """

    def __init__(self, path: str | Path | None = None, enabled: bool = True) -> None:
        self.enabled = enabled and is_main_process()
        self.path = Path(path) if path is not None else None
        if self.enabled and self.path is not None:
            self.path.parent.mkdir(parents=True, exist_ok=True)
            self.path.write_text("", encoding="utf-8")

    def log(self, record: dict[str, Any]) -> None:
        if not self.enabled:
            return
        line = json.dumps(record, sort_keys=True)
        if self.path is not None:
            with open(self.path, "a", encoding="utf-8") as fh:
                fh.write(line + "\n")
        if "step" not in record:
            print(line, flush=True)
            return
        parts = [f"step {record['step']}"]
        for key in _CONSOLE_KEYS:
            value = record.get(key)
            if value is None:
                continue
            parts.append(f"{key}={value:.4g}" if isinstance(value, float) else f"{key}={value}")
        print(" | ".join(parts), flush=True)


def _to_cpu(value: Any) -> Any:
    if isinstance(value, torch.Tensor):
        return value.detach().to("cpu", copy=True)
    if isinstance(value, dict):
        return {k: _to_cpu(v) for k, v in value.items()}
    if isinstance(value, (list, tuple)):
        return type(value)(_to_cpu(v) for v in value)
    return value


class AsyncCheckpointWriter:
    """Snapshot a state dict to host memory, then write it on a background thread.

    The write is atomic (``<path>.tmp`` then ``os.replace``).  ``on_done`` runs on
    the writer thread after the rename, which is where the checkpoint commit
    marker is written, so a crash mid-write never leaves a directory that looks
    complete.
    """

    def __init__(self) -> None:
        self._thread: threading.Thread | None = None
        self._error: BaseException | None = None

    def busy(self) -> bool:
        return self._thread is not None and self._thread.is_alive()

    def submit(self, state: dict[str, Any], path: str | Path, on_done=None) -> bool:
        if self.busy():
            return False
        target = Path(path)
        target.parent.mkdir(parents=True, exist_ok=True)
        snapshot = _to_cpu(state)

        def _run() -> None:
            try:
                tmp = target.with_suffix(target.suffix + ".tmp")
                torch.save(snapshot, tmp)
                os.replace(tmp, target)
                if on_done is not None:
                    on_done()
            except BaseException as exc:  # surfaced by wait()
                self._error = exc

        self._thread = threading.Thread(target=_run, name="packbalance-ckpt", daemon=True)
        self._thread.start()
        return True

    def wait(self) -> None:
        if self._thread is not None:
            self._thread.join()
            self._thread = None
        if self._error is not None:
            err, self._error = self._error, None
            raise RuntimeError("asynchronous checkpoint write failed") from err


def get_autocast_dtype(dtype: str) -> torch.dtype | None:
    return {"bf16": torch.bfloat16, "fp16": torch.float16}.get(dtype)


def count_parameters(model: torch.nn.Module, trainable_only: bool = False) -> int:
    return sum(p.numel() for p in model.parameters() if p.requires_grad or not trainable_only)
