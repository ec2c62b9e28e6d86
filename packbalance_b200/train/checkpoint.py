"""Checkpoints in the reference's on-disk format, with a commit marker and pruning.

Layout (reference ``train/checkpoint.py:31-105``)::

    <output_dir>/checkpoints/step_{step:07d}/state.pt   (single process / DDP, rank 0)
        {"model": state_dict, "optimizer": AdamW-format state_dict, "step": int, "extra": dict}
    <output_dir>/checkpoints/step_{step:07d}/dcp/        (FSDP: torch.distributed.checkpoint)
    <output_dir>/checkpoints/step_{step:07d}/meta.json   {"step": step, **extra}

Differences that close the reference's failure windows (all backward compatible):

* ``meta.json`` is written *after* ``state.pt`` (or the DCP save) is durable, so it is
  a commit marker; :func:`find_latest_checkpoint` only returns committed directories
  and skips torn ones left by a crash mid-write.
* ``keep_last`` (declared but unused in the reference) prunes older committed
  directories.
* ``extra`` carries the RNG states so a resumed run continues the same random stream.
"""

from __future__ import annotations

import json
import os
import random
import shutil
from pathlib import Path
from typing import Any

import numpy as np
import torch
import torch.distributed as dist

from packbalance_b200.utils import AsyncCheckpointWriter, is_main_process

META = "meta.json"


def _step_of(p: Path) -> int:
    try:
        return int(p.name.split("_")[-1])
    except ValueError:
        return -1


def committed_checkpoints(root: Path) -> list[Path]:
    if not root.exists():
        return []
    dirs = [p for p in root.iterdir() if p.is_dir() and p.name.startswith("step_") and _step_of(p) >= 0]
    return sorted((p for p in dirs if (p / META).exists()), key=_step_of)


def _latest_step_dir(root: Path) -> Path | None:
    done = committed_checkpoints(root)
    return done[-1] if done else None


def find_latest_checkpoint(output_dir: str | Path) -> Path | None:
    return _latest_step_dir(Path(output_dir) / "checkpoints")


def _write_meta(ckpt_dir: Path, step: int, extra: dict[str, Any] | None) -> None:
    meta = {"step": step, **{k: v for k, v in (extra or {}).items() if k != "rng"}}
    tmp = ckpt_dir / (META + ".tmp")
    tmp.write_text(json.dumps(meta, indent=2), encoding="utf-8")
    os.replace(tmp, ckpt_dir / META)


def prune_checkpoints(root: Path, keep_last: int) -> None:
    if keep_last <= 0 or not is_main_process():
        return
    for old in committed_checkpoints(root)[:-keep_last]:
        shutil.rmtree(old, ignore_errors=True)


def rng_state() -> dict[str, Any]:
    state = {"python": random.getstate(), "numpy": np.random.get_state(), "torch": torch.get_rng_state()}
    if torch.cuda.is_available():
        state["cuda"] = torch.cuda.get_rng_state_all()
    return state


def restore_rng_state(state: dict[str, Any] | None) -> None:
    if not state:
        return
    random.setstate(state["python"])
    np.random.set_state(state["numpy"])
    torch.set_rng_state(state["torch"])
    if "cuda" in state and torch.cuda.is_available() and len(state["cuda"]) == torch.cuda.device_count():
        torch.cuda.set_rng_state_all(state["cuda"])


def save_checkpoint(
    model: torch.nn.Module,
    optimizer: torch.optim.Optimizer,
    step: int,
    output_dir: str | Path,
    *,
    fsdp: bool,
    async_writer: AsyncCheckpointWriter | None = None,
    extra: dict[str, Any] | None = None,
    keep_last: int = 0,
) -> Path:
    root = Path(output_dir)
    ckpt_dir = root / f"step_{step:07d}"
    ckpt_dir.mkdir(parents=True, exist_ok=True)
    if fsdp and dist.is_available() and dist.is_initialized():
        import torch.distributed.checkpoint as dcp

        dcp.save({"model": model.state_dict(), "optimizer": optimizer.state_dict()}, checkpoint_id=str(ckpt_dir / "dcp"))
        dist.barrier()
        if is_main_process():
            _write_meta(ckpt_dir, step, extra)
            prune_checkpoints(root, keep_last)
        return ckpt_dir
    if not is_main_process():
        return ckpt_dir
    raw = getattr(model, "module", model)
    state = {"model": raw.state_dict(), "optimizer": optimizer.state_dict(), "step": step, "extra": extra or {}}
    path = ckpt_dir / "state.pt"

    def commit() -> None:
        _write_meta(ckpt_dir, step, extra)
        prune_checkpoints(root, keep_last)

    if async_writer is not None:
        if not async_writer.submit(state, path, on_done=commit):
            async_writer.wait()
            async_writer.submit(state, path, on_done=commit)
    else:
        tmp = path.with_suffix(".pt.tmp")
        torch.save(state, tmp)
        os.replace(tmp, path)
        commit()
    return ckpt_dir


def load_checkpoint(
    path: str | Path,
    model: torch.nn.Module,
    optimizer: torch.optim.Optimizer | None,
    *,
    fsdp: bool,
    device: torch.device,
) -> dict[str, Any]:
    """Load model (+ optimizer) state in place; returns ``{"step", **extra}``."""
    ckpt = Path(path)
    if fsdp and dist.is_available() and dist.is_initialized():
        import torch.distributed.checkpoint as dcp

        state = {"model": model.state_dict(), "optimizer": optimizer.state_dict() if optimizer is not None else {}}
        dcp.load(state, checkpoint_id=str(ckpt / "dcp"))
        model.load_state_dict(state["model"])
        if optimizer is not None:
            optimizer.load_state_dict(state["optimizer"])
        meta_file = ckpt / META
        return json.loads(meta_file.read_text(encoding="utf-8")) if meta_file.exists() else {}
    raw = getattr(model, "module", model)
    state = torch.load(ckpt / "state.pt", map_location="cpu", weights_only=False)
    with torch.no_grad():
        own = raw.state_dict()
        for key, value in state["model"].items():
            if key not in own:
                raise KeyError(f"unexpected key in checkpoint: {key}")
            own[key].copy_(value)
        missing = set(own) - set(state["model"])
        if missing:
            raise KeyError(f"checkpoint is missing keys: {sorted(missing)}")
    if optimizer is not None and "optimizer" in state:
        optimizer.load_state_dict(state["optimizer"])
    return {"step": int(state.get("step", 0)), **state.get("extra", {})}
