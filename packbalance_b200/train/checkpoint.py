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

        if hasattr(optimizer, "full_state_dict"):
            state = sharded_state_dicts(optimizer)
        else:
            state = {"model": model.state_dict(), "optimizer": optimizer.state_dict()}
        dcp.save(state, checkpoint_id=str(ckpt_dir / "dcp"))
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
    if fsdp and dist.is_available() and dist.is_initialized() and hasattr(optimizer, "full_state_dict"):
        load_sharded_dcp(optimizer, ckpt / "dcp")
        meta_file = ckpt / META
        return json.loads(meta_file.read_text(encoding="utf-8")) if meta_file.exists() else {}
    if fsdp and dist.is_available() and dist.is_initialized():
        import torch.distributed.checkpoint as dcp

        state = {"model": model.state_dict(), "optimizer": optimizer.state_dict() if optimizer is not None else {}}
        current_groups = [dict(g) for g in state["optimizer"].get("param_groups", [])]
        # param-group fields the writer did not have (a run without an LR scheduler has
        # no ``initial_lr``) are not requested; they keep this run's values
        saved = dcp.FileSystemReader(str(ckpt / "dcp")).read_metadata().state_dict_metadata
        for i, g in enumerate(state["optimizer"].get("param_groups", [])):
            for k in [k for k in g if k != "params" and f"optimizer.param_groups.{i}.{k}" not in saved]:
                del g[k]
        dcp.load(state, checkpoint_id=str(ckpt / "dcp"))
        model.load_state_dict(state["model"])
        if optimizer is not None:
            for g, cur in zip(state["optimizer"].get("param_groups", []), current_groups):
                for k, v in cur.items():
                    g.setdefault(k, v)
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


# ---- native sharded engine ------------------------------------------------------------
def sharded_state_dicts(optimizer) -> dict[str, Any]:
    """DCP state of the native sharded engine: full tensors under the reference's keys
    (``model.<name>``, ``optimizer.state.<i>.{step,exp_avg,exp_avg_sq}``,
    ``optimizer.param_groups``).  Each parameter is written by one rank (index % W), so
    no rank holds more than its share of the model on the host.  Collective."""
    sp = optimizer.sp
    model = sp.full_tensors("param", owner_only=True)
    optim = optimizer.full_state_dict(owner_only=True)
    if dist.get_rank() != 0:
        optim.pop("param_groups")
    return {"model": model, "optimizer": optim}


def load_sharded_dcp(optimizer, dcp_dir: Path) -> None:
    """Inverse of :func:`sharded_state_dicts`, one sharding unit at a time (bounded host
    memory).  Collective: every rank reads every tensor of a unit and keeps its chunk."""
    import torch.distributed.checkpoint as dcp

    sp = optimizer.sp
    order = sp.model_order()
    index = {s.name: i for i, s in enumerate(order)}
    groups = [sp.rep_slots] + [u.slots for u in sp.units]
    step = 0.0
    for slots in groups:
        model = {s.name: torch.empty(s.shape, dtype=torch.float32) for s in slots}
        state = {
            index[s.name]: {"step": torch.zeros(()), "exp_avg": torch.empty(s.shape, dtype=torch.float32),
                            "exp_avg_sq": torch.empty(s.shape, dtype=torch.float32)}
            for s in slots
        }
        dcp.load({"model": model, "optimizer": {"state": state}}, checkpoint_id=str(dcp_dir))
        sp.load_full_tensors(model, "param")
        sp.load_full_tensors({s.name: state[index[s.name]]["exp_avg"] for s in slots}, "exp_avg")
        sp.load_full_tensors({s.name: state[index[s.name]]["exp_avg_sq"] for s in slots}, "exp_avg_sq")
        step = max([step] + [float(st["step"]) for st in state.values()])
    # param_groups entries are stored one key per field (optimizer.param_groups.0.<k>)
    prefix = "optimizer.param_groups.0."
    keys = [k[len(prefix):] for k in dcp.FileSystemReader(str(dcp_dir)).read_metadata().state_dict_metadata
            if k.startswith(prefix)]
    group = {k: None for k in keys}
    if group:
        dcp.load({"optimizer": {"param_groups": [group]}}, checkpoint_id=str(dcp_dir))
    optimizer.step_count = int(step)
    for k, v in group.items():
        if k != "params":
            optimizer.param_groups[0][k] = v
