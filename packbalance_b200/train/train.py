"""Distributed packed-sequence pretraining entry point.

Usage::

    torchrun --standalone --nproc_per_node=8 -m packbalance_b200.train.train --config configs/bench.yaml

CLI, metrics JSONL records, checkpoint layout, resume semantics and profiler phase
names follow the reference (``train/train.py:175-507``).  Differences:

* the step runs through :class:`~packbalance_b200.train.engine.TrainEngine` (native
  kernels, flat buffers, fused gradient all-reduce);
* step time is device-timed (CUDA events) and the logged throughput uses the max
  over ranks; each log record also carries the measured rank imbalance
  (max rank time / mean rank time - 1) next to the analytical one;
* the host never waits for the step it has just launched: step i's device time and
  scalars are read after step i+1 is enqueued (:class:`LaggedSteps`), the loss
  all-reduce and the cross-rank gather of step times run only at log / save steps,
  and the run's average loss is one all-reduce at the end (the reference calls
  ``.item()`` and synchronises every step, ``train/train.py:364-380``);
* checkpoints carry a commit marker and RNG state, and ``keep_last`` prunes.
"""

from __future__ import annotations

import argparse
import time
from dataclasses import asdict
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist
from torch.profiler import record_function

from packbalance_b200.config import PackBalanceConfig, apply_overrides, load_config, save_config
from packbalance_b200.data.cost import FlopModel
from packbalance_b200.data.dataset import build_dataloader, to_device
from packbalance_b200.data.packer import build_packs, pack_stats
from packbalance_b200.data.sampler import build_schedule
from packbalance_b200.data.store import TokenStore
from packbalance_b200.models.llama import count_parameters
from packbalance_b200.parallel.distributed import cleanup_distributed, init_distributed
from packbalance_b200.profiling.profiler import make_profiler
from packbalance_b200.train.checkpoint import (
    find_latest_checkpoint,
    load_checkpoint,
    restore_rng_state,
    rng_state,
    save_checkpoint,
)
from packbalance_b200.train.engine import TrainEngine
from packbalance_b200.utils import (
    AsyncCheckpointWriter,
    JsonlLogger,
    all_gather_floats,
    get_rank,
    get_world_size,
    is_main_process,
    seed_everything,
)


def _all_reduce_sum(value: torch.Tensor) -> torch.Tensor:
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(value, op=dist.ReduceOp.SUM)
    return value


class LaggedSteps:
    """Step records resolved one step late, so the host never waits for the step it
    has just launched.

    :meth:`launched` is called right after step i's kernels are enqueued; it records
    step i's end event, starts non-blocking copies of the step's device scalars into
    pinned memory (only for records that need them), and returns the records of the
    steps before i, now complete: waiting on step i-1's end event while step i is
    queued behind it keeps the device busy.  :meth:`drain` returns the rest.  Every
    record is returned exactly once, in step order, so ranks that call the
    collectives of a returned record do so at the same steps."""

    def __init__(self, cuda: bool, lag: int = 1) -> None:
        self.cuda = cuda
        self.lag = lag
        self._pending: list[dict] = []
        self._ev0 = None
        self._t0 = 0.0

    def begin(self) -> None:
        """Mark the start of a step (before its kernels are enqueued)."""
        self._t0 = time.perf_counter()
        if self.cuda:
            self._ev0 = torch.cuda.Event(enable_timing=True)
            self._ev0.record()

    def launched(self, record: dict, scalars: dict[str, torch.Tensor] | None = None) -> list[dict]:
        """Attach timing (and, if given, host copies of ``scalars``) to ``record``."""
        entry = {"record": record, "ev0": self._ev0, "t0": self._t0, "names": [], "host": None}
        if self.cuda:
            ev1 = torch.cuda.Event(enable_timing=True)
            ev1.record()
            entry["ev1"] = ev1
        else:
            entry["ms"] = (time.perf_counter() - self._t0) * 1e3
        if scalars:
            names = list(scalars)
            vals = torch.stack([scalars[n].detach().reshape(()).float() for n in names])
            if vals.is_cuda:
                host = torch.empty(vals.shape, dtype=vals.dtype, pin_memory=True)
                host.copy_(vals, non_blocking=True)
            else:
                host = vals.clone()
            entry["names"], entry["host"] = names, host
        self._pending.append(entry)
        out = []
        while len(self._pending) > self.lag:
            out.append(self._resolve(self._pending.pop(0)))
        return out

    def drain(self) -> list[dict]:
        out = [self._resolve(e) for e in self._pending]
        self._pending = []
        return out

    @staticmethod
    def _resolve(entry: dict) -> dict:
        rec = dict(entry["record"])
        if "ev1" in entry:
            entry["ev1"].synchronize()
            rec["step_ms"] = entry["ev0"].elapsed_time(entry["ev1"])
        else:
            rec["step_ms"] = entry["ms"]
        if entry["host"] is not None:
            rec.update({n: float(v) for n, v in zip(entry["names"], entry["host"].tolist())})
        return rec


@torch.no_grad()
def evaluate(engine: TrainEngine, store, val_packs, cfg: PackBalanceConfig, rank: int, world: int) -> dict:
    """Summed validation loss over this rank's strided share, normalised by the global
    useful-token count (reference ``train/train.py:131-172``)."""
    model = engine.model
    device = engine.device
    model.eval()
    idx = list(range(rank, len(val_packs), world))[: cfg.train.eval_steps * cfg.train.grad_accum]
    total = torch.zeros((), device=device, dtype=torch.float32)
    tokens = 0
    if idx:
        for batch in build_dataloader(store, val_packs, cfg.data, idx):
            batch = to_device(batch, device)
            with engine.autocast():
                out = model(
                    batch["input_ids"].unsqueeze(0),
                    labels=batch["labels"].unsqueeze(0),
                    position_ids=batch["position_ids"].unsqueeze(0),
                    doc_ids=batch["doc_ids"].unsqueeze(0),
                    doc_start=batch["doc_start"],
                )
            total += out.loss.float()
            tokens += int(batch["useful_tokens"])
    _all_reduce_sum(total)
    tok = torch.tensor([float(tokens)], device=device, dtype=torch.float64)
    _all_reduce_sum(tok)
    model.train()
    n = int(tok.item())
    return {"val_loss": float(total.item() / n) if n else float("nan"), "val_tokens": n}


def _schedule_for_epoch(train_packs, world, cfg, epoch: int):
    return build_schedule(
        train_packs, world, cfg.train.grad_accum, seed=cfg.data.seed + epoch, mode=cfg.data.schedule
    )


def train(cfg: PackBalanceConfig, device: torch.device, resume: bool = False) -> None:
    rank, world = get_rank(), get_world_size()
    out_dir = Path(cfg.train.output_dir)
    if is_main_process():
        out_dir.mkdir(parents=True, exist_ok=True)
        save_config(cfg, out_dir / "config.yaml")
    seed_everything(cfg.train.seed, cfg.train.deterministic)

    flop_model = FlopModel.from_config(cfg.model)
    store = TokenStore.open(cfg.data.data_dir)
    train_packs = build_packs(store, cfg.data, flop_model, split="train")
    val_packs = build_packs(store, cfg.data, flop_model, split="val") if cfg.data.val_fraction > 0 else []
    stats = pack_stats(train_packs, flop_model)
    if is_main_process():
        print(
            f"[data] {cfg.data.mode}: {stats['num_packs']:,} packs, {stats['useful_tokens']:,} useful tokens, "
            f"padding waste {stats['padding_waste']:.2%}, cost CV {stats['cv']:.3f}",
            flush=True,
        )
    schedule = _schedule_for_epoch(train_packs, world, cfg, 0)
    per_epoch = schedule.steps_per_epoch
    sched_stats = schedule.stats()
    if is_main_process():
        print(
            f"[schedule] steps/epoch={per_epoch:,} step_cost_cv={sched_stats['step_cost_cv']:.3f} "
            f"rank_imbalance={sched_stats['rank_cost_imbalance']:.3f}",
            flush=True,
        )

    latest = find_latest_checkpoint(out_dir) if resume else None
    if cfg.train.compile:
        print("[warn] train.compile is ignored: the native kernels are the compiled path", flush=True)
    engine = TrainEngine(cfg, device)
    model, optimizer = engine.model, engine.optimizer
    start = 0
    if latest is not None:
        meta = load_checkpoint(latest, model, optimizer, fsdp=engine.fsdp, device=device)
        if engine.flat is not None:
            engine.flat.refresh_shadow(force=True)
        start = int(meta.get("step", 0))
        restore_rng_state(meta.get("rng"))
        engine.rebuild_scheduler(start)
        if is_main_process():
            print(f"[resume] loaded {latest} at step {start}", flush=True)

    logger = JsonlLogger(out_dir / "metrics.jsonl")
    writer = AsyncCheckpointWriter()
    if is_main_process():
        logger.log(
            {
                "event": "start",
                "world_size": world,
                "device": str(device),
                "params": count_parameters(model),
                "pack_stats": stats,
                "schedule_stats": sched_stats,
                "config": asdict(cfg),
            }
        )
    prof = None
    if cfg.train.profile:
        prof = make_profiler(out_dir / "profile", wait=1, warmup=cfg.train.profile_warmup, active=cfg.train.profile_steps)
        prof.start()

    epoch, epoch_step = divmod(start, per_epoch) if per_epoch else (0, start)
    if epoch:
        schedule = _schedule_for_epoch(train_packs, world, cfg, epoch)
    A = cfg.train.grad_accum
    loader_iter = iter(build_dataloader(store, train_packs, cfg.data, schedule.rank_indices(rank)[epoch_step * A :]))
    step = start
    run_t0 = time.perf_counter()
    tokens_done, data_ms_sum = 0, 0.0
    window_ms: list[float] = []
    cuda = device.type == "cuda"
    ckpt_root = out_dir / "checkpoints"
    lagged = LaggedSteps(cuda)
    # this rank's summed token loss over the run, reduced once at the end
    loss_acc = torch.zeros((), device=device, dtype=torch.float32)

    def _log(rec: dict) -> None:
        # Runs on every rank for every step, one step late (LaggedSteps); the
        # collective below runs at the same log steps on every rank.
        nonlocal window_ms
        window_ms.append(rec["step_ms"])
        if not rec["log"]:
            return
        per_rank = all_gather_floats([rec["step_ms"]], device)
        times = [r[0] for r in per_rank]
        t_max = max(times)
        tps = rec["tokens"] / max(t_max / 1e3, 1e-9)
        mfu = None
        if cfg.train.peak_tflops > 0:
            mfu = 3.0 * rec["cost"] / (t_max / 1e3) / (world * cfg.train.peak_tflops * 1e12)
        logger.log(
            {
                "step": rec["step"],
                "loss": rec["loss"],
                "lr": rec["lr"],
                "grad_norm": rec["grad_norm"],
                "tokens_per_sec": tps,
                "step_ms": t_max,
                "step_ms_p99_window": float(np.percentile(window_ms, 99)),
                "data_ms": rec["data_ms"],
                "gpu_mem_gb": torch.cuda.max_memory_allocated() / 1e9 if cuda else None,
                "mfu": mfu,
                "usd_per_b_tokens": (1e9 / tps) * (world * cfg.train.gpu_hourly_cost / 3600.0) if tps > 0 else None,
                "tokens": rec["tokens"],
                "cost_cv": sched_stats["step_cost_cv"],
                "rank_imbalance_measured": t_max / (sum(times) / len(times)) - 1.0,
                "skipped": int(rec.get("skipped", 0)),
            }
        )
        window_ms = []
        if cuda:
            torch.cuda.reset_peak_memory_stats()

    def _save(at: int, extra: dict) -> None:
        save_checkpoint(
            model, optimizer, at, ckpt_root, fsdp=engine.fsdp, async_writer=None if engine.fsdp else writer,
            extra={**extra, "rng": rng_state()}, keep_last=cfg.train.keep_last,
        )

    try:
        while step < cfg.train.max_steps:
            if epoch_step >= len(schedule.steps):
                epoch, epoch_step = epoch + 1, 0
                schedule = _schedule_for_epoch(train_packs, world, cfg, epoch)
                loader_iter = iter(build_dataloader(store, train_packs, cfg.data, schedule.rank_indices(rank)))
            plan = schedule.steps[epoch_step]
            d0 = time.perf_counter()
            with record_function("packbalance/data"):
                packs = [next(loader_iter) for _ in range(A)]
            data_ms = (time.perf_counter() - d0) * 1e3
            lagged.begin()
            out = engine.step(packs, plan.step_tokens)
            lr = engine.scheduler.get_last_lr()[0]
            loss_acc += out["loss_sum"].detach().float()
            log_now = step % cfg.train.log_interval == 0
            save_now = bool(cfg.train.save_interval) and (step + 1) % cfg.train.save_interval == 0
            scalars = None
            if log_now or save_now:
                # the loss all-reduce runs only where a value is read, at the same
                # steps on every rank
                scalars = {"loss": engine.global_loss(out["loss_sum"], plan.step_tokens), "grad_norm": out["grad_norm"]}
                if not engine.fsdp:
                    scalars["skipped"] = engine.optimizer.last_skipped
            record = {"step": step, "log": log_now, "tokens": plan.step_tokens, "cost": plan.step_cost,
                      "data_ms": data_ms, "lr": lr}
            for rec in lagged.launched(record, scalars):
                _log(rec)
            tokens_done += plan.step_tokens
            data_ms_sum += data_ms

            if cfg.train.eval_interval and val_packs and (step + 1) % cfg.train.eval_interval == 0:
                metrics = evaluate(engine, store, val_packs, cfg, rank, world)
                if is_main_process():
                    logger.log({"step": step, **metrics})
            if save_now:
                for rec in lagged.drain():
                    _log(rec)
                _save(step + 1, {"loss": float(scalars["loss"]), "tokens": plan.step_tokens})
            if prof is not None:
                prof.step()
            step += 1
            epoch_step += 1
    except KeyboardInterrupt:
        if is_main_process():
            print("[train] interrupted; saving checkpoint", flush=True)
        _save(step, {"interrupted": True})
    finally:
        for rec in lagged.drain():
            _log(rec)
        if prof is not None:
            prof.stop()
        writer.wait()
        total_loss = float(_all_reduce_sum(loss_acc).item())
        if step > start and is_main_process():
            logger.log(
                {
                    "event": "finish",
                    "step": step,
                    "avg_loss": total_loss / max(1, tokens_done),
                    "tokens": tokens_done,
                    "elapsed_s": time.perf_counter() - run_t0,
                    "avg_data_ms": data_ms_sum / max(1, step - start),
                }
            )
        _save(step, {"final": True})
        writer.wait()
        if is_main_process():
            print(f"[train] final checkpoint: {ckpt_root / f'step_{step:07d}'}", flush=True)
        engine.close()
        cleanup_distributed()


def parse_args(argv=None) -> argparse.Namespace:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--config", required=True)
    ap.add_argument("--max-steps", type=int, default=None)
    ap.add_argument("--seed", type=int, default=None)
    ap.add_argument("--output-dir", type=str, default=None)
    ap.add_argument("--device", type=str, default=None)
    ap.add_argument("--resume", action="store_true")
    ap.add_argument("--fsdp", action="store_true")
    ap.add_argument("--compile", action="store_true")
    ap.add_argument("--profile", action="store_true")
    ap.add_argument("--no-fused-ce", action="store_true")
    ap.add_argument("--set", action="append", default=[], metavar="SECTION.KEY=VALUE",
                    help="config override, e.g. train.grad_reduce_dtype=bf16 (repeatable)")
    return ap.parse_args(argv)


def main(argv=None) -> None:
    args = parse_args(argv)
    cfg = apply_overrides(load_config(args.config), args.set)
    if args.max_steps is not None:
        cfg.train.max_steps = args.max_steps
    if args.seed is not None:
        cfg.train.seed = args.seed
    if args.output_dir is not None:
        cfg.train.output_dir = args.output_dir
    if args.fsdp:
        cfg.train.fsdp = True
    if args.compile:
        cfg.train.compile = True
    if args.profile:
        cfg.train.profile = True
    if args.no_fused_ce:
        cfg.model.use_fused_ce = False
    device = init_distributed(args.device, cfg.train.pg_timeout_s)
    train(cfg, device, resume=args.resume or cfg.train.resume)


if __name__ == "__main__":
    main()
