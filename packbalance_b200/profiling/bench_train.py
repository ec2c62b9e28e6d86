"""End-to-end step time across packing modes (single process).

    python -m packbalance_b200.profiling.bench_train --config configs/bench.yaml
        [--modes pad,pack_random,pack_ffd,isoflop] [--steps N] [--warmup 3]
        [--device cuda|cpu] [--prepare] [--output artifacts/train_bench.json]

Same model, optimizer and token budget for every mode; only the way documents become
sequences changes, so useful tokens/s (tokens the loss uses) is the comparison.  Each
mode builds its packs, a one-rank schedule of ``grad_accum`` packs per step, a fresh
model and :class:`~packbalance_b200.train.engine.TrainEngine`, and times
``engine.step`` (data loading and the host->device copy included) after ``--warmup``
steps.  On CUDA the step time is device time from CUDA events on the launching stream
(a synchronize on both sides); on CPU it is wall time.  Output fields follow the
reference's ``profiling/bench_train.py`` (``bench_mode`` 54-163): useful / compute
tokens/s, p50 / p99 step ms, peak memory, MFU, $ per billion useful tokens, padding
waste, pack and step cost CV, analytical rank imbalance.
"""

from __future__ import annotations

import argparse
import gc
import json
import time
from dataclasses import replace
from pathlib import Path

import numpy as np
import torch

from packbalance_b200.config import load_config
from packbalance_b200.data.cost import FlopModel
from packbalance_b200.data.dataset import build_dataloader
from packbalance_b200.data.packer import build_packs, pack_stats
from packbalance_b200.data.prepare import prepare_synthetic
from packbalance_b200.data.sampler import build_schedule
from packbalance_b200.data.store import TokenStore
from packbalance_b200.train.engine import TrainEngine
from packbalance_b200.utils import seed_everything


def bench_mode(cfg, mode: str, store: TokenStore, fm: FlopModel, device: torch.device, steps: int,
               warmup: int) -> dict:
    dcfg = replace(cfg.data, mode=mode)
    packs = build_packs(store, dcfg, fm, split="train")
    stats = pack_stats(packs, fm)
    A = cfg.train.grad_accum
    sched = build_schedule(packs, world_size=1, grad_accum=A, seed=cfg.data.seed, mode=cfg.data.schedule)
    steps = min(steps, len(sched.steps))
    if steps <= 0:
        raise ValueError(f"no schedule steps for mode {mode}")
    warmup = min(warmup, len(sched.steps) - steps)
    indices = sched.rank_indices(0)[: (warmup + steps) * A]
    it = iter(build_dataloader(store, packs, dcfg, indices))
    seed_everything(cfg.train.seed)
    engine = TrainEngine(replace(cfg, data=dcfg), device)
    cuda = device.type == "cuda"
    if cuda:
        torch.cuda.reset_peak_memory_stats(device)
    times, data_ms = [], []
    for s in range(warmup + steps):
        plan = sched.steps[s]
        d0 = time.perf_counter()
        local = [next(it) for _ in range(A)]
        d1 = time.perf_counter()
        if cuda:
            torch.cuda.synchronize(device)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            engine.step(local, plan.step_tokens)
            e1.record()
            torch.cuda.synchronize(device)
            ms = e0.elapsed_time(e1)
        else:
            t0 = time.perf_counter()
            engine.step(local, plan.step_tokens)
            ms = (time.perf_counter() - t0) * 1e3
        if s >= warmup:
            times.append(ms)
            data_ms.append((d1 - d0) * 1e3)
    timed_plans = sched.steps[warmup: warmup + steps]
    total_s = sum(times) / 1e3
    useful = sum(p.step_tokens for p in timed_plans)
    compute = sum(p.step_compute_tokens for p in timed_plans)
    flops = 3.0 * sum(p.step_cost for p in timed_plans)
    ups = useful / total_s
    st = sched.stats()
    out = {
        "mode": mode,
        "num_packs": len(packs),
        "steps": steps,
        "padding_waste": stats["padding_waste"],
        "pack_cost_cv": stats["cv"],
        "step_cost_cv": st["step_cost_cv"],
        "rank_cost_imbalance": st["rank_cost_imbalance"],
        "useful_tokens_per_s": ups,
        "compute_tokens_per_s": compute / total_s,
        "useful_tokens_per_step": useful / steps,
        "compute_tokens_per_step": compute / steps,
        "step_ms_p50": float(np.percentile(times, 50)),
        "step_ms_p99": float(np.percentile(times, 99)),
        "data_ms_mean": float(np.mean(data_ms)),
        "peak_gpu_gb": torch.cuda.max_memory_allocated(device) / 1e9 if cuda else 0.0,
        "mfu": flops / total_s / (cfg.train.peak_tflops * 1e12) if cfg.train.peak_tflops > 0 else float("nan"),
        "usd_per_b_tokens": (1e9 / ups) * (cfg.train.gpu_hourly_cost / 3600.0) if cfg.train.gpu_hourly_cost > 0 else 0.0,
        "timing": "cuda events" if cuda else "wall clock",
    }
    engine.close()
    del engine
    gc.collect()
    if cuda:
        torch.cuda.empty_cache()
    return out


def main(argv: list[str] | None = None) -> list[dict]:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", required=True)
    ap.add_argument("--modes", default="pad,pack_random,pack_ffd,isoflop")
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--prepare", action="store_true")
    ap.add_argument("--output", default="artifacts/train_bench.json")
    args = ap.parse_args(argv)
    cfg = load_config(args.config)
    steps = args.steps if args.steps is not None else cfg.train.max_steps
    data_dir = Path(cfg.data.data_dir)
    if args.prepare or not (data_dir / "meta.json").exists():
        prepare_synthetic(cfg.data, data_dir)
    store = TokenStore.open(data_dir)
    fm = FlopModel.from_config(cfg.model)
    device = torch.device(args.device)
    rows = []
    for mode in [m.strip() for m in args.modes.split(",") if m.strip()]:
        print(f"\n=== {mode} ===", flush=True)
        r = bench_mode(cfg, mode, store, fm, device, steps, args.warmup)
        rows.append(r)
        print(json.dumps(r, indent=2), flush=True)
    out = Path(args.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(rows, indent=2), encoding="utf-8")
    print(f"\n{'mode':<12} {'waste':>7} {'step cv':>8} {'useful tok/s':>14} {'p50 ms':>8} {'p99 ms':>8} "
          f"{'peak GB':>8} {'MFU':>7} {'$/B tok':>8}")
    for r in rows:
        print(f"{r['mode']:<12} {r['padding_waste']:>6.1%} {r['step_cost_cv']:>8.3f} {r['useful_tokens_per_s']:>14,.0f} "
              f"{r['step_ms_p50']:>8.1f} {r['step_ms_p99']:>8.1f} {r['peak_gpu_gb']:>8.2f} {r['mfu']:>7.3f} "
              f"{r['usd_per_b_tokens']:>8.2f}")
    print(f"\nwrote {out}")
    return rows


if __name__ == "__main__":
    main()
