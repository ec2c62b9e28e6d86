"""Scheduler ablation: round-robin vs the cost-balanced two-level scheduler.

    python -m packbalance_b200.profiling.bench_schedule --config configs/bench.yaml
        [--modes pad,pack_random,pack_ffd,isoflop] [--schedules random,balanced]
        [--world-size 8] [--prepare] [--output artifacts/schedule_bench.json]

Analytical only (no model, no GPU): for every packing mode and schedule policy, the
step-cost coefficient of variation, p99/mean step cost and the rank cost imbalance
(max rank cost / mean - 1) of the schedule that W ranks with ``grad_accum`` packs each
would run.  Same CLI and output fields as the reference's ``profiling/bench_schedule.py``
(``main`` 22-66).
"""

from __future__ import annotations

import argparse
import json
from dataclasses import replace
from pathlib import Path

from packbalance_b200.config import load_config
from packbalance_b200.data.cost import FlopModel
from packbalance_b200.data.packer import build_packs
from packbalance_b200.data.prepare import prepare_synthetic
from packbalance_b200.data.sampler import build_schedule
from packbalance_b200.data.store import TokenStore


def _csv(s: str) -> list[str]:
    return [x.strip() for x in s.split(",") if x.strip()]


def run(cfg, modes: list[str], schedules: list[str], world_size: int) -> list[dict]:
    store = TokenStore.open(cfg.data.data_dir)
    fm = FlopModel.from_config(cfg.model)
    rows = []
    for mode in modes:
        packs = build_packs(store, replace(cfg.data, mode=mode), fm, split="train")
        for policy in schedules:
            sched = build_schedule(packs, world_size=world_size, grad_accum=cfg.train.grad_accum,
                                   seed=cfg.data.seed, mode=policy)
            rows.append({"mode": mode, "schedule": policy, **sched.stats()})
    return rows


def main(argv: list[str] | None = None) -> list[dict]:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", required=True)
    ap.add_argument("--modes", default="pad,pack_random,pack_ffd,isoflop")
    ap.add_argument("--schedules", default="random,balanced")
    ap.add_argument("--world-size", type=int, default=8)
    ap.add_argument("--prepare", action="store_true")
    ap.add_argument("--output", default="artifacts/schedule_bench.json")
    args = ap.parse_args(argv)
    cfg = load_config(args.config)
    data_dir = Path(cfg.data.data_dir)
    if args.prepare or not (data_dir / "meta.json").exists():
        prepare_synthetic(cfg.data, data_dir)
    rows = run(cfg, _csv(args.modes), _csv(args.schedules), args.world_size)
    print(f"{'mode':<12} {'schedule':<9} {'steps':>6} {'step cv':>8} {'p99/mean':>9} {'rank imb':>9} {'tokens':>12}")
    for r in rows:
        print(f"{r['mode']:<12} {r['schedule']:<9} {r['steps']:>6} {r['step_cost_cv']:>8.4f} "
              f"{r['step_cost_p99_over_mean']:>9.4f} {r['rank_cost_imbalance']:>9.4f} {r['tokens']:>12,}")
    out = Path(args.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(rows, indent=2), encoding="utf-8")
    print(f"\nwrote {out}")
    return rows


if __name__ == "__main__":
    main()
