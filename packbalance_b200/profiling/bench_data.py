"""Data-loader throughput: useful / compute tokens per second vs worker count.

    python -m packbalance_b200.profiling.bench_data --config configs/bench.yaml
        [--modes pad,pack_random,pack_ffd,isoflop] [--workers 0,2,4,8]
        [--num-batches 50] [--warmup 5] [--prepare] [--output artifacts/data_bench.json]

Times the per-rank loader alone (memory-mapped token store -> pack tensors, no model),
on the single-rank schedule of each packing mode, and reports padding waste and the
schedule's step-cost CV beside it.  Same CLI and output fields as the reference's
``profiling/bench_data.py`` (``_bench_loader`` 24-52, ``main`` 55-113); rows also carry
``doc_start``, the extra key this framework's attention kernel reads.
"""

from __future__ import annotations

import argparse
import json
import time
from dataclasses import replace
from pathlib import Path

from packbalance_b200.config import load_config
from packbalance_b200.data.cost import FlopModel
from packbalance_b200.data.dataset import build_dataloader
from packbalance_b200.data.packer import build_packs, pack_stats
from packbalance_b200.data.prepare import prepare_synthetic
from packbalance_b200.data.sampler import build_schedule
from packbalance_b200.data.store import TokenStore


def time_loader(store, packs, data_cfg, indices: list[int], num_batches: int, warmup: int) -> dict:
    loader = build_dataloader(store, packs, data_cfg, indices)

    def batches():
        while True:
            yield from loader

    it = batches()
    for _ in range(warmup):
        next(it)
    useful = compute = 0
    t0 = time.perf_counter()
    for _ in range(num_batches):
        b = next(it)
        useful += int(b["useful_tokens"])
        compute += int(b["compute_tokens"])
    dt = time.perf_counter() - t0
    return {"useful_tokens": useful, "compute_tokens": compute, "useful_tokens_per_s": useful / dt,
            "compute_tokens_per_s": compute / dt, "packs_per_s": num_batches / dt,
            "mean_batch_ms": 1e3 * dt / num_batches}


def main(argv: list[str] | None = None) -> list[dict]:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", required=True)
    ap.add_argument("--modes", default="pad,pack_random,pack_ffd,isoflop")
    ap.add_argument("--workers", default="0,2,4,8")
    ap.add_argument("--num-batches", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--prepare", action="store_true")
    ap.add_argument("--output", default="artifacts/data_bench.json")
    args = ap.parse_args(argv)
    cfg = load_config(args.config)
    data_dir = Path(cfg.data.data_dir)
    if args.prepare or not (data_dir / "meta.json").exists():
        prepare_synthetic(cfg.data, data_dir)
    store = TokenStore.open(data_dir)
    fm = FlopModel.from_config(cfg.model)
    rows = []
    print(f"{'mode':<12} {'workers':>7} {'useful tok/s':>14} {'compute tok/s':>14} {'packs/s':>9} "
          f"{'batch ms':>9} {'waste':>7} {'cost cv':>8}")
    for mode in [m.strip() for m in args.modes.split(",") if m.strip()]:
        dcfg = replace(cfg.data, mode=mode)
        packs = build_packs(store, dcfg, fm, split="train")
        stats = pack_stats(packs, fm)
        sched = build_schedule(packs, world_size=1, grad_accum=1, seed=cfg.data.seed, mode=cfg.data.schedule)
        cv = sched.stats()["step_cost_cv"]
        for w in [int(x) for x in args.workers.split(",") if x.strip()]:
            run_cfg = replace(dcfg, num_workers=w, pin_memory=False, persistent_workers=w > 0)
            m = time_loader(store, packs, run_cfg, sched.rank_indices(0), args.num_batches, args.warmup)
            rows.append({"mode": mode, "workers": w, **m, "padding_waste": stats["padding_waste"],
                         "pack_cost_cv": stats["cv"], "step_cost_cv": cv})
            print(f"{mode:<12} {w:>7} {m['useful_tokens_per_s']:>14,.0f} {m['compute_tokens_per_s']:>14,.0f} "
                  f"{m['packs_per_s']:>9.1f} {m['mean_batch_ms']:>9.2f} {stats['padding_waste']:>6.1%} {cv:>8.3f}")
    out = Path(args.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(rows, indent=2), encoding="utf-8")
    print(f"\nwrote {out}")
    return rows


if __name__ == "__main__":
    main()
