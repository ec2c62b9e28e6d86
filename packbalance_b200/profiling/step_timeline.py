"""Per-rank kernel timeline of one training step: where the communication overlaps compute.

    python -m packbalance_b200.profiling.step_timeline [--config configs/b2_100m.yaml]
    torchrun --nproc-per-node N -m packbalance_b200.profiling.step_timeline --output-dir T

Builds the benchmark's engine and data (benchmark config #2 by default), runs warm-up steps
(so the step is a CUDA-graph replay where the engine captures one), then records two steps
with ``torch.profiler`` (CUPTI kernel records, device timestamps) and summarises the second
one per rank into ``<output-dir>/step_timeline_w{W}_r{rank}.json``:

* ``step_span_us``: first kernel start to last kernel end of the step;
* ``collectives``: start (relative to the step), duration and the compute time that ran
  beside each collective kernel (``allreduce`` / ``reduce_scatter`` / ``fsdp_adamw``);
* ``optimizer_start_us``: start of the AdamW kernel, i.e. the end of the gradient phase;
* ``main_stream_gaps_us``: idle time of the stream that runs the attention backward;
* ``top_kernels``: summed device time per kernel name.

``--trace`` also writes the Chrome trace.  Device times under the profiler are close to
the undisturbed ones (no replay, no counters), but the numbers of record are bench.py's.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist
from torch.profiler import ProfilerActivity, profile

ROOT = Path(__file__).resolve().parents[2]
COLLECTIVE = ("allreduce", "reduce_scatter", "fsdp_adamw")


def summarize(events: list[tuple[float, float, str, int]]) -> dict:
    """``events``: (start_us, end_us, name, stream) of one step's device activities."""
    events = sorted(events)
    t0 = events[0][0]
    comm = [e for e in events if any(c in e[2] for c in COLLECTIVE)]
    comp = [e for e in events if not any(c in e[2] for c in COLLECTIVE)]

    def beside(c):
        return sum(max(0.0, min(c[1], e[1]) - max(c[0], e[0])) for e in comp)

    attn_streams = {e[3] for e in comp if "attn_bwd" in e[2]}
    main = [e for e in comp if e[3] in attn_streams]
    gaps = sum(max(0.0, b[0] - a[1]) for a, b in zip(main, main[1:]))
    adam = [e for e in events if "adamw" in e[2]]
    agg: dict[str, list[float]] = {}
    for e in comp:
        a = agg.setdefault(e[2][:90], [0, 0.0])
        a[0] += 1
        a[1] += e[1] - e[0]
    return {
        "step_span_us": round(events[-1][1] - t0, 1),
        "collectives": [{"start_us": round(c[0] - t0, 1), "dur_us": round(c[1] - c[0], 1),
                         "compute_beside_us": round(beside(c), 1), "name": c[2][:60]} for c in comm],
        "optimizer_start_us": round(adam[0][0] - t0, 1) if adam else None,
        "main_stream_gaps_us": round(gaps, 1),
        "top_kernels": [{"name": n, "count": v[0], "us": round(v[1], 1)}
                        for n, v in sorted(agg.items(), key=lambda kv: -kv[1][1])[:25]],
    }


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--config", default=str(ROOT / "configs" / "b2_100m.yaml"))
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--output-dir", default="artifacts/timeline")
    ap.add_argument("--trace", action="store_true")
    args = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    sys.path.insert(0, str(ROOT))
    import bench

    from packbalance_b200.config import load_config
    from packbalance_b200.data.dataset import PackedDataset, concat_packs
    from packbalance_b200.train.engine import TrainEngine, to_device_batch

    cfg = load_config(args.config)
    total = args.warmup + 2
    store, packs, sched, _ = bench.build_data(cfg, cfg.data.mode, world, rank, total)
    ds = PackedDataset(store, packs, cfg.data)
    plans = sched.steps[:total]
    host = [concat_packs([ds[i] for i in p.rank_packs[rank]]) for p in plans]
    torch.manual_seed(cfg.train.seed)
    cfg.train.max_steps = max(cfg.train.max_steps, 4 * total)
    eng = TrainEngine(cfg, dev)
    batches = [to_device_batch(eng.prepare_batch(h), dev) for h in host]
    for i in range(args.warmup):
        eng.step([batches[i]], plans[i].step_tokens)
    torch.cuda.synchronize()
    bench.barrier()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for i in (args.warmup, args.warmup + 1):
            eng.step([batches[i]], plans[i].step_tokens)
        torch.cuda.synchronize()
    bench.barrier()
    out = Path(args.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    if args.trace:
        prof.export_chrome_trace(str(out / f"trace_w{world}_r{rank}.json"))
    evs = [(e.time_range.start, e.time_range.end, e.name, int(getattr(e, "device_resource_id", 0) or 0))
           for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    evs.sort()
    # the second step starts after the first step's optimizer kernel
    first_adam = next((e for e in evs if "adamw" in e[2]), None)
    step2 = [e for e in evs if first_adam is None or e[0] >= first_adam[1]]
    res = {"world": world, "rank": rank, **summarize(step2)}
    (out / f"step_timeline_w{world}_r{rank}.json").write_text(json.dumps(res, indent=1))
    if rank == 0:
        print(json.dumps({k: v for k, v in res.items() if k != "top_kernels"}), flush=True)
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return res


if __name__ == "__main__":
    main()
