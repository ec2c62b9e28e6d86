"""torch.profiler setup: wait/warmup/active schedule, Chrome-trace export and a
key-averages table (reference ``profiling/profiler.py:11-40``).  Phase ranges are the
``packbalance/{data,block_mask,forward,backward,optimizer,comm}`` record_function
labels the trainer emits."""

from __future__ import annotations

import time
from pathlib import Path

import torch


def make_profiler(output_dir: str | Path, *, wait: int = 1, warmup: int = 1, active: int = 3, repeat: int = 1):
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    acts = [torch.profiler.ProfilerActivity.CPU]
    if torch.cuda.is_available():
        acts.append(torch.profiler.ProfilerActivity.CUDA)

    def _ready(prof) -> None:
        path = out / f"trace_{int(time.time())}.json"
        prof.export_chrome_trace(str(path))
        print(f"[profiler] wrote {path}", flush=True)
        key = "cuda_time_total" if torch.cuda.is_available() else "cpu_time_total"
        print(prof.key_averages().table(sort_by=key, row_limit=25), flush=True)

    return torch.profiler.profile(
        activities=acts,
        schedule=torch.profiler.schedule(wait=wait, warmup=warmup, active=active, repeat=repeat),
        on_trace_ready=_ready,
        record_shapes=True,
        profile_memory=True,
        with_stack=False,
    )
