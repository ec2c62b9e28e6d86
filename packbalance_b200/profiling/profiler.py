"""Step-window profiler for the trainer (reference role: ``profiling/profiler.py:11-40``).

A :class:`StepProfiler` watches the step counter the trainer advances with
:meth:`StepProfiler.step`.  It skips ``wait`` steps, runs ``warmup`` steps under the
profiler with recording discarded, then records ``active`` steps; ``repeat`` windows
of that shape follow each other.  When a window closes, it writes

* ``trace_steps{first}-{last}.json`` - the Chrome trace of the recorded steps,
* ``summary_steps{first}-{last}.json`` - the phase / top-kernel report of
  :func:`packbalance_b200.profiling.analyze_trace.analyze` on that trace,

and prints one line per phase.  The phases are the ``packbalance/{data, block_mask,
forward, backward, optimizer, comm}`` ``record_function`` ranges the trainer emits, so
the summaries compare directly with the reference's reports.

Device work is captured through CUPTI (``ProfilerActivity.CUDA``) when a GPU is
present; tensor shapes and allocator events are kept so the trace can be used for
memory analysis as well.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch
from torch.profiler import ProfilerActivity

from packbalance_b200.profiling.analyze_trace import PHASES, analyze


class StepProfiler:
    """Context-managed wrapper around ``torch.profiler.profile`` keyed on step windows."""

    def __init__(self, output_dir: str | Path, *, wait: int = 1, warmup: int = 1, active: int = 3,
                 repeat: int = 1) -> None:
        if active < 1:
            raise ValueError("active must be >= 1")
        self.dir = Path(output_dir)
        self.wait, self.warmup, self.active, self.repeat = wait, warmup, active, repeat
        self.steps_seen = 0
        self.written: list[Path] = []
        activities = [ProfilerActivity.CPU]
        if torch.cuda.is_available():
            activities.append(ProfilerActivity.CUDA)
        self._prof = torch.profiler.profile(
            activities=activities,
            schedule=torch.profiler.schedule(wait=wait, warmup=warmup, active=active, repeat=repeat),
            on_trace_ready=self._window_done,
            record_shapes=True,
            profile_memory=True,
        )

    # -- window bookkeeping ---------------------------------------------------------
    def _window_bounds(self) -> tuple[int, int]:
        """First and last step (0-based, as counted by :meth:`step`) of the window that
        just closed."""
        last = self.steps_seen - 1
        return last - self.active + 1, last

    def _window_done(self, prof) -> None:
        self.dir.mkdir(parents=True, exist_ok=True)
        first, last = self._window_bounds()
        tag = f"steps{first}-{last}"
        trace = self.dir / f"trace_{tag}.json"
        prof.export_chrome_trace(str(trace))
        report = analyze(trace)
        summary = self.dir / f"summary_{tag}.json"
        summary.write_text(json.dumps(report, indent=2), encoding="utf-8")
        self.written += [trace, summary]
        lines = [f"[profiler] steps {first}-{last}: {report['total_step_ms']:.2f} ms recorded -> {trace.name}"]
        for ph in PHASES:
            if ph in report["phases_ms"]:
                lines.append(f"[profiler]   {ph:<24} {report['phases_ms'][ph]:9.2f} ms "
                             f"({report['phase_pct'][ph]:.1f}%)")
        if report["top_kernels"]:
            name, ms = report["top_kernels"][0]
            lines.append(f"[profiler]   top kernel {name[:60]} {ms:.2f} ms")
        print("\n".join(lines), flush=True)

    # -- trainer hooks -------------------------------------------------------------
    def start(self) -> "StepProfiler":
        self._prof.start()
        return self

    def step(self) -> None:
        """Call once after every training step."""
        self.steps_seen += 1
        self._prof.step()

    def stop(self) -> None:
        self._prof.stop()

    def __enter__(self) -> "StepProfiler":
        return self.start()

    def __exit__(self, *exc) -> None:
        self.stop()


def make_profiler(output_dir: str | Path, *, wait: int = 1, warmup: int = 1, active: int = 3,
                  repeat: int = 1) -> StepProfiler:
    """The trainer's profiler (same call as the reference's ``make_profiler``)."""
    return StepProfiler(output_dir, wait=wait, warmup=warmup, active=active, repeat=repeat)
