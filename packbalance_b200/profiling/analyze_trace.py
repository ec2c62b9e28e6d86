"""Chrome trace -> phase / top-kernel / top-CPU-op report (Markdown + JSON).

Contract of the reference analyser (``profiling/analyze_trace.py:19-125``): durations
of ``user_annotation`` events named ``packbalance/*`` are summed per phase,
``ProfilerStep*`` events give the step total, ``kernel`` and ``cpu_op`` events are
ranked by summed duration.
"""

from __future__ import annotations

import argparse
import json
from collections import defaultdict
from pathlib import Path

PHASES = (
    "packbalance/data",
    "packbalance/block_mask",
    "packbalance/forward",
    "packbalance/backward",
    "packbalance/optimizer",
    "packbalance/comm",
)


def _pct(part: float, whole: float) -> float:
    return 100.0 * part / whole if whole else 0.0


def analyze(trace_path: str | Path) -> dict:
    events = json.loads(Path(trace_path).read_text(encoding="utf-8")).get("traceEvents", [])
    phase_us: dict[str, float] = defaultdict(float)
    kernel_us: dict[str, float] = defaultdict(float)
    cpu_us: dict[str, float] = defaultdict(float)
    steps: list[float] = []
    for ev in events:
        if ev.get("ph") != "X":
            continue
        name, cat, dur = ev.get("name", ""), ev.get("cat", ""), float(ev.get("dur", 0.0))
        if cat == "user_annotation":
            if name.startswith("packbalance/"):
                phase_us[name] += dur
            elif name.startswith("ProfilerStep"):
                steps.append(dur)
        elif cat == "kernel":
            kernel_us[name] += dur
        elif cat == "cpu_op":
            cpu_us[name] += dur
    total_ms = sum(steps) / 1e3
    phases = {k: v / 1e3 for k, v in phase_us.items()}
    other = max(0.0, total_ms - sum(phases.get(k, 0.0) for k in PHASES))
    kern = sorted(((k, v / 1e3) for k, v in kernel_us.items()), key=lambda kv: kv[1], reverse=True)
    kern_total = sum(v for _, v in kern)
    cpu = sorted(((k, v / 1e3) for k, v in cpu_us.items()), key=lambda kv: kv[1], reverse=True)
    return {
        "trace": str(trace_path),
        "profiled_steps": len(steps),
        "total_step_ms": total_ms,
        "phases_ms": phases,
        "other_ms": other,
        "phase_pct": {k: _pct(v, total_ms) for k, v in phases.items()},
        "top_kernels": kern[:15],
        "kernel_pct": {k: _pct(v, kern_total) for k, v in kern[:15]},
        "total_kernel_ms": kern_total,
        "top_cpu_ops": cpu[:15],
        "total_cpu_ms": sum(v for _, v in cpu),
    }


def to_markdown(report: dict) -> str:
    out = [
        f"# Profile report: `{Path(report['trace']).name}`",
        "",
        f"- Profiled steps: **{report['profiled_steps']}**",
        f"- Wall time: **{report['total_step_ms']:.2f} ms**",
        "",
        "## Step phases",
        "",
        "| phase | ms | % of step |",
        "|---|---:|---:|",
    ]
    for k in PHASES:
        if k in report["phases_ms"]:
            out.append(f"| {k} | {report['phases_ms'][k]:.2f} | {report['phase_pct'][k]:.1f}% |")
    out.append(f"| other | {report['other_ms']:.2f} | {_pct(report['other_ms'], report['total_step_ms']):.1f}% |")
    out += ["", "## Top GPU kernels", ""]
    if report["top_kernels"]:
        out += ["| kernel | ms | % of kernel time |", "|---|---:|---:|"]
        for name, ms in report["top_kernels"]:
            out.append(f"| `{name}` | {ms:.2f} | {report['kernel_pct'][name]:.1f}% |")
        out += ["", f"Total kernel time: **{report['total_kernel_ms']:.2f} ms**"]
    else:
        out.append("_CPU-only trace (or no CUDA kernels recorded)._")
    out += ["", "## Top CPU ops", "", "| op | ms |", "|---|---:|"]
    out += [f"| `{name}` | {ms:.2f} |" for name, ms in report["top_cpu_ops"]]
    out += ["", f"Total CPU op time: **{report['total_cpu_ms']:.2f} ms**"]
    return "\n".join(out)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--trace", required=True)
    ap.add_argument("--output", default="artifacts/profile_report.md")
    args = ap.parse_args()
    report = analyze(args.trace)
    md = to_markdown(report)
    out = Path(args.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(md, encoding="utf-8")
    out.with_suffix(".json").write_text(json.dumps(report, indent=2), encoding="utf-8")
    print(md)
    print(f"\nwrote {out} and {out.with_suffix('.json')}")


if __name__ == "__main__":
    main()
