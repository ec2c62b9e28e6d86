"""Plot a training run's metrics JSONL (loss curves and throughput) as SVG.

    python -m packbalance_b200.utils.plot_metrics --metrics artifacts/run/metrics.jsonl \
        --output artifacts/run/loss_curve.svg [--title "..."] [--ema-span 50]

Two panels: training loss (raw and exponential moving average with ``--ema-span``)
with validation loss points, and useful tokens/s per logged step.  Same CLI as the
reference's ``scripts/plot_metrics.py`` (``main`` 28-130); the SVG is written directly
(no plotting library needed).  An output name ending in ``.png`` is written as SVG
with the ``.svg`` suffix.
"""

from __future__ import annotations

import argparse
import html
import json
from pathlib import Path

import numpy as np


def ema(values: np.ndarray, span: int) -> np.ndarray:
    a = 2.0 / (span + 1.0)
    out = np.empty(len(values), dtype=np.float64)
    acc = float(values[0]) if len(values) else 0.0
    for i, v in enumerate(values):
        acc = a * float(v) + (1.0 - a) * acc if i else float(v)
        out[i] = acc
    return out


def read_metrics(path: Path) -> tuple[dict[str, np.ndarray], list[tuple[int, float]]]:
    steps, loss, tps, val = [], [], [], []
    for line in path.read_text(encoding="utf-8").splitlines():
        if not line.strip():
            continue
        r = json.loads(line)
        if "val_loss" in r and r.get("val_loss") is not None:
            val.append((int(r["step"]), float(r["val_loss"])))
        elif "loss" in r and "step" in r and r.get("event") is None:
            steps.append(int(r["step"]))
            loss.append(float(r["loss"]))
            tps.append(float(r.get("tokens_per_sec") or 0.0))
    return {"step": np.asarray(steps), "loss": np.asarray(loss), "tps": np.asarray(tps)}, val


class Panel:
    """Axes box inside the SVG with linear x/y mapping."""

    def __init__(self, x0, y0, w, h, xr, yr):
        self.x0, self.y0, self.w, self.h = x0, y0, w, h
        self.xr = (xr[0], xr[1] if xr[1] > xr[0] else xr[0] + 1)
        self.yr = (yr[0], yr[1] if yr[1] > yr[0] else yr[0] + 1)

    def pt(self, x, y):
        px = self.x0 + (x - self.xr[0]) / (self.xr[1] - self.xr[0]) * self.w
        py = self.y0 + self.h - (y - self.yr[0]) / (self.yr[1] - self.yr[0]) * self.h
        return px, py

    def line(self, xs, ys, color, width=1.5, opacity=1.0):
        if len(xs) == 0:
            return ""
        pts = " ".join(f"{a:.1f},{b:.1f}" for a, b in (self.pt(x, y) for x, y in zip(xs, ys)))
        return (f'<polyline fill="none" stroke="{color}" stroke-width="{width}" stroke-opacity="{opacity}" '
                f'points="{pts}"/>')

    def dots(self, pts, color):
        return "".join(f'<circle cx="{a:.1f}" cy="{b:.1f}" r="3" fill="{color}"/>'
                       for a, b in (self.pt(x, y) for x, y in pts))

    def frame(self, xlabel, ylabel):
        s = [f'<rect x="{self.x0}" y="{self.y0}" width="{self.w}" height="{self.h}" fill="none" stroke="#444"/>']
        for i in range(5):
            fx = self.xr[0] + (self.xr[1] - self.xr[0]) * i / 4
            fy = self.yr[0] + (self.yr[1] - self.yr[0]) * i / 4
            px, _ = self.pt(fx, self.yr[0])
            _, py = self.pt(self.xr[0], fy)
            s.append(f'<text x="{px:.0f}" y="{self.y0 + self.h + 16}" font-size="11" text-anchor="middle">{fx:,.0f}</text>')
            s.append(f'<text x="{self.x0 - 6}" y="{py + 4:.0f}" font-size="11" text-anchor="end">{fy:,.3g}</text>')
            s.append(f'<line x1="{self.x0}" x2="{self.x0 + self.w}" y1="{py:.1f}" y2="{py:.1f}" stroke="#ddd"/>')
        s.append(f'<text x="{self.x0 + self.w / 2}" y="{self.y0 + self.h + 34}" font-size="12" '
                 f'text-anchor="middle">{xlabel}</text>')
        s.append(f'<text x="{self.x0 - 52}" y="{self.y0 + self.h / 2}" font-size="12" text-anchor="middle" '
                 f'transform="rotate(-90 {self.x0 - 52} {self.y0 + self.h / 2})">{ylabel}</text>')
        return "".join(s)


def render(metrics: dict[str, np.ndarray], val: list[tuple[int, float]], title: str, span: int) -> str:
    W, H = 960, 420
    st, loss, tps = metrics["step"], metrics["loss"], metrics["tps"]
    xr = (float(st.min()) if len(st) else 0.0, float(st.max()) if len(st) else 1.0)
    ys = np.concatenate([loss, np.asarray([v for _, v in val])]) if len(loss) or val else np.asarray([0.0, 1.0])
    left = Panel(80, 50, 360, 300, xr, (float(ys.min()), float(ys.max())))
    right = Panel(560, 50, 360, 300, xr, (0.0, float(tps.max()) * 1.1 if len(tps) and tps.max() > 0 else 1.0))
    parts = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{W}" height="{H}" font-family="sans-serif">',
             '<rect width="100%" height="100%" fill="white"/>',
             f'<text x="{W / 2}" y="24" font-size="16" text-anchor="middle">{html.escape(title)}</text>',
             left.frame("step", "loss"), right.frame("step", "useful tokens/s"),
             left.line(st, loss, "#1f77b4", 1.0, 0.35),
             left.line(st, ema(loss, span) if len(loss) else loss, "#1f77b4", 2.0),
             left.dots(val, "#d62728"), right.line(st, tps, "#2ca02c", 1.5),
             f'<text x="{left.x0 + 8}" y="{left.y0 + 16}" font-size="11" fill="#1f77b4">train (EMA {span})</text>',
             f'<text x="{left.x0 + 8}" y="{left.y0 + 30}" font-size="11" fill="#d62728">validation</text>',
             "</svg>"]
    return "\n".join(parts)


def main(argv: list[str] | None = None) -> Path:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--metrics", required=True)
    ap.add_argument("--output", required=True)
    ap.add_argument("--title", default="packbalance training")
    ap.add_argument("--ema-span", type=int, default=50)
    args = ap.parse_args(argv)
    metrics, val = read_metrics(Path(args.metrics))
    out = Path(args.output)
    if out.suffix.lower() != ".svg":
        out = out.with_suffix(".svg")
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(render(metrics, val, args.title, args.ema_span), encoding="utf-8")
    print(f"wrote {out} ({len(metrics['step'])} steps, {len(val)} eval points)")
    return out


if __name__ == "__main__":
    main()
