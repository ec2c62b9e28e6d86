"""Command-line tools: benches, thesis validation, metrics plot (CPU)."""

import json
from pathlib import Path

import pytest
import yaml

from packbalance_b200.config import config_to_dict, load_config


@pytest.fixture
def tiny_config(tmp_path: Path) -> Path:
    cfg = load_config(Path(__file__).resolve().parents[1] / "configs" / "tiny.yaml")
    d = config_to_dict(cfg)
    d["data"]["data_dir"] = str(tmp_path / "data")
    d["data"]["synthetic_num_docs"] = 400
    d["train"]["output_dir"] = str(tmp_path / "out")
    p = tmp_path / "cfg.yaml"
    p.write_text(yaml.safe_dump(d), encoding="utf-8")
    return p


def test_bench_schedule_balanced_not_worse(tiny_config: Path, tmp_path: Path) -> None:
    from packbalance_b200.profiling import bench_schedule

    rows = bench_schedule.main(["--config", str(tiny_config), "--modes", "pack_ffd,isoflop", "--world-size", "4",
                                "--output", str(tmp_path / "s.json")])
    by = {(r["mode"], r["schedule"]): r for r in rows}
    for mode in ("pack_ffd", "isoflop"):
        assert by[(mode, "balanced")]["step_cost_cv"] <= by[(mode, "random")]["step_cost_cv"] + 1e-12
    assert json.loads((tmp_path / "s.json").read_text())


def test_bench_data_counts_tokens(tiny_config: Path, tmp_path: Path) -> None:
    from packbalance_b200.profiling import bench_data

    rows = bench_data.main(["--config", str(tiny_config), "--modes", "pad,pack_ffd", "--workers", "0",
                            "--num-batches", "4", "--warmup", "1", "--output", str(tmp_path / "d.json")])
    assert len(rows) == 2 and all(r["useful_tokens"] > 0 for r in rows)
    pad = next(r for r in rows if r["mode"] == "pad")
    assert pad["compute_tokens"] >= pad["useful_tokens"]


def test_bench_train_cpu_step(tiny_config: Path, tmp_path: Path) -> None:
    from packbalance_b200.profiling import bench_train

    rows = bench_train.main(["--config", str(tiny_config), "--modes", "pack_ffd", "--steps", "1", "--warmup", "1",
                             "--device", "cpu", "--output", str(tmp_path / "t.json")])
    assert rows[0]["useful_tokens_per_s"] > 0 and rows[0]["timing"] == "wall clock"


@pytest.mark.slow
def test_prove_intuition_quick(tiny_config: Path, tmp_path: Path) -> None:
    from packbalance_b200.profiling import prove_intuition

    res = prove_intuition.main(["--config", str(tiny_config), "--output-dir", str(tmp_path / "thesis"), "--quick"])
    assert res["packing"]["pad"]["padding_waste"] > res["packing"]["pack_ffd"]["padding_waste"]
    assert res["packing"]["pad"]["flops_ratio_vs_pack_ffd"] > 1.0
    assert res["doc_mask"]["correct_mask_max_abs_error"] < 1e-4 < res["doc_mask"]["broken_mask_max_abs_error"]
    assert res["attention"]["fit_linear_plus_quadratic"]["r2"] > 0.9
    assert (tmp_path / "thesis" / "report.md").exists()


def test_plot_metrics_writes_svg(tmp_path: Path) -> None:
    from packbalance_b200.utils import plot_metrics

    log = tmp_path / "metrics.jsonl"
    recs = [{"event": "start", "world_size": 1}]
    recs += [{"step": i, "loss": 10.0 / (i + 1), "tokens_per_sec": 1000.0 + i} for i in range(1, 30)]
    recs += [{"step": 10, "val_loss": 2.5}, {"event": "finish", "step": 29}]
    log.write_text("\n".join(json.dumps(r) for r in recs), encoding="utf-8")
    out = plot_metrics.main(["--metrics", str(log), "--output", str(tmp_path / "curve.png")])
    text = out.read_text()
    assert out.suffix == ".svg" and text.startswith("<svg") and text.count("<polyline") == 3


def test_step_profiler_writes_window_trace_and_summary(tmp_path: Path) -> None:
    import torch
    from torch.profiler import record_function

    from packbalance_b200.profiling.profiler import make_profiler

    prof = make_profiler(tmp_path / "prof", wait=1, warmup=1, active=2)
    with prof:
        for _ in range(5):
            with record_function("packbalance/forward"):
                torch.randn(64, 64) @ torch.randn(64, 64)
            prof.step()
    names = sorted(p.name for p in prof.written)
    assert names == ["summary_steps2-3.json", "trace_steps2-3.json"]
    summary = json.loads((tmp_path / "prof" / "summary_steps2-3.json").read_text())
    assert summary["profiled_steps"] == 2
    assert summary["phases_ms"]["packbalance/forward"] > 0


def test_attn_trace_summary_of_synthetic_stamps() -> None:
    """The attention trace summary on hand-made stamps: two CTAs, three forward tiles."""
    import numpy as np

    from packbalance_b200.profiling.attn_trace import N_EV, N_ROLES, summarize

    tr = np.zeros((2, N_ROLES, N_EV), dtype=np.int64)
    for c in range(2):
        tr[c, 0, N_EV - 1] = 1000  # start
        tr[c, 2, :3] = [1100, 1500, 1900]  # S issued
        tr[c, 4, :3] = [1200, 1600, 2000]  # S read
        tr[c, 5, :3] = [1450, 1850, 2250]  # P ready
        tr[c, 6, :1] = [2300]
        tr[c, 7, :1] = [2400]
    s = summarize(tr, "fwd")
    assert s["s_issue_to_read"] == 100 and s["softmax_per_tile"] == 250
    assert s["idle_between_tiles"] == 150 and s["tile_period"] == 400 and s["epilogue_per_item"] == 100
    assert s["span_per_cta_median"] == 1400 and s["span_per_cta_max"] == 1400


def test_step_timeline_summary_of_synthetic_events() -> None:
    """The step-timeline summary: collectives with the compute that ran beside them, the
    optimizer start, idle time of the attention stream, per-kernel totals."""
    from packbalance_b200.profiling.step_timeline import summarize

    ev = [
        (0.0, 10.0, "pb::gemm_pair_kernel", 7),
        (12.0, 30.0, "pb::attn_bwd_kernel<64>", 7),
        (14.0, 24.0, "pb::nvls_allreduce_kernel", 9),   # 10 us, all of it beside attn_bwd
        (30.0, 40.0, "void pb::fused_allreduce_kernel<2>", 9),  # nothing beside it
        (35.0, 38.0, "pb::gemm_pair_kernel", 7),
        (41.0, 50.0, "pb::adamw_kernel", 7),
    ]
    s = summarize(ev)
    assert s["step_span_us"] == 50.0 and s["optimizer_start_us"] == 41.0
    beside = {c["start_us"]: c["compute_beside_us"] for c in s["collectives"]}
    assert beside == {14.0: 10.0, 30.0: 3.0 + 0.0}
    # the attention stream (7) idles 0-10 -> 12 and 30 -> 35 and 38 -> 41
    assert s["main_stream_gaps_us"] == 2.0 + 5.0 + 3.0
    tops = {t["name"]: t for t in s["top_kernels"]}
    assert tops["pb::gemm_pair_kernel"]["count"] == 2 and tops["pb::gemm_pair_kernel"]["us"] == 13.0
