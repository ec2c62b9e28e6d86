from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from dataclasses import asdict
from pathlib import Path

import pytest
import yaml

from packbalance_b200.config import DataConfig, ModelConfig, PackBalanceConfig, TrainConfig

ROOT = Path(__file__).resolve().parents[1]


def _config(out: Path, data_dir: str, **train) -> PackBalanceConfig:
    return PackBalanceConfig(
        # 3 layers, GQA 4/2 at head_dim 10, the odd vocabulary of the shared corpus
        # fixture; a corpus tail past the 72-token pack length, so documents are split
        model=ModelConfig(vocab_size=203, d_model=40, n_layers=3, n_heads=4, n_kv_heads=2, d_ff=72, max_seq_len=72,
                          attention_backend="eager", use_fused_ce=False, ce_chunk_size=20),
        data=DataConfig(dataset="synthetic", data_dir=data_dir, seq_len=72, mode="isoflop", pad_batch_size=3,
                        max_doc_len=72, min_doc_len=2, synthetic_num_docs=210, synthetic_mu=3.2, synthetic_sigma=1.0,
                        synthetic_min_len=4, synthetic_max_len=150, synthetic_vocab_size=203, num_workers=0,
                        prefetch_factor=1, val_fraction=0.2, seed=23, schedule="balanced"),
        train=TrainConfig(**{**dict(output_dir=str(out), max_steps=2, grad_accum=1, lr=1e-3, min_lr=1e-4,
                                    warmup_steps=1, dtype="fp32", log_interval=1, save_interval=1, eval_interval=0,
                                    gpu_hourly_cost=0.0, peak_tflops=0.0), **train}),
    )


def _write(cfg, path: Path) -> Path:
    path.write_text(yaml.safe_dump(asdict(cfg), sort_keys=False), encoding="utf-8")
    return path


def _run(args, env=None, timeout=240):
    return subprocess.run([sys.executable, *args], cwd=ROOT, capture_output=True, text=True, timeout=timeout,
                          env={**os.environ, "CUDA_VISIBLE_DEVICES": "", **(env or {})})


def test_training_smoke_and_resume(tmp_path: Path, store, data_cfg) -> None:
    cfg = _write(_config(tmp_path / "run", data_cfg.data_dir, eval_interval=1), tmp_path / "c.yaml")
    r = _run(["-m", "packbalance_b200.train.train", "--config", str(cfg), "--max-steps", "1"])
    assert r.returncode == 0, r.stdout + r.stderr
    run = tmp_path / "run"
    assert (run / "metrics.jsonl").exists() and (run / "config.yaml").exists()
    assert (run / "checkpoints" / "step_0000001" / "state.pt").exists()
    recs = [json.loads(line) for line in (run / "metrics.jsonl").read_text().splitlines()]
    assert recs[0]["event"] == "start" and any("val_loss" in r for r in recs)
    step = next(r for r in recs if "loss" in r)
    for key in ("loss", "lr", "grad_norm", "tokens_per_sec", "step_ms", "data_ms", "tokens", "cost_cv"):
        assert key in step
    r = _run(["-m", "packbalance_b200.train.train", "--config", str(cfg), "--max-steps", "2", "--resume"])
    assert r.returncode == 0, r.stdout + r.stderr
    assert "[resume]" in r.stdout
    assert (run / "checkpoints" / "step_0000002" / "state.pt").exists()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


@pytest.mark.slow
@pytest.mark.parametrize("fsdp,wire", [(False, "fp32"), (True, "fp32"), (False, "bf16")])
def test_two_rank_gloo_smoke(tmp_path: Path, store, data_cfg, fsdp: bool, wire: str) -> None:
    cfg = _write(_config(tmp_path / "ddp", data_cfg.data_dir, max_steps=2, save_interval=0, fsdp=fsdp,
                         grad_reduce_dtype=wire), tmp_path / "c.yaml")
    r = _run(["-m", "torch.distributed.run", "--standalone", "--nnodes=1", "--nproc_per_node=2",
              "-m", "packbalance_b200.train.train", "--config", str(cfg)],
             env={"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(_free_port()), "OMP_NUM_THREADS": "1"})
    assert r.returncode == 0, r.stdout + r.stderr
    final = tmp_path / "ddp" / "checkpoints" / "step_0000002"
    assert (final / "meta.json").exists()
    assert (final / ("dcp" if fsdp else "state.pt")).exists()
