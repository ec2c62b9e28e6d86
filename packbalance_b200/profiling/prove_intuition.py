"""Thesis validation before GPU time: the framework's assumptions as measurements.

    python -m packbalance_b200.profiling.prove_intuition [--config configs/bench.yaml]
        [--output-dir artifacts/thesis] [--device cpu|cuda] [--quick]

Experiments (the reference's ``profiling/prove_intuition.py`` runs the same seven on
CPU; ``main`` 864-868 is its CLI):

1. ``packing``       padding is a large compute tax: FLOPs per useful token, padding
                     waste and attention share for pad / pack_random / pack_ffd /
                     isoflop on the config's corpus, with the W=8 balanced schedule.
2. ``attention``     one-document steps of growing length: time fits
                     a + b L + c L^2 and is linear in the analytical cost.
3. ``cost_model``    packs spread over the cost range: measured forward+backward time
                     against tokens and sum of squared document lengths (R^2), and its
                     correlation with the cost model.
4. ``scheduling``    simulated step times (cost-proportional pack times with lognormal
                     noise) of random vs balanced schedules, natural and with stress
                     multipliers (10 % of packs x5, 2 % x20): p99 step time and
                     straggler ratio (slowest rank / mean rank).
5. ``splitting``     max_doc_len 1024 / 512 / 256: FLOPs per useful token, attention
                     share, cost CV, simulated p99.
6. ``ce_memory``     peak RSS of full-logits CE vs chunked CE (separate processes).
7. ``doc_mask``      packed forward equals per-document isolated forwards under the
                     document mask; a broken mask (one document) does not.

Timing experiments run the model on ``--device`` (CPU: eager ops, one thread, min of
5 repetitions; CUDA: the native kernels, CUDA events).  Writes ``report.md`` and
``results.json`` to ``--output-dir``.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from dataclasses import replace
from pathlib import Path

import numpy as np
import torch

from packbalance_b200.config import DataConfig, ModelConfig, load_config
from packbalance_b200.data.cost import FlopModel
from packbalance_b200.data.dataset import PackedDataset
from packbalance_b200.data.packer import build_packs, pack_stats
from packbalance_b200.data.prepare import prepare_synthetic
from packbalance_b200.data.sampler import build_schedule
from packbalance_b200.data.store import TokenStore
from packbalance_b200.models.llama import LlamaForCausalLM

MODES = ("pad", "pack_random", "pack_ffd", "isoflop")


def r2(y: np.ndarray, yhat: np.ndarray) -> float:
    tot = float(((y - y.mean()) ** 2).sum())
    return 1.0 - float(((y - yhat) ** 2).sum()) / tot if tot else 0.0


def lstsq(cols: list[np.ndarray], y: np.ndarray) -> tuple[np.ndarray, float]:
    X = np.stack(cols, axis=1)
    coef, *_ = np.linalg.lstsq(X, y, rcond=None)
    return coef, r2(y, X @ coef)


def time_ms(fn, device: torch.device, warmup: int = 2, reps: int = 5) -> float:
    for _ in range(warmup):
        fn()
    if device.type == "cuda":
        torch.cuda.synchronize(device)
        out = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize(device)
            out.append(a.elapsed_time(b))
        return float(np.min(out))
    out = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        out.append((time.perf_counter() - t0) * 1e3)
    return float(np.min(out))  # min: least disturbed by CPU scheduling noise


def train_step_fn(model, batch: dict, device: torch.device):
    ids = batch["input_ids"].unsqueeze(0).to(device)
    kw = dict(labels=batch["labels"].unsqueeze(0).to(device), position_ids=batch["position_ids"].unsqueeze(0).to(device),
              doc_ids=batch["doc_ids"].unsqueeze(0).to(device))
    if "doc_start" in batch:
        kw["doc_start"] = batch["doc_start"].to(device)

    def step() -> None:
        out = model(ids, **kw)
        out.loss.backward()
        model.zero_grad(set_to_none=True)

    return step


def single_doc_batch(length: int, vocab: int) -> dict:
    g = torch.Generator().manual_seed(length)
    ids = torch.randint(0, vocab, (length,), generator=g)
    labels = torch.full((length,), -100, dtype=torch.long)
    labels[:-1] = ids[1:]
    return {"input_ids": ids, "labels": labels, "position_ids": torch.arange(length),
            "doc_ids": torch.zeros(length, dtype=torch.long), "doc_start": torch.zeros(length, dtype=torch.int32)}


def thesis_configs(data_dir: Path) -> tuple[DataConfig, ModelConfig]:
    """Small model and 1024-token corpus for the timing experiments."""
    data = DataConfig(dataset="synthetic", data_dir=str(data_dir), seq_len=1024, mode="isoflop", pad_batch_size=8,
                      max_doc_len=1024, min_doc_len=8, synthetic_num_docs=2500, synthetic_mu=5.2, synthetic_sigma=1.0,
                      synthetic_min_len=16, synthetic_max_len=2048, synthetic_vocab_size=4096, num_workers=0,
                      prefetch_factor=1, val_fraction=0.0, seed=11)
    model = ModelConfig(vocab_size=4096, d_model=256, n_layers=4, n_heads=4, n_kv_heads=2, d_ff=768, max_seq_len=1024,
                        attention_backend="auto", ce_chunk_size=128)
    return data, model


# ---- 1. packing tax ---------------------------------------------------------------
def exp_packing(cfg, store, fm) -> dict:
    res = {}
    for mode in MODES:
        packs = build_packs(store, replace(cfg.data, mode=mode), fm, split="train")
        st = pack_stats(packs, fm)
        useful = sum(p.useful_tokens for p in packs)
        flops = sum(p.cost for p in packs)
        if mode == "pad":
            attn = sum(fm.attention_flops_coeff * p.rows * cfg.data.seq_len ** 2 for p in packs)
        else:
            attn = sum(fm.attention_flops_coeff * s.length ** 2 for p in packs for s in p.segments)
        sched = build_schedule(packs, world_size=8, grad_accum=cfg.train.grad_accum, seed=cfg.data.seed,
                               mode="balanced").stats()
        res[mode] = {"padding_waste": st["padding_waste"], "compute_per_useful_token": st["compute_tokens"] / useful,
                     "flops_per_useful_token": flops / useful, "attention_share": attn / flops,
                     "pack_cost_cv": st["cv"], "step_cost_cv": sched["step_cost_cv"],
                     "rank_cost_imbalance": sched["rank_cost_imbalance"], "num_packs": len(packs)}
    base = res["pack_ffd"]["flops_per_useful_token"]
    for r in res.values():
        r["flops_ratio_vs_pack_ffd"] = r["flops_per_useful_token"] / base
    return res


# ---- 2. attention scaling -----------------------------------------------------------
def exp_attention(mcfg: ModelConfig, device: torch.device, lengths=(128, 256, 512, 1024)) -> dict:
    torch.manual_seed(0)
    model = LlamaForCausalLM(mcfg).to(device).train()
    ms = {L: time_ms(train_step_fn(model, single_doc_batch(L, mcfg.vocab_size), device), device) for L in lengths}
    Ls = np.asarray(lengths, dtype=np.float64)
    y = np.asarray([ms[L] for L in lengths])
    one = np.ones_like(Ls)
    cq, r2q = lstsq([one, Ls, Ls ** 2], y)
    cl, r2l = lstsq([one, Ls], y)
    fm = FlopModel.from_config(mcfg)
    costs = np.asarray([fm.pack_cost([int(L)]) for L in lengths], dtype=np.float64)
    cc, r2c = lstsq([one, costs], y)
    return {"lengths": list(lengths), "measured_ms": {str(k): v for k, v in ms.items()},
            "fit_linear_plus_quadratic": {"coef": cq.tolist(), "r2": r2q},
            "fit_linear_only": {"coef": cl.tolist(), "r2": r2l},
            "fit_time_vs_cost": {"coef": cc.tolist(), "r2": r2c},
            "ratio_1024_over_512": ms[lengths[-1]] / ms[lengths[-2]] if len(lengths) > 1 else None}


# ---- 3. cost model vs measured time ------------------------------------------------
def exp_cost_model(dcfg: DataConfig, mcfg: ModelConfig, device: torch.device, n: int = 12) -> dict:
    if not (Path(dcfg.data_dir) / "meta.json").exists():
        prepare_synthetic(dcfg, Path(dcfg.data_dir))
    store = TokenStore.open(dcfg.data_dir)
    fm = FlopModel.from_config(mcfg)
    packs = build_packs(store, dcfg, fm, split="train")
    order = np.argsort([p.cost for p in packs])
    chosen = [packs[int(order[int(q * (len(order) - 1))])] for q in np.linspace(0, 1, n)]
    torch.manual_seed(0)
    model = LlamaForCausalLM(mcfg).to(device).train()
    ds = PackedDataset(store, chosen, dcfg)
    y = np.asarray([time_ms(train_step_fn(model, ds[i], device), device, warmup=2, reps=5) for i in range(len(chosen))])
    tok = np.asarray([p.tokens for p in chosen], dtype=np.float64)
    sq = np.asarray([sum(s.length ** 2 for s in p.segments) for p in chosen], dtype=np.float64)
    coef, fit = lstsq([np.ones_like(tok), tok, sq], y)
    cost = np.asarray([p.cost for p in chosen], dtype=np.float64)
    return {"num_packs": len(chosen), "coef": coef.tolist(), "r2_tokens_plus_sumsq": fit,
            "pearson_time_vs_cost": float(np.corrcoef(y, cost)[0, 1]),
            "measurements": [{"tokens": int(t), "sum_sq": int(s), "cost": float(c), "ms": float(m)}
                             for t, s, c, m in zip(tok, sq, cost, y)]}


# ---- 4/5. scheduling simulation ------------------------------------------------------
def simulate(schedule, base: np.ndarray, noise: list[np.ndarray]) -> dict:
    p99, mean, ratio = [], [], []
    for nz in noise:
        t = base * nz
        step, ideal = [], []
        for plan in schedule.steps:
            ranks = [float(sum(t[i] for i in ids)) for ids in plan.rank_packs]
            step.append(max(ranks))
            ideal.append(sum(ranks) / len(ranks))
        step_a, ideal_a = np.asarray(step), np.asarray(ideal)
        p99.append(float(np.percentile(step_a, 99)))
        mean.append(float(step_a.mean()))
        ratio.append(float(np.mean(step_a / ideal_a)))
    return {"mean_step": float(np.mean(mean)), "p99_step": float(np.mean(p99)),
            "straggler_ratio_mean": float(np.mean(ratio)), "straggler_ratio_p99": float(np.percentile(ratio, 99))}


def schedule_condition(packs, mult: np.ndarray, trials: int, seed: int) -> dict:
    saved = [p.cost for p in packs]
    scaled = np.asarray(saved) * mult
    for p, c in zip(packs, scaled):
        p.cost = float(c)
    base = 1.0 + 100.0 * scaled / scaled.mean()  # time linear in cost (experiment 2)
    rng = np.random.default_rng(seed)
    noise = [rng.lognormal(0.0, 0.05, len(packs)) for _ in range(trials)]
    out = {}
    for policy in ("random", "balanced"):
        sched = build_schedule(packs, world_size=8, grad_accum=4, seed=seed, mode=policy)
        out[policy] = {**simulate(sched, base, noise), "scheduler": sched.stats()}
    for p, c in zip(packs, saved):
        p.cost = c
    out["p99_reduction"] = 1.0 - out["balanced"]["p99_step"] / out["random"]["p99_step"]
    out["straggler_reduction"] = 1.0 - out["balanced"]["straggler_ratio_mean"] / out["random"]["straggler_ratio_mean"]
    return out


def exp_scheduling(cfg, store, fm, trials: int) -> dict:
    packs = build_packs(store, cfg.data, fm, split="train")
    n = len(packs)
    rng = np.random.default_rng(42)
    conds = {"natural": np.ones(n), "stress_10pct_5x": np.where(rng.random(n) < 0.10, 5.0, 1.0),
             "stress_2pct_20x": np.where(rng.random(n) < 0.02, 20.0, 1.0)}
    return {"trials": trials, "noise_sigma": 0.05, "world_size": 8, "grad_accum": 4, "num_packs": n,
            **{k: schedule_condition(packs, m, trials, cfg.data.seed) for k, m in conds.items()}}


def exp_splitting(dcfg: DataConfig, mcfg: ModelConfig, trials: int) -> dict:
    store = TokenStore.open(dcfg.data_dir)
    fm = FlopModel.from_config(mcfg)
    rng = np.random.default_rng(321)
    rows = {}
    for max_len in (1024, 512, 256):
        packs = build_packs(store, replace(dcfg, max_doc_len=max_len), fm, split="train")
        st = pack_stats(packs, fm)
        useful = sum(p.useful_tokens for p in packs)
        flops = sum(p.cost for p in packs)
        attn = sum(fm.attention_flops_coeff * s.length ** 2 for p in packs for s in p.segments)
        costs = np.asarray([p.cost for p in packs])
        base = 1.0 + 100.0 * costs / costs.mean()
        noise = [rng.lognormal(0.0, 0.05, len(packs)) for _ in range(trials)]
        sched = build_schedule(packs, world_size=8, grad_accum=4, seed=dcfg.seed, mode="balanced")
        rows[str(max_len)] = {"padding_waste": st["padding_waste"], "pack_cost_cv": st["cv"],
                              "flops_per_useful_token": flops / useful, "attention_share": attn / flops,
                              **sched.stats(), **simulate(sched, base, noise)}
    return rows


# ---- 6. CE memory ---------------------------------------------------------------------
_RSS = """
import resource, sys, torch, torch.nn.functional as F
torch.manual_seed(0)
T, V, D, C = {T}, {V}, {D}, {C}
x = torch.randn(T, D, requires_grad=True); w = torch.randn(V, D, requires_grad=True)
t = torch.randint(0, V, (T,))
if {kind!r} == "full":
    F.cross_entropy(x @ w.t(), t, reduction="sum").backward()
else:
    from packbalance_b200.ops.reference import chunked_linear_cross_entropy
    chunked_linear_cross_entropy(x, w, t, chunk_size=C).backward()
print(resource.getrusage(resource.RUSAGE_SELF).ru_maxrss)
"""


def exp_ce_memory(T: int = 2048, V: int = 16384, D: int = 256, C: int = 128) -> dict:
    root = Path(__file__).resolve().parents[2]
    env = {**os.environ, "PYTHONPATH": str(root), "OMP_NUM_THREADS": "4", "CUDA_VISIBLE_DEVICES": ""}

    def rss(kind: str) -> float:
        out = subprocess.check_output([sys.executable, "-c", _RSS.format(T=T, V=V, D=D, C=C, kind=kind)], env=env,
                                      text=True)
        return float(out.strip().splitlines()[-1]) / 1e3  # KiB -> MB (Linux)

    full, chunked = rss("full"), rss("chunked")
    return {"tokens": T, "vocab": V, "dim": D, "chunk": C, "full_peak_rss_mb": full, "chunked_peak_rss_mb": chunked,
            "rss_reduction_mb": full - chunked, "analytical_full_logits_mb": T * V * 4 / 1e6,
            "analytical_chunk_logits_mb": C * V * 4 / 1e6}


# ---- 7. document mask ------------------------------------------------------------------
def exp_doc_mask(dcfg: DataConfig, mcfg: ModelConfig) -> dict:
    store = TokenStore.open(dcfg.data_dir)
    fm = FlopModel.from_config(mcfg)
    packs = build_packs(store, dcfg, fm, split="train")
    pack = next(p for p in packs if p.kind == "packed" and len(p.segments) >= 2)
    item = PackedDataset(store, [pack], dcfg)[0]
    torch.manual_seed(0)
    model = LlamaForCausalLM(replace(mcfg, attention_backend="eager")).eval()
    with torch.no_grad():
        packed = model.model(item["input_ids"][None], item["position_ids"][None], item["doc_ids"][None])
        broken = model.model(item["input_ids"][None], item["position_ids"][None],
                             torch.zeros_like(item["doc_ids"])[None])
        ok_err = bad_err = 0.0
        at = 0
        for s in pack.segments:
            toks = torch.from_numpy(store.read(s.start, s.length))
            iso = model.model(toks[None], torch.arange(s.length)[None], torch.zeros(1, s.length, dtype=torch.long))
            ok_err = max(ok_err, float((packed[0, at: at + s.length] - iso[0]).abs().max()))
            bad_err = max(bad_err, float((broken[0, at: at + s.length] - iso[0]).abs().max()))
            at += s.length
    return {"num_segments": len(pack.segments), "correct_mask_max_abs_error": ok_err,
            "broken_mask_max_abs_error": bad_err}


# ---- report -------------------------------------------------------------------------
def table(headers: list[str], rows: list[list[str]]) -> str:
    out = ["| " + " | ".join(headers) + " |", "|" + "|".join(["---"] + ["---:"] * (len(headers) - 1)) + "|"]
    out += ["| " + " | ".join(r) + " |" for r in rows]
    return "\n".join(out)


def report(res: dict) -> str:
    p = res["packing"]
    lines = ["# Thesis validation", "", f"device: {res['device']}", "", "## 1. Padding tax", "",
             table(["mode", "waste", "FLOPs/useful token vs pack_ffd", "attention share", "step cost CV", "rank imbalance"],
                   [[m, f"{p[m]['padding_waste']:.1%}", f"{p[m]['flops_ratio_vs_pack_ffd']:.2f}x",
                     f"{p[m]['attention_share']:.1%}", f"{p[m]['step_cost_cv']:.4f}", f"{p[m]['rank_cost_imbalance']:.2%}"]
                    for m in MODES])]
    a = res["attention"]
    lines += ["", "## 2. Attention scaling (one document of length L, forward + backward)", "",
              table(["L", "ms"], [[str(k), f"{v:.2f}"] for k, v in a["measured_ms"].items()]), "",
              f"fit a + bL + cL^2: R^2 = {a['fit_linear_plus_quadratic']['r2']:.4f}; linear only: "
              f"R^2 = {a['fit_linear_only']['r2']:.4f}; time vs analytical cost: R^2 = {a['fit_time_vs_cost']['r2']:.4f}; "
              f"t(1024)/t(512) = {a['ratio_1024_over_512']:.2f}"]
    c = res["cost_model"]
    lines += ["", "## 3. Cost model vs measured pack time", "",
              f"{c['num_packs']} packs across the cost range: R^2 (tokens + sum L^2) = {c['r2_tokens_plus_sumsq']:.4f}, "
              f"Pearson(time, cost) = {c['pearson_time_vs_cost']:.4f}"]
    s = res["scheduling"]
    rows = []
    for k in ("natural", "stress_10pct_5x", "stress_2pct_20x"):
        r = s[k]
        rows.append([k, f"{r['random']['p99_step']:.1f}", f"{r['balanced']['p99_step']:.1f}", f"{r['p99_reduction']:.1%}",
                     f"{r['random']['scheduler']['rank_cost_imbalance']:.2%}",
                     f"{r['balanced']['scheduler']['rank_cost_imbalance']:.2%}"])
    lines += ["", "## 4. Scheduling (simulated, W=8, A=4)", "",
              table(["condition", "p99 random", "p99 balanced", "p99 reduction", "rank imb random", "rank imb balanced"], rows)]
    sp = res["splitting"]
    lines += ["", "## 5. Document splitting", "",
              table(["max_doc_len", "FLOPs/useful token", "attention share", "pack cost CV", "simulated p99"],
                    [[k, f"{v['flops_per_useful_token']:.3e}", f"{v['attention_share']:.1%}", f"{v['pack_cost_cv']:.3f}",
                      f"{v['p99_step']:.1f}"] for k, v in sp.items()])]
    ce = res["ce_memory"]
    lines += ["", "## 6. Chunked CE memory", "",
              f"peak RSS full logits {ce['full_peak_rss_mb']:.0f} MB vs chunked {ce['chunked_peak_rss_mb']:.0f} MB "
              f"(analytical logits {ce['analytical_full_logits_mb']:.0f} MB vs {ce['analytical_chunk_logits_mb']:.0f} MB)"]
    dm = res["doc_mask"]
    lines += ["", "## 7. Document mask", "",
              f"{dm['num_segments']} documents in one pack: packed vs isolated max |error| = "
              f"{dm['correct_mask_max_abs_error']:.2e}; with the mask broken = {dm['broken_mask_max_abs_error']:.2e}", ""]
    return "\n".join(lines)


def main(argv: list[str] | None = None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", default="configs/bench.yaml")
    ap.add_argument("--output-dir", default="artifacts/thesis")
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--quick", action="store_true", help="fewer trials and shorter timing sweeps (smoke test)")
    args = ap.parse_args(argv)
    device = torch.device(args.device)
    if device.type == "cpu":
        torch.set_num_threads(1)
    out = Path(args.output_dir)
    out.mkdir(parents=True, exist_ok=True)
    cfg = load_config(args.config)
    if not (Path(cfg.data.data_dir) / "meta.json").exists():
        prepare_synthetic(cfg.data, Path(cfg.data.data_dir))
    store = TokenStore.open(cfg.data.data_dir)
    fm = FlopModel.from_config(cfg.model)
    dcfg, mcfg = thesis_configs(out / "thesis_data")
    trials = 5 if args.quick else 30
    lengths = (64, 128, 256) if args.quick else (128, 256, 512, 1024)
    res = {"device": str(device), "config": args.config}
    res["packing"] = exp_packing(cfg, store, fm)
    res["attention"] = exp_attention(mcfg, device, lengths)
    res["cost_model"] = exp_cost_model(dcfg, mcfg, device, n=4 if args.quick else 12)
    res["scheduling"] = exp_scheduling(cfg, store, fm, trials)
    res["splitting"] = exp_splitting(dcfg, mcfg, trials)
    res["ce_memory"] = exp_ce_memory(*((256, 4096, 64, 64) if args.quick else ()))
    res["doc_mask"] = exp_doc_mask(dcfg, mcfg)
    (out / "results.json").write_text(json.dumps(res, indent=2), encoding="utf-8")
    (out / "report.md").write_text(report(res), encoding="utf-8")
    print(report(res))
    return res


if __name__ == "__main__":
    main()
