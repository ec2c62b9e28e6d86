"""Headline benchmark: useful tokens/s of the 100M packed + balanced DDP training step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N ...

Config: benchmark config #2 (``configs/b2_100m.yaml``): 12 layers, d_model 768, 12/4
heads, SwiGLU 2048, vocab 32000, tied embeddings, random init; synthetic heavy-tail
documents (lognormal median 256, sigma 1.2, clipped [16, 2048], Zipf(1.1) ids),
``pack_ffd`` packing to 2048 tokens, balanced schedule, 4 packs per rank per step,
bf16 compute.  Weak scaling: every rank runs its own 4 packs.

``value`` times K steps on the device (CUDA events on the launching stream, a barrier
and a synchronize on both sides, max over ranks) with the step's inputs already on
the device; ``e2e`` times the same K steps through the public ``TrainEngine.step``
API with the host->device copy of each step's pinned inputs and a device->host read
of the step's loss inside the timed region.  The per-step working set (weights,
optimizer state and several GB of activations) is far larger than the 126 MB L2, so
no explicit flush is done between steps.  Rank 0 prints one JSON line.

``--impl reference`` runs the unmodified reference (``baseline/_ref``) through its
own modules (model, DDP wrapper, optimizer, block-mask builder, microbatch loop) on
the same corpus, packs and schedule, and prints the same line with
``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import contextlib
import csv
import io
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parent
CONFIG = ROOT / "configs" / "b2_100m.yaml"
METRIC = "useful tokens/s (device-timed, max over ranks)"


# ----------------------------------------------------------------------------------
def parse_args():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default=str(CONFIG))
    ap.add_argument("--mode", default="pack_ffd")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-count", action="store_true", help="skip the profiler pass that counts kernel launches")
    ap.add_argument("--set", action="append", default=[], metavar="SECTION.KEY=VALUE",
                    help="config override, e.g. train.fsdp_weight_windows=2 (repeatable)")
    return ap.parse_args()


def setup_dist(n: int) -> tuple[int, int, torch.device]:
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}; launch with torchrun --nproc-per-node {n}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    return rank, world, dev


def barrier() -> None:
    if dist.is_initialized():
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x: float, dev) -> float:
    if not dist.is_initialized():
        return x
    t = torch.tensor([x], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather(values: list[float], dev) -> list[list[float]]:
    if not dist.is_initialized():
        return [values]
    t = torch.tensor(values, device=dev, dtype=torch.float64)
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [o.tolist() for o in out]


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons of the job's GPUs, polled every 10 ms
    through NVML in a background thread during the timed region (read-only queries).
    Falls back to ``nvidia-smi -lms 50`` when NVML is unavailable."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, enabled: bool, gpus: list[int] | None = None) -> None:
        import threading

        self.samples: list[tuple[int, float, float, set]] = []
        self.proc = None
        self.thread = None
        self.stop_flag = threading.Event()
        if not enabled:
            return
        try:
            import pynvml

            pynvml.nvmlInit()
            handles = [(i, pynvml.nvmlDeviceGetHandleByIndex(i)) for i in (gpus or [0])]
            masks = [(name, getattr(pynvml, attr)) for name, attr in self.REASONS]

            def poll() -> None:
                while not self.stop_flag.is_set():
                    for i, h in handles:
                        try:
                            sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                            mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
                            r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        except pynvml.NVMLError:
                            continue
                        self.samples.append((i, float(sm), float(mx), {n for n, m in masks if r & m}))
                    self.stop_flag.wait(0.01)

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
        except Exception:  # no NVML: nvidia-smi
            fields = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                      "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                      "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={fields}", "--format=csv,noheader,nounits", "-lms", "50"],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
                )
            except (OSError, ValueError):
                self.proc = None

    def stop(self, gpus: list[int]) -> dict:
        if self.thread is not None:
            self.stop_flag.set()
            self.thread.join(timeout=5)
        elif self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=10)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            for row in csv.reader(io.StringIO(out)):
                try:
                    idx, sm, mx = int(row[0]), float(row[1]), float(row[2])
                except (ValueError, IndexError):
                    continue
                names = {n for (n, _), v in zip(self.REASONS, row[5:9]) if v.strip().lower() == "active"}
                self.samples.append((idx, sm, mx, names))
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        rows = [r for r in self.samples if r[0] in gpus]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        reasons = set().union(*(r[3] for r in rows))
        return {
            "sm_mhz": float(np.median([r[1] for r in rows])),
            "sm_max_mhz": max(r[2] for r in rows),
            "reasons": sorted(reasons),
            "samples": len(rows),
        }


# ----------------------------------------------------------------------------------
def build_data(cfg, mode: str, world: int, rank: int, needed_steps: int):
    """Corpus (prepared once by rank 0), packs and the W-rank balanced schedule."""
    from packbalance_b200.data.cost import FlopModel
    from packbalance_b200.data.packer import build_packs, pack_stats
    from packbalance_b200.data.prepare import prepare_synthetic
    from packbalance_b200.data.sampler import build_schedule
    from packbalance_b200.data.store import TokenStore

    data_dir = ROOT / cfg.data.data_dir
    if rank == 0 and not (data_dir / "meta.json").exists():
        prepare_synthetic(cfg.data, data_dir)
    barrier()
    cfg.data.mode = mode
    store = TokenStore.open(data_dir)
    fm = FlopModel.from_config(cfg.model)
    packs = build_packs(store, cfg.data, fm, split="train")
    sched = build_schedule(packs, world, cfg.train.grad_accum, seed=cfg.data.seed, mode=cfg.data.schedule)
    if len(sched.steps) < needed_steps:
        raise SystemExit(f"schedule has {len(sched.steps)} steps, need {needed_steps}; add synthetic docs")
    return store, packs, sched, pack_stats(packs, fm)


def clocks_gpus(world: int) -> list[int]:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        return [int(x) for x in vis.split(",")[:world] if x.strip().isdigit()]
    return list(range(world))


def report(args, world, dev, rank, impl, step_ms_ranks, e2e_ms, tokens_steps, launches, clocks, extra_cfg, h2d, d2h):
    """step_ms_ranks: [world][K] device ms per step."""
    per_step_max = np.max(np.array(step_ms_ranks), axis=0)
    total_ms = max(sum(r) for r in step_ms_ranks)
    tokens = float(sum(tokens_steps))
    value = tokens / (total_ms / 1e3)
    imb = float(np.mean(np.max(step_ms_ranks, 0) / np.mean(step_ms_ranks, 0) - 1.0)) if world > 1 else 0.0
    rec = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps,
        "p99_step_ms": float(np.percentile(per_step_max, 99)),
        "rank_imbalance": imb,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": extra_cfg.pop("data_desc", "synthetic; random-init weights"),
        "config": {**extra_cfg, **({"overrides": list(args.set)} if args.set else {})},
        "clocks": clocks,
        "gpu_launches": launches,
    }
    if impl == "reference":
        rec["impl"] = "reference"
    if e2e_ms is not None:
        rec["e2e"] = {
            "value": tokens / (e2e_ms / 1e3),
            "unit": "tokens/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
        }
    if rank == 0:
        print(json.dumps(rec), flush=True)


def time_steps(fn, steps: int, dev) -> list[float]:
    """Device ms of each of ``steps`` calls, bracketed by barrier + synchronize."""
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    barrier()
    evs[0].record()
    for i in range(steps):
        fn(i)
        evs[i + 1].record()
    torch.cuda.synchronize()
    barrier()
    return [evs[i].elapsed_time(evs[i + 1]) for i in range(steps)]


# ----------------------------------------------------------------------------------
def run_ours(args, rank, world, dev) -> None:
    sys.path.insert(0, str(ROOT))
    from packbalance_b200.config import apply_overrides, load_config
    from packbalance_b200.data.dataset import PackedDataset, batch_tensor_bytes, concat_packs
    from packbalance_b200.ops import _native
    from packbalance_b200.train.engine import TrainEngine, to_device_batch

    cfg = apply_overrides(load_config(args.config), args.set)
    total = args.warmup + args.steps
    store, packs, sched, pstats = build_data(cfg, args.mode, world, rank, total)
    ds = PackedDataset(store, packs, cfg.data)
    A = cfg.train.grad_accum
    plans = sched.steps[:total]
    host = []
    for plan in plans:
        b = concat_packs([ds[i] for i in plan.rank_packs[rank]])
        host.append({k: (v.pin_memory() if isinstance(v, torch.Tensor) else v) for k, v in b.items()})
    torch.manual_seed(cfg.train.seed)
    cfg.train.max_steps = max(cfg.train.max_steps, 4 * total)
    engine = TrainEngine(cfg, dev)
    _native.module()  # fail loudly if the extension is missing

    # inputs staged on the device, each with its attention work lists (built on the host
    # like doc_start; the end-to-end measurement below builds them inside its timed region)
    dev_batches = [to_device_batch(engine.prepare_batch(h), dev) for h in host]
    for i in range(args.warmup):
        engine.step([dev_batches[i]], plans[i].step_tokens)
    torch.cuda.synchronize()
    _native.check_status(dev)

    sampler = ClockSampler(rank == 0, clocks_gpus(world))
    timed = list(range(args.warmup, total))
    ms = time_steps(lambda i: engine.step([dev_batches[timed[i]]], plans[timed[i]].step_tokens), args.steps, dev)
    clocks = sampler.stop(clocks_gpus(world))
    _native.check_status(dev)
    step_ms_ranks = gather(ms, dev)
    free, total_mem = torch.cuda.mem_get_info(dev)
    mem_used_gb = max_over_ranks((total_mem - free) / 1e9, dev)  # everything on the device, max over ranks

    e2e_ms = None
    h2d = batch_tensor_bytes(engine.prepare_batch(host[0]))
    d2h = 4
    if not args.no_e2e:
        from packbalance_b200.train.engine import HostScalars

        # Every step: H2D of its inputs from pinned memory (inside engine.step) and a
        # D2H read of its global loss; the read of step i completes after step i+1 has
        # been launched (HostScalars, lag 1), so host work overlaps the device.
        reader = HostScalars(lag=1)
        losses: list[float] = []

        def e2e_step(i):
            j = timed[i]
            out = engine.step([host[j]], plans[j].step_tokens)
            v = reader.push(engine.global_loss(out["loss_sum"], plans[j].step_tokens))
            if v is not None:
                losses.append(v)

        barrier()
        t0 = time.perf_counter()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for i in range(args.steps):
            e2e_step(i)
        losses += reader.drain()
        ev1.record()
        torch.cuda.synchronize()
        assert len(losses) == args.steps and all(math.isfinite(x) for x in losses), losses
        e2e_ms = max_over_ranks(ev0.elapsed_time(ev1), dev)
        barrier()
        _ = time.perf_counter() - t0

    launches = None
    if not args.no_count:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            engine.step([dev_batches[timed[0]]], plans[timed[0]].step_tokens)
            torch.cuda.synchronize()
        names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
        mine = [n for n in names if "pb::" in n]
        launches = len(mine) * args.steps
        if rank == 0:
            print(f"[bench] kernels per step: {len(mine)} native / {len(names)} total", file=sys.stderr, flush=True)
    if engine.sharded is not None:
        comm = "sharded: all-gather fused into GEMMs, reduce-scatter fused with AdamW (peer memory)"
    elif engine.dp is not None and engine.dp.fused is not None:
        comm = f"fused peer-memory all-reduce ({engine.dp.fused.mode})"
    else:
        comm = "nccl"
    extra = {
        "model": describe_model(cfg.model),
        "global_batch": world * A,
        "global_batch_unit": f"packs of {cfg.data.seq_len} tokens",
        "seq_len": cfg.data.seq_len,
        "parallelism": f"{'fsdp' if engine.fsdp else 'dp'}{world}",
        "packing": args.mode,
        "schedule": cfg.data.schedule,
        "packs_per_rank": A,
        "padding_waste": pstats["padding_waste"],
        "analytical_rank_imbalance": sched.stats()["rank_cost_imbalance"],
        "l2": "no flush; per-step working set (weights+Adam state+activations) >> 126 MB L2",
        "comm": comm,
        "device_mem_used_gb": round(mem_used_gb, 2),
        "data_desc": describe_data(cfg.data),
    }
    report(args, world, dev, rank, "ours", step_ms_ranks, e2e_ms, [p.step_tokens for p in plans[args.warmup:]],
           launches, clocks, extra, h2d, d2h)
    engine.close()


def describe_data(d) -> str:
    """The ``data`` field of the JSON line, from the config actually run."""
    med = d.synthetic_median if d.synthetic_median is not None else math.exp(d.synthetic_mu)
    ids = f"Zipf({d.synthetic_zipf_s:g}) ids" if d.synthetic_token_dist == "zipf" else "uniform ids"
    long_docs = f", {d.synthetic_long_doc_frac:g} of documents {d.seq_len} tokens" if d.synthetic_long_doc_frac else ""
    return (f"synthetic (lognormal median {med:g} sigma {d.synthetic_sigma:g} clipped [{d.synthetic_min_len},"
            f"{d.synthetic_max_len}]{long_docs}, {ids}; random-init weights)")


def describe_model(m) -> str:
    """Model name of the JSON line, from the config actually run."""
    from packbalance_b200.data.cost import FlopModel

    n = FlopModel.from_config(m).total_params
    tie = "tied" if m.tie_embeddings else "untied"
    return (f"llama-{n / 1e6:.0f}M ({m.n_layers}L d{m.d_model} {m.n_heads}H/{m.n_kv_heads}KV ff{m.d_ff} "
            f"V{m.vocab_size} {tie})")


def run_reference(args, rank, world, dev) -> None:
    sys.path.insert(0, str(ROOT))
    from packbalance_b200.utils.reference import locate_reference

    ref_root, tried = locate_reference(ROOT)
    if ref_root is None:
        if rank == 0:
            print(json.dumps({"impl": "reference",
                              "unavailable": "reference not found; tried " + "; ".join(tried)}), flush=True)
        return
    sys.path.insert(0, ref_root)
    from packbalance.config import DataConfig as RDataConfig
    from packbalance.config import ModelConfig as RModelConfig
    from packbalance.config import PackBalanceConfig as RConfig
    from packbalance.config import TrainConfig as RTrainConfig
    from packbalance.data.cost import FlopModel
    from packbalance.data.dataset import PackedDataset, to_device
    from packbalance.data.packer import build_packs, pack_stats
    from packbalance.data.sampler import build_schedule
    from packbalance.data.store import TokenStore
    from packbalance.model.llama import LlamaForCausalLM
    from packbalance.train import train as rtrain
    from packbalance.train.distributed import no_sync, wrap_model

    sys.path.insert(1, str(ROOT))
    from packbalance_b200.config import apply_overrides, load_config
    from packbalance_b200.data.prepare import prepare_synthetic

    ours = apply_overrides(load_config(args.config), args.set)
    data_dir = ROOT / ours.data.data_dir
    if rank == 0 and not (data_dir / "meta.json").exists():
        prepare_synthetic(ours.data, data_dir)  # same corpus format; the reference reads it with its TokenStore
    barrier()
    m, d, t = ours.model, ours.data, ours.train
    rcfg = RConfig(
        model=RModelConfig(vocab_size=m.vocab_size, d_model=m.d_model, n_layers=m.n_layers, n_heads=m.n_heads,
                           n_kv_heads=m.n_kv_heads, d_ff=m.d_ff, max_seq_len=m.max_seq_len,
                           tie_embeddings=m.tie_embeddings, rope_theta=m.rope_theta,
                           gradient_checkpointing=m.gradient_checkpointing, attention_backend="auto",
                           use_fused_ce=True, ce_chunk_size=m.ce_chunk_size),
        data=RDataConfig(dataset="synthetic", data_dir=str(data_dir), seq_len=d.seq_len, mode=args.mode,
                         schedule=d.schedule, max_doc_len=d.max_doc_len, min_doc_len=d.min_doc_len,
                         val_fraction=0.0, seed=d.seed, num_workers=0),
        train=RTrainConfig(grad_accum=t.grad_accum, lr=t.lr, min_lr=t.min_lr, warmup_steps=t.warmup_steps,
                           dtype="bf16", max_steps=1000, grad_clip=t.grad_clip, fsdp=t.fsdp),
    )
    total = args.warmup + args.steps
    store = TokenStore.open(data_dir)
    fm = FlopModel.from_config(rcfg.model)
    packs = build_packs(store, rcfg.data, fm, split="train")
    sched = build_schedule(packs, world, rcfg.train.grad_accum, seed=rcfg.data.seed, mode=rcfg.data.schedule)
    ds = PackedDataset(store, packs, rcfg.data)
    plans = sched.steps[:total]
    host = [[{k: (v.pin_memory() if isinstance(v, torch.Tensor) else v) for k, v in ds[i].items()}
             for i in p.rank_packs[rank]] for p in plans]
    torch.manual_seed(t.seed)
    model = LlamaForCausalLM(rcfg.model).to(dev)
    model = wrap_model(model, rcfg.train, dev)
    opt = rtrain._make_optimizer(model, rcfg)
    A = rcfg.train.grad_accum

    def ref_step(batches, step_tokens, read_loss: bool):
        # The reference trainer's step body (train/train.py:318-362) on its own modules.
        loss_scale = world / step_tokens
        opt.zero_grad(set_to_none=True)
        local = torch.zeros((), device=dev)
        for micro, batch in enumerate(batches):
            batch = to_device(batch, dev)
            with no_sync(model, enabled=world > 1 and micro != A - 1):
                with torch.autocast("cuda", dtype=torch.bfloat16):
                    out = rtrain._forward_microbatch(model, batch, dev, rcfg, need_block_mask=True)
                (out.loss * loss_scale).backward()
            local += out.loss.detach().float()
        rtrain._clip_grads(model, rcfg.train.grad_clip)
        opt.step()
        if read_loss:
            float(rtrain._all_reduce_sum(local) / step_tokens)

    dev_batches = [[to_device(b, dev) for b in hb] for hb in host]
    for i in range(args.warmup):
        ref_step(dev_batches[i], plans[i].step_tokens, False)
    torch.cuda.synchronize()
    sampler = ClockSampler(rank == 0, clocks_gpus(world))
    ms = time_steps(lambda i: ref_step(dev_batches[args.warmup + i], plans[args.warmup + i].step_tokens, False),
                    args.steps, dev)
    clocks = sampler.stop(clocks_gpus(world))
    step_ms_ranks = gather(ms, dev)
    e2e_ms = None
    h2d = sum(v.numel() * v.element_size() for b in host[0] for v in b.values() if isinstance(v, torch.Tensor))
    if not args.no_e2e:
        barrier()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for i in range(args.steps):
            ref_step(host[args.warmup + i], plans[args.warmup + i].step_tokens, True)
        ev1.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(ev0.elapsed_time(ev1), dev)
        barrier()
    extra = {
        "model": describe_model(ours.model),
        "global_batch": world * A,
        "global_batch_unit": f"packs of {rcfg.data.seq_len} tokens",
        "seq_len": rcfg.data.seq_len,
        "parallelism": f"{'fsdp' if rcfg.train.fsdp and world > 1 else 'dp'}{world}",
        "packing": args.mode,
        "schedule": rcfg.data.schedule,
        "packs_per_rank": A,
        "padding_waste": pack_stats(packs, fm)["padding_waste"],
        "l2": "no flush; per-step working set >> 126 MB L2",
        "comm": "torch FSDP2 (NCCL)" if rcfg.train.fsdp and world > 1 else "torch DDP (NCCL)",
        "data_desc": describe_data(ours.data),
    }
    report(args, world, dev, rank, "reference", step_ms_ranks, e2e_ms, [p.step_tokens for p in plans[args.warmup:]],
           None, clocks, extra, h2d, 4)


def main() -> None:
    args = parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if not torch.cuda.is_available():
        rec = {"metric": METRIC, "unavailable": "no CUDA device"}
        if args.impl == "reference":
            rec["impl"] = "reference"
        print(json.dumps(rec), flush=True)
        return
    rank, world, dev = setup_dist(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world, dev)
        else:
            run_ours(args, rank, world, dev)
    finally:
        if dist.is_initialized():
            with contextlib.suppress(Exception):
                dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
