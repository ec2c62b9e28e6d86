"""Gradient all-reduce microbenchmark: fused peer-memory kernel vs NCCL.

    torchrun --nproc-per-node N -m packbalance_b200.profiling.bench_comm [--mb 400] [--buckets 16]

Averages an fp32 buffer of ``--mb`` MB split into ``--buckets`` contiguous buckets (the
flat gradient of the 100M model is 400 MB in 16 x 25 MB buckets), timed with CUDA events
on the launching stream, max over ranks.  The roofline is the NVLink bytes a two-shot
all-reduce must move per rank, 2 (W - 1) / W x size, at the measured 770 GB/s peer-copy
bandwidth per direction.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--mb", type=float, default=400.0)
    ap.add_argument("--buckets", type=int, default=16)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--ctas", type=int, default=0, help="override the fused kernel's CTA count")
    ap.add_argument("--modes", default="p2p,auto", help="fused kernel variants to time (p2p, nvls, auto)")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from packbalance_b200.parallel.comm import FusedAllReduce

    n = int(args.mb * 1e6 / 4) // 4 * 4
    grad = torch.randn(n, device=dev)
    cuts = [round(i * n / args.buckets) // 4 * 4 for i in range(args.buckets)] + [n]
    fused_by_mode = {}
    for m in args.modes.split(","):
        f = FusedAllReduce(grad, mode=m)
        if args.ctas:
            f.ctas = f.ctas_tail = args.ctas
        fused_by_mode[f"fused_{f.mode}"] = f

    def runner(f, tail):
        def run():
            f.start_step()
            for lo, hi in zip(cuts[:-1], cuts[1:]):
                f.all_reduce_mean(lo, hi, tail=tail)

        return run

    def run_nccl():
        for lo, hi in zip(cuts[:-1], cuts[1:]):
            dist.all_reduce(grad[lo:hi])

    res = {}
    # narrow: the launch width used beside the backward pass; tail: the whole GPU
    cases = [(f"{k}_{w}", runner(f, w == "tail")) for k, f in fused_by_mode.items() for w in ("narrow", "tail")]
    for name, fn in [*cases, ("nccl", run_nccl)]:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        ms = torch.tensor([a.elapsed_time(b) / args.iters], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        t = float(ms.item())
        need = 2 * (world - 1) / world * n * 4
        res[name] = {"ms": t, "busbw_gbs": need / t / 1e6, "frac_of_nvlink_770": need / t / 1e6 / NVLINK_GBS}
    for f in fused_by_mode.values():
        f.check()
    f0 = next(iter(fused_by_mode.values()))
    if rank == 0:
        print(json.dumps({"world": world, "mb": args.mb, "buckets": args.buckets, "ctas_narrow": f0.ctas,
                          "ctas_tail": f0.ctas_tail, **res}), flush=True)
    for f in fused_by_mode.values():
        f.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
