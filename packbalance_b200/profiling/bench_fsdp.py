"""Sharded-engine collectives: fused kernels against NCCL, with roofline fractions.

    torchrun --nproc-per-node N -m packbalance_b200.profiling.bench_fsdp [--config configs/b4_1b_fsdp.yaml]
             [--tokens 8192] [--iters 10]

On one decoder layer of the config's shape (sharded over the N ranks):

* ``ag_gemm_qkv`` / ``ag_gemm_gateup``: the QKV (and gate|up + SwiGLU) GEMM with the
  weight all-gather fused in (copy warps fetch the peer chunks while the MMAs run),
  against the same GEMM on weights that are already local, and against
  ``all_gather_into_tensor`` (NCCL) followed by the GEMM.  Roofline: the slower of
  2 M N K / bf16 peak and the bytes this rank must receive, (W - 1) / W of the bf16
  weight segment, at the measured 770 GB/s peer bandwidth.
* ``reduce_scatter``: the per-unit fp32 gradient reduce-scatter kernel against NCCL
  ``reduce_scatter_tensor``.  Roofline: (W - 1) / W of the unit's fp32 gradient over
  NVLink.
* ``adamw_step``: the optimizer step of the sharded engine (norm all-reduce of the
  replicated RMSNorm weights + the fused reduce-scatter/AdamW kernel over the whole
  shard).  Roofline: the shard's optimizer bytes (read p, m, v, g; write p, m, v and
  the bf16 copy: 30 B per element) at the measured HBM bandwidth.

CUDA-event timing on the launching stream after warm-up, max over ranks.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
from dataclasses import replace
from pathlib import Path

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0


def peaks() -> tuple[float, float]:
    p = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 1590.0, 6650.0


def timed(fn, iters: int, dev) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    t = torch.tensor([a.elapsed_time(b) / iters], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--config", default="configs/b4_1b_fsdp.yaml")
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    from packbalance_b200.config import load_config
    from packbalance_b200.models.llama import LlamaForCausalLM
    from packbalance_b200.ops.gemm import EPI_BF16, EPI_SWIGLU, gemm
    from packbalance_b200.parallel.sharded import ShardedParameters

    cfg = load_config(args.config)
    mcfg = replace(cfg.model, n_layers=1)
    torch.manual_seed(0)
    model = LlamaForCausalLM(mcfg).to(dev)
    sp = ShardedParameters(model)
    tf, hbm = peaks()
    T, d, F = args.tokens, mcfg.d_model, mcfg.d_ff
    nqkv = (mcfg.n_heads + 2 * mcfg.n_kv_heads) * mcfg.head_dim
    layer = model.model.layers[0]
    a, mlp = layer.self_attn, layer.mlp
    x = torch.randn(T, d, device=dev, dtype=torch.bfloat16)
    res: dict[str, dict] = {}

    def ag_case(name, params, n_out, epi, seg_params):
        u, seg = sp._segment(params[0])
        seg_bytes = 2 * (seg[1] - seg[0])
        w_full = sp.shadow_of(*params)
        out = torch.empty(T, n_out // (2 if epi == EPI_SWIGLU else 1), device=dev, dtype=torch.bfloat16)
        aux = torch.empty(T, n_out, device=dev, dtype=torch.bfloat16) if epi == EPI_SWIGLU else None
        n = w_full.shape[0]

        def fused():
            sp._gathered_segs.discard(seg)
            gemm(x, w_full, out, T, n, d, epi=epi, aux=aux, ag=sp.gather_spec(*params))

        def local_only():
            gemm(x, w_full, out, T, n, d, epi=epi, aux=aux)

        shard = sp.owned[u.soff: u.soff + u.cs].clone()
        full = torch.empty(world * u.cs, device=dev, dtype=torch.bfloat16)

        def nccl():
            dist.all_gather_into_tensor(full, shard)
            gemm(x, w_full, out, T, n, d, epi=epi, aux=aux)

        t_f, t_l, t_n = timed(fused, args.iters, dev), timed(local_only, args.iters, dev), timed(nccl, args.iters, dev)
        flops = 2.0 * T * n * d
        remote = seg_bytes * (world - 1) / world
        roof_ms = max(flops / (tf * 1e9), remote / (NVLINK_GBS * 1e6))
        res[name] = {"fused_ms": t_f, "gemm_only_ms": t_l, "nccl_ag_then_gemm_ms": t_n, "roofline_ms": roof_ms,
                     "frac_of_roofline": roof_ms / t_f, "remote_mb": remote / 1e6, "tflops_fused": flops / t_f / 1e9}

    ag_case("ag_gemm_qkv", (a.q_proj.weight, a.k_proj.weight, a.v_proj.weight), nqkv, EPI_BF16, None)
    ag_case("ag_gemm_gateup", (mlp.gate_proj.weight, mlp.up_proj.weight), 2 * F, EPI_SWIGLU, None)

    # reduce-scatter of one layer unit
    u = sp.units[1]
    ug = sp._unit_grad(u)  # where the unit's gradient lives (a rotating window for layers)
    ug.normal_()
    out = torch.empty(u.cs, device=dev)

    def rs_fused(tail):
        def run():
            sp._issued.discard(u.order)
            sp._issue_rs(u, tail=tail)
            torch.cuda.current_stream().wait_stream(sp.comm)

        return run

    def rs_nccl():
        dist.reduce_scatter_tensor(out, ug)

    # narrow: the launch width used beside the backward pass; tail: the whole GPU
    t_f, t_w = timed(rs_fused(False), args.iters, dev), timed(rs_fused(True), args.iters, dev)
    t_n = timed(rs_nccl, args.iters, dev)
    byt = 4 * world * u.cs * (world - 1) / world
    roof = byt / (NVLINK_GBS * 1e6)
    res["reduce_scatter"] = {"fused_ms": t_f, "fused_tail_ms": t_w, "nccl_ms": t_n, "roofline_ms": roof,
                             "frac_of_roofline": roof / t_f, "frac_of_roofline_tail": roof / t_w,
                             "unit_mb_fp32": 4 * world * u.cs / 1e6}

    def opt():
        sp._issued = {v.order for v in sp.units}
        sp.optimizer_step(1e-4, 0.9, 0.95, 1e-8, 0.1, 0.1, 0.01, 1.0)

    t_o = timed(opt, args.iters, dev)
    byt = 30.0 * sp.shard_numel
    roof = byt / (hbm * 1e6)
    res["adamw_step"] = {"ms": t_o, "shard_elems": sp.shard_numel, "roofline_ms": roof, "frac_of_roofline": roof / t_o}
    sp.check()
    if rank == 0:
        print(json.dumps({"world": world, "mode": sp.mode, "config": args.config, "tokens": T, "peaks": {"bf16_tflops": tf,
                          "hbm_gbs": hbm, "nvlink_gbs": NVLINK_GBS}, **res}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
