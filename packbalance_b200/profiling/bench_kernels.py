"""Kernel microbenchmarks (reference ``profiling/bench_kernels.py``) plus the sm100 kernels.

Every case is timed with CUDA events on the launching stream after warm-up, with a
synchronize on both sides, and reported with its roofline fraction against the
measured peaks in ``MEASURED_PEAKS.json`` (copy bandwidth and cuBLAS bf16 burst).

Cases (``--cases``, comma separated):
  rmsnorm, swiglu          fp32 8192 x 768 (the reference's shapes; bytes model of the reference)
  ce                       fused LM-head CE fwd+bwd, T x d x V (6 T d V FLOPs)
  gemm                     the 100M model's GEMM shapes (fwd / dgrad / wgrad)
  attn_fwd, attn_bwd       document-masked attention on the bench corpus's document lengths

``--iters 1 --warmup 1`` with ``--cases attn_bwd`` gives a single launch for an ncu capture.
"""

from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def timeit(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def doc_starts(lengths: list[int], device) -> torch.Tensor:
    out, off = [], 0
    for n in lengths:
        out += [off] * n
        off += n
    return torch.tensor(out, device=device, dtype=torch.int32)


def bench_doc_lengths(total: int, seed: int = 0) -> list[int]:
    """Packs of 2048 tokens filled with lognormal(median 256, sigma 1.2) documents."""
    rng = np.random.default_rng(seed)
    lengths: list[int] = []
    while sum(lengths) < total:
        room = 2048
        while room > 0:
            n = int(np.clip(rng.lognormal(math.log(256), 1.2), 16, 2048))
            n = min(n, room)
            lengths.append(n)
            room -= n
    return lengths[: len(lengths)]


def run(args) -> list[dict]:
    from packbalance_b200.ops import _native
    from packbalance_b200.ops.attention import attention_plan, attn_backward_packed, attn_forward_packed
    from packbalance_b200.ops.cross_entropy import linear_cross_entropy
    from packbalance_b200.ops.gemm import EPI_BF16, EPI_ROPE, EPI_SWIGLU, EPI_SWIGLU_BWD, gemm, linear_wgrad
    from packbalance_b200.ops.reference import rmsnorm_reference, swiglu_reference
    from packbalance_b200.ops.rmsnorm import rmsnorm
    from packbalance_b200.ops.swiglu import swiglu

    dev = torch.device(args.device)
    pk = peaks()
    cases = args.cases.split(",")
    res: list[dict] = []

    def add(name, ms, flops=None, nbytes=None, **kw):
        rec = {"case": name, "ms": ms, **kw}
        if flops:
            rec["tflops"] = flops / ms / 1e9
            rec["frac_of_" + pk["source"] + "_bf16"] = rec["tflops"] / pk["bf16_tflops"]
        if nbytes:
            rec["gbs"] = nbytes / ms / 1e6
            rec["frac_of_" + pk["source"] + "_hbm"] = rec["gbs"] / pk["hbm_gbs"]
        res.append(rec)
        print(json.dumps(rec), flush=True)

    if "rmsnorm" in cases:
        x = torch.randn(args.rows, args.dim, device=dev)
        w = torch.ones(args.dim, device=dev)
        nb = 2 * args.rows * args.dim * 4 + args.dim * 4
        add("rmsnorm_ref", timeit(lambda: rmsnorm_reference(x, w, 1e-5), args.iters, args.warmup), nbytes=nb)
        add("rmsnorm_native", timeit(lambda: rmsnorm(x, w, 1e-5), args.iters, args.warmup), nbytes=nb)
    if "swiglu" in cases:
        g = torch.randn(args.rows, args.dim, device=dev)
        u = torch.randn(args.rows, args.dim, device=dev)
        nb = 3 * args.rows * args.dim * 4
        add("swiglu_ref", timeit(lambda: swiglu_reference(g, u), args.iters, args.warmup), nbytes=nb)
        add("swiglu_native", timeit(lambda: swiglu(g, u), args.iters, args.warmup), nbytes=nb)
    if "ce" in cases:
        t, d, v = args.tokens, args.ce_dim, args.vocab
        x = (torch.randn(t, d, device=dev) * 0.5).to(torch.bfloat16).requires_grad_()
        w = (torch.randn(v, d, device=dev) * 0.02).to(torch.bfloat16).requires_grad_()
        tgt = torch.randint(0, v, (t,), device=dev)

        def ce():
            loss = linear_cross_entropy(x, w, tgt)
            loss.backward()
            x.grad = None
            w.grad = None

        add("linear_ce_fused_fwd_bwd", timeit(ce, args.iters, args.warmup), flops=6.0 * t * d * v, shape=[t, d, v])
    if "lmhead" in cases:
        # the training step's LM head (T = 4 packs of 2048): logits recomputed in the
        # backward vs kept from the forward, forward and backward timed separately
        from packbalance_b200.ops.cross_entropy import lmhead_ce_backward, lmhead_ce_forward

        t, d, v = args.tokens * 4, args.ce_dim, args.vocab
        x = (torch.randn(t, d, device=dev) * 0.5).to(torch.bfloat16)
        w = (torch.randn(v, d, device=dev) * 0.02).to(torch.bfloat16)
        tgt = torch.randint(0, v, (t,), device=dev)
        g = torch.tensor(1.0 / t, device=dev)
        dw = torch.empty(v, d, device=dev)
        logits = torch.empty(t, v, device=dev, dtype=torch.bfloat16)
        for keep in (False, True):
            lo = logits if keep else None
            tag = "kept" if keep else "recomputed"
            add(f"lmhead_fwd_{tag}", timeit(lambda: lmhead_ce_forward(x, w, tgt, logits_out=lo), args.iters,
                                           args.warmup), flops=2.0 * t * d * v, shape=[t, d, v])
            _, lse = lmhead_ce_forward(x, w, tgt, logits_out=lo)

            def bwd():
                if keep:
                    lmhead_ce_forward(x, w, tgt, logits_out=lo)  # refill: the backward overwrites them
                lmhead_ce_backward(x, w, tgt, lse, g, dw, False, logits=lo)

            ms = timeit(bwd, args.iters, args.warmup)
            if keep:
                ms -= res[-1]["ms"]  # minus the forward that refilled the logits (timed just above)
            add(f"lmhead_bwd_{tag}", ms, flops=(4.0 if keep else 6.0) * t * d * v, shape=[t, d, v])
        # recomputing backward with smaller dlogits chunks (a chunk of 1024 rows x 32000 is
        # 65 MB of bf16 and stays in the 126 MB L2 between its GEMMs)
        for rows in (1024, 2048, 4096):
            add(f"lmhead_bwd_recomputed_chunk{rows}",
                timeit(lambda: lmhead_ce_backward(x, w, tgt, lse, g, dw, False, chunk_rows=rows), args.iters,
                       args.warmup), flops=6.0 * t * d * v, shape=[t, d, v])
    if "gemm" in cases:
        t = args.tokens * 4
        for name, (m, n, k) in {"qkv": (t, 1280, 768), "o": (t, 768, 768), "gateup": (t, 4096, 768),
                                "down": (t, 768, 2048)}.items():
            a = torch.randn(m, k, device=dev).to(torch.bfloat16)
            b = torch.randn(n, k, device=dev).to(torch.bfloat16)
            o = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
            add(f"gemm_fwd_{name}", timeit(lambda: gemm(a, b, o, m, n, k, epi=EPI_BF16), args.iters, args.warmup),
                flops=2.0 * m * n * k, shape=[m, n, k])
            # the library's bf16 GEMM on the same shape (baseline for the tile-count effects)
            add(f"gemm_fwd_{name}_cublas", timeit(lambda: torch.matmul(a, b.t(), out=o), args.iters, args.warmup),
                flops=2.0 * m * n * k, shape=[m, n, k])
            dy = torch.randn(m, n, device=dev).to(torch.bfloat16)
            gw = torch.empty(n, k, device=dev)
            add(f"gemm_wgrad_{name}", timeit(lambda: linear_wgrad(dy, a, gw), args.iters, args.warmup),
                flops=2.0 * m * n * k, shape=[n, k, m])
        # the fused forward epilogues of the training step
        m, k = t, 768
        a = torch.randn(m, k, device=dev).to(torch.bfloat16)
        wgu = torch.randn(4096, k, device=dev).to(torch.bfloat16)
        h = torch.empty(m, 2048, device=dev, dtype=torch.bfloat16)
        gu = torch.empty(m, 4096, device=dev, dtype=torch.bfloat16)
        add("gemm_fwd_gateup_swiglu", timeit(lambda: gemm(a, wgu, h, m, 4096, k, epi=EPI_SWIGLU, aux=gu), args.iters,
                                             args.warmup), flops=2.0 * m * 4096 * k, shape=[m, 4096, k])
        dy = torch.randn(m, k, device=dev).to(torch.bfloat16)
        wd = torch.randn(k, 2048, device=dev).to(torch.bfloat16)
        dgu = torch.empty(m, 4096, device=dev, dtype=torch.bfloat16)
        add("gemm_dgrad_down_swiglu_bwd", timeit(lambda: gemm(dy, wd, dgu, m, 2048, k, b_mn=True, epi=EPI_SWIGLU_BWD,
                                                               aux=gu), args.iters, args.warmup),
            flops=2.0 * m * 2048 * k, shape=[m, 2048, k])
        wqkv = torch.randn(1280, k, device=dev).to(torch.bfloat16)
        qkv = torch.empty(m, 1280, device=dev, dtype=torch.bfloat16)
        pos = (torch.arange(m, device=dev) % 2048).to(torch.int32)
        inv = 1.0 / (10000.0 ** (torch.arange(0, 64, 2, device=dev).float() / 64))
        ang = torch.outer(torch.arange(2048, device=dev).float(), inv)
        cos, sin = torch.cat([ang, ang], -1).cos(), torch.cat([ang, ang], -1).sin()
        add("gemm_fwd_qkv_rope", timeit(lambda: gemm(a, wqkv, qkv, m, 1280, k, epi=EPI_ROPE, pos=pos, cos=cos, sin=sin,
                                                     head_dim=64, n_rope_cols=1024), args.iters, args.warmup),
            flops=2.0 * m * 1280 * k, shape=[m, 1280, k])
        # large square GEMM: the kernel's main loop against cuBLAS (library baseline)
        n = 8192
        a = torch.randn(n, n, device=dev).to(torch.bfloat16)
        b = torch.randn(n, n, device=dev).to(torch.bfloat16)
        o = torch.empty(n, n, device=dev, dtype=torch.bfloat16)
        add("gemm_8192_sm100", timeit(lambda: gemm(a, b, o, n, n, n, epi=EPI_BF16), args.iters, args.warmup),
            flops=2.0 * n ** 3, shape=[n, n, n])
        add("gemm_8192_cublas", timeit(lambda: torch.matmul(a, b.t(), out=o), args.iters, args.warmup),
            flops=2.0 * n ** 3, shape=[n, n, n])
    if "attn_fwd" in cases or "attn_bwd" in cases:
        h, hk, d = 12, 4, 64
        # --doc-len L: every document L tokens long (per-item overheads amortised over
        # more key/query tiles); default: the bench corpus's length law
        lengths = bench_doc_lengths(args.tokens * 4) if args.doc_len <= 0 else \
            [args.doc_len] * -(-(args.tokens * 4) // args.doc_len)
        ds = doc_starts(lengths, dev)[: args.tokens * 4]
        t = ds.numel()
        qkv = torch.randn(t, (h + 2 * hk) * d, device=dev).to(torch.bfloat16)
        plan = attention_plan(ds, h, hk)
        lens = np.bincount(ds.cpu().numpy())
        lens = lens[lens > 0]
        pairs = float((lens * (lens + 1) / 2).sum())
        fwd_flops = 4.0 * h * d * pairs
        if "attn_fwd" in cases:
            add("attn_fwd", timeit(lambda: attn_forward_packed(qkv, plan, h, hk, d), args.iters, args.warmup),
                flops=fwd_flops, tokens=t)
        if "attn_bwd" in cases:
            o, lse = attn_forward_packed(qkv, plan, h, hk, d)
            do = torch.randn_like(o)
            add("attn_bwd", timeit(lambda: attn_backward_packed(qkv, o, do, lse, plan, h, hk, d), args.iters,
                                   args.warmup), flops=2.5 * fwd_flops, tokens=t)
    _native.check_status(dev)
    return res


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--cases", default="rmsnorm,swiglu,ce,gemm,attn_fwd,attn_bwd")
    ap.add_argument("--rows", type=int, default=8192)
    ap.add_argument("--dim", type=int, default=768)
    ap.add_argument("--tokens", type=int, default=2048)
    ap.add_argument("--ce-dim", type=int, default=768)
    ap.add_argument("--vocab", type=int, default=32000)
    ap.add_argument("--doc-len", type=int, default=0, help="attention cases: fixed document length (0: bench law)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--output", default=None)
    ap.add_argument("--pair", type=int, default=-1,
                    help="GEMMs with 256-wide tiles on CTA pairs (1) or single CTAs (0); default: the library default")
    args = ap.parse_args()
    if args.pair >= 0:
        from packbalance_b200.ops import _native

        _native.module().gemm_pair_mode(args.pair)
    res = run(args)
    if args.output:
        Path(args.output).parent.mkdir(parents=True, exist_ok=True)
        Path(args.output).write_text(json.dumps(res, indent=2))


if __name__ == "__main__":
    main()
