"""One launch of every hot kernel of the 100M training step, for ncu captures.

    python -m packbalance_b200.profiling.profile_kernels [--tokens 8192] [--warmup 1]

Runs each kernel ``--warmup`` times and then once more (the launch to capture) on the
shapes of benchmark config #2 (d_model 768, 12/4 heads of 64, SwiGLU 2048, vocab 32000,
8192 tokens = 4 packs of 2048 from the bench corpus's document-length law), and prints
each kernel's CUDA-event time of the last launch with its algorithmic FLOPs or bytes.
Inputs total a few hundred MB, above the 126 MB L2.

Capture one kernel per ncu run, after the same command has run once without ncu:

    ncu --set full --clock-control none -k <one kernel name> -s <its warm-up launches> -c 1 \
        -o prof python -m packbalance_b200.profiling.profile_kernels --warmup 1

and read the others' times from this script's CUDA-event output (or an ncu run with
``--metrics gpu__time_duration.sum`` only, which takes one pass per launch).

Kernels: QKV GEMM with the RoPE epilogue, gate|up GEMM with the SwiGLU epilogue,
down-projection dgrad GEMM, wgrad GEMM (split-K, fp32 reduce-add), LM-head GEMM with the
CE-forward epilogue, CE-backward (dlogits) GEMM, attention forward and backward,
add+RMSNorm forward, RMSNorm backward, SwiGLU backward, AdamW over 100 M parameters.
"""

from __future__ import annotations

import argparse
import json

import torch

from packbalance_b200.profiling.bench_kernels import bench_doc_lengths, doc_starts, peaks


def main(argv: list[str] | None = None) -> list[dict]:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--warmup", type=int, default=1)
    args = ap.parse_args(argv)

    from packbalance_b200.ops import _native
    from packbalance_b200.ops.attention import attention_plan, attn_backward_packed, attn_forward_packed
    from packbalance_b200.ops.cross_entropy import lmhead_ce_forward
    from packbalance_b200.ops.gemm import EPI_BF16, EPI_CE_BWD, EPI_ROPE, EPI_SWIGLU, gemm, linear_wgrad

    dev = torch.device("cuda")
    C = _native.module()
    pk = peaks()
    T, d, F, V, H, Hk, D = args.tokens, 768, 2048, 32000, 12, 4, 64
    bf = torch.bfloat16
    torch.manual_seed(0)
    rows: list[dict] = []

    def run(name, fn, flops=None, nbytes=None):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        r = {"kernel": name, "ms": ms}
        if flops:
            r["tflops"] = flops / ms / 1e9
            r["frac_of_measured_bf16"] = r["tflops"] / pk["bf16_tflops"]
        if nbytes:
            r["gbs"] = nbytes / ms / 1e6
            r["frac_of_measured_hbm"] = r["gbs"] / pk["hbm_gbs"]
        rows.append(r)
        print(json.dumps(r), flush=True)

    # GEMMs
    x = (torch.randn(T, d, device=dev) * 0.5).to(bf)
    wqkv = (torch.randn((H + 2 * Hk) * D, d, device=dev) * 0.02).to(bf)
    qkv = torch.empty(T, (H + 2 * Hk) * D, device=dev, dtype=bf)
    pos = (torch.arange(T, device=dev) % 2048).to(torch.int32)
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2, device=dev).float() / D))
    ang = torch.outer(torch.arange(2048, device=dev).float(), inv)
    cos, sin = torch.cat([ang, ang], -1).cos().contiguous(), torch.cat([ang, ang], -1).sin().contiguous()
    run("gemm_qkv_rope", lambda: gemm(x, wqkv, qkv, T, qkv.shape[1], d, epi=EPI_ROPE, pos=pos, cos=cos, sin=sin,
                                      head_dim=D, n_rope_cols=(H + Hk) * D), flops=2.0 * T * qkv.shape[1] * d)
    wgu = (torch.randn(2 * F, d, device=dev) * 0.02).to(bf)
    h = torch.empty(T, F, device=dev, dtype=bf)
    gu = torch.empty(T, 2 * F, device=dev, dtype=bf)
    run("gemm_gateup_swiglu", lambda: gemm(x, wgu, h, T, 2 * F, d, epi=EPI_SWIGLU, aux=gu), flops=2.0 * T * 2 * F * d)
    wd = (torch.randn(d, F, device=dev) * 0.02).to(bf)
    dy = (torch.randn(T, d, device=dev) * 0.1).to(bf)
    dh = torch.empty(T, F, device=dev, dtype=bf)
    run("gemm_down_dgrad", lambda: gemm(dy, wd, dh, T, F, d, b_mn=True, epi=EPI_BF16), flops=2.0 * T * F * d)
    gw = torch.empty(d, F, device=dev)
    run("gemm_down_wgrad_splitk", lambda: linear_wgrad(dy, h, gw), flops=2.0 * T * F * d)
    wv = (torch.randn(V, d, device=dev) * 0.02).to(bf)
    tgt = torch.randint(0, V, (T,), device=dev)
    run("lmhead_ce_forward", lambda: lmhead_ce_forward(x, wv, tgt), flops=2.0 * T * V * d)
    _, lse = lmhead_ce_forward(x, wv, tgt)
    rs = torch.full((T,), 1.0 / T, device=dev)
    chunk = 4096
    dl = torch.empty(chunk, V, device=dev, dtype=bf)
    run("gemm_ce_bwd_dlogits", lambda: gemm(x[:chunk], wv, dl, chunk, V, d, epi=EPI_CE_BWD, bn=256, targets=tgt[:chunk],
                                            lse=lse[:chunk], row_scale=rs[:chunk]), flops=2.0 * chunk * V * d)
    # attention on the corpus's document-length law
    lengths = bench_doc_lengths(T)
    ds = doc_starts(lengths, dev)[:T]
    plan = attention_plan(ds, H, Hk)
    qkv_a = torch.randn(T, (H + 2 * Hk) * D, device=dev).to(bf)
    lens = torch.bincount(ds.long()).cpu()
    lens = lens[lens > 0].double()
    pairs = float((lens * (lens + 1) / 2).sum())
    fwd_flops = 4.0 * H * D * pairs
    run("attn_fwd", lambda: attn_forward_packed(qkv_a, plan, H, Hk, D), flops=fwd_flops)
    o, lse_a = attn_forward_packed(qkv_a, plan, H, Hk, D)
    do = torch.randn_like(o)
    run("attn_bwd", lambda: attn_backward_packed(qkv_a, o, do, lse_a, plan, H, Hk, D), flops=2.5 * fwd_flops)
    # memory-bound kernels
    xr = torch.randn(T, d, device=dev)
    delta = torch.randn(T, d, device=dev).to(bf)
    wn = torch.randn(d, device=dev)
    run("add_rmsnorm_fwd", lambda: C.add_rmsnorm_fwd(xr, delta, wn, 1e-5, True), nbytes=T * d * (4 + 2 + 4 + 2))
    xo, _, rstd = C.add_rmsnorm_fwd(xr, delta, wn, 1e-5, True)
    g32 = torch.randn(T, d, device=dev)
    dres = torch.randn(T, d, device=dev)
    dxb = torch.empty(T, d, device=dev, dtype=bf)
    dw = torch.empty(d, device=dev)
    run("rmsnorm_bwd", lambda: C.rmsnorm_bwd(g32, xo, wn, rstd, dres, dxb, dw, False), nbytes=T * d * (4 * 4 + 2))
    dgu = torch.empty(T, 2 * F, device=dev, dtype=bf)
    run("swiglu_bwd_packed", lambda: C.swiglu_bwd_packed(dh, gu, dgu), nbytes=T * F * 2 * 5)
    n = 100_000_000
    p, g, m, v = (torch.randn(n, device=dev) for _ in range(4))
    v.abs_()
    sh = torch.empty(n, device=dev, dtype=bf)
    norm = torch.ones((), device=dev)
    sk = torch.zeros((), device=dev, dtype=torch.int32)
    run("adamw", lambda: C.adamw_step(p, g, m, v, sh, norm, sk, 1e-4, 0.9, 0.95, 1e-8, 0.1, 0.5, 0.5, 1.0, True, None),
        nbytes=n * 30)
    _native.check_status(dev)
    return rows


if __name__ == "__main__":
    main()
