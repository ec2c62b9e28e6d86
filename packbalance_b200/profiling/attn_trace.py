"""Where an attention work item's time goes: per-CTA event traces of the sm_100a kernels.

    python -m packbalance_b200.profiling.attn_trace [--tokens 8192] [--doc-len L] [--json out.json]

Runs the forward and backward kernels once more after warm-up with the kernels' event
trace switched on (``_C.attn_trace``: lane 0 of each role stamps the SM clock at its
steps, ``csrc/attention.cu``), on the bench corpus's document-length law (or fixed
``--doc-len`` documents), 12/4 heads of 64 as in benchmark config #2, and prints per-step
medians over all CTAs and tiles, in SM clock cycles:

forward   S issued -> S read by softmax warp 2 (TMEM result latency), softmax of one
          tile (S read -> P ready), idle between tiles, epilogue per item, tile period
backward  S^T / dP^T issued -> read by gradient warp 2, gradient math of one tile (S^T
          read -> dS^T ready), dS^T ready -> MMA warp sees all warps ready, dV/dK/dQ
          issue, tile period

plus the kernel span per CTA (first to last stamp).  The trace costs one global store per
stamp; the numbers of record for kernel time are bench_kernels' CUDA-event timings.
"""

from __future__ import annotations

import argparse
import json

import numpy as np
import torch

ROLES_FWD = ("q_load", "kv_load", "s_issue", "pv_issue", "s_read", "p_ready", "epi_begin", "epi_end")
ROLES_BWD = ("kv_load", "qd_load", "st_issue", "ds_seen", "mma2_issue", "st_read", "ds_ready", "dkv_done")
N_ROLES, N_EV = 8, 128


def _events(tr: np.ndarray, role: int) -> np.ndarray:
    v = tr[role, : N_EV - 1].astype(np.int64)
    n = int(np.argmax(v == 0)) if (v == 0).any() else v.size  # stamps are written in order from 0
    return v[:n]


def _med(xs: list[np.ndarray]) -> float | None:
    a = np.concatenate([x for x in xs if x.size]) if any(x.size for x in xs) else np.zeros(0)
    return float(np.median(a)) if a.size else None


def summarize(trace: np.ndarray, kind: str) -> dict:
    """``trace``: [CTAs, 8 roles, 128 events] SM clock stamps of one launch."""
    out: dict = {}
    spans = []
    pairs: dict[str, list[np.ndarray]] = {}

    def add(name: str, a: np.ndarray, b: np.ndarray, shift: int = 0) -> None:
        # b[i + shift] - a[i] over the indices both have
        n = min(a.size, b.size - shift)
        if n > 0:
            pairs.setdefault(name, []).append(b[shift : shift + n] - a[:n])

    for cta in range(trace.shape[0]):
        tr = trace[cta]
        t0 = int(tr[0, N_EV - 1])
        ev = [_events(tr, r) for r in range(N_ROLES)]
        last = max((int(e[-1]) for e in ev if e.size), default=t0)
        if t0:
            spans.append(last - t0)
        if kind == "fwd":
            s_iss, s_read, p_ready, e0, e1 = ev[2], ev[4], ev[5], ev[6], ev[7]
            add("s_issue_to_read", s_iss, s_read)
            add("softmax_per_tile", s_read, p_ready)
            add("idle_between_tiles", p_ready, s_read, 1)
            add("epilogue_per_item", e0, e1)
            add("tile_period", s_read, s_read, 1)
        else:
            st_iss, ds_seen, mma2, st_read, ds_ready, dkv = ev[2], ev[3], ev[4], ev[5], ev[6], ev[7]
            add("st_issue_to_read", st_iss, st_read)
            add("gradient_math_per_tile", st_read, ds_ready)
            add("ds_ready_to_mma_warp", ds_ready, ds_seen)
            add("dv_dk_dq_issue", ds_seen, mma2)
            add("tile_period", st_iss, st_iss, 1)
            out["items"] = out.get("items", 0) + int(dkv.size)
    out.update({k: _med(v) for k, v in pairs.items()})
    out["span_per_cta_median"] = float(np.median(spans)) if spans else None
    out["span_per_cta_max"] = float(np.max(spans)) if spans else None
    return {k: (round(v, 1) if isinstance(v, float) else v) for k, v in out.items()}


def main(argv=None) -> dict:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--doc-len", type=int, default=0, help="fixed document length (0: the bench corpus's law)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--json", default=None)
    args = ap.parse_args(argv)
    from packbalance_b200.ops import _native
    from packbalance_b200.ops.attention import attention_plan, attn_backward_packed, attn_forward_packed
    from packbalance_b200.profiling.bench_kernels import bench_doc_lengths, doc_starts

    dev = torch.device("cuda", torch.cuda.current_device())
    C = _native.module()
    h, hk, d = 12, 4, 64
    lengths = bench_doc_lengths(args.tokens) if args.doc_len <= 0 else [args.doc_len] * -(-args.tokens // args.doc_len)
    ds = doc_starts(lengths, dev)[: args.tokens]
    qkv = torch.randn(ds.numel(), (h + 2 * hk) * d, device=dev).to(torch.bfloat16)
    plan = attention_plan(ds, h, hk)
    o, lse = attn_forward_packed(qkv, plan, h, hk, d)
    do = torch.randn_like(o)
    for _ in range(args.warmup):
        attn_forward_packed(qkv, plan, h, hk, d)
        attn_backward_packed(qkv, o, do, lse, plan, h, hk, d)
    torch.cuda.synchronize(dev)
    n_ctas = torch.cuda.get_device_properties(dev).multi_processor_count
    res = {"tokens": int(ds.numel()), "doc_len": args.doc_len or "bench law", "unit": "SM clock cycles"}
    for kind in ("fwd", "bwd"):
        buf = torch.zeros(n_ctas * N_ROLES * N_EV, dtype=torch.int64, device=dev)
        C.attn_trace(buf.data_ptr())
        try:
            if kind == "fwd":
                attn_forward_packed(qkv, plan, h, hk, d)
            else:
                attn_backward_packed(qkv, o, do, lse, plan, h, hk, d)
            torch.cuda.synchronize(dev)
        finally:
            C.attn_trace(0)
        res[kind] = summarize(buf.view(n_ctas, N_ROLES, N_EV).cpu().numpy(), kind)
    _native.check_status(dev)
    print(json.dumps(res))
    if args.json:
        with open(args.json, "w", encoding="utf-8") as fh:
            json.dump(res, fh, indent=1)
    return res


if __name__ == "__main__":
    main()
