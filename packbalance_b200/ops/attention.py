"""Document-masked causal GQA attention over a packed token stream.

Layout: one bf16 buffer ``qkv`` of shape ``[T, (H + 2*Hkv) * D]`` (the fused QKV GEMM
output, RoPE already applied to the q and k columns).  Token ``q`` attends to key
``k`` iff ``doc_start[q] <= k <= q``; the kernel never touches a key tile that lies
outside every document of its query tile.

Work items are (query tile of 128 tokens, head) for the forward and (key tile, kv
head) for the backward.  :func:`attention_plan` orders them by their number of
key / query tiles, most expensive first, so the long documents that dominate the
step start first and short ones fill the tail (the per-tile cost is the cost
model's O(L^2) attention term at tile granularity), and deals them to the kernels'
persistent CTAs so that every CTA's total cost is close to the mean.  :func:`attention_plan_host`
builds the plan with numpy next to the rest of the batch on the host (the trainer
ships it with the step's inputs); :func:`attention_plan` builds the same plan on the
device with a few torch ops and no host synchronisation, for batches that arrive
without one.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from packbalance_b200.ops import _native
from packbalance_b200.ops.reference import varlen_attention_reference

TILE = 128
# The kernels run min(items, SMs) persistent CTAs and CTA b takes items b, b + G, ...;
# the plans deal the cost-sorted items for G = PLAN_CTAS (B200: 148 SMs).
PLAN_CTAS = 148


def _deal_order(n: int, g: int) -> np.ndarray:
    """Position -> rank in the cost-sorted item list.  Items are dealt to the G CTAs in
    rounds of G, alternate rounds in reverse and the first round reversed: a CTA that
    takes a heavy item in one round takes a light one in the next, and the CTAs that
    get one item more in the short last round (the first ones) start with the lightest
    items of the first round.  On the bench corpus the busiest CTA's load drops from
    1.22x the mean (plain round-robin) to 1.05x."""
    p = np.arange(n, dtype=np.int64)
    r0 = (p // g) * g
    m = np.minimum(g, n - r0)
    b = p - r0
    return r0 + np.where((p // g) % 2 == 0, m - 1 - b, b)


_DEAL_CACHE: dict[tuple[int, int, str], torch.Tensor] = {}


def _deal_tensor(n: int, g: int, dev: torch.device) -> torch.Tensor:
    """:func:`_deal_order` as a device tensor, cached per (items, CTAs, device): the
    device-built plans copy it to the GPU once, not on every call."""
    key = (n, g, str(dev))
    t = _DEAL_CACHE.get(key)
    if t is None:
        if len(_DEAL_CACHE) >= 64:
            _DEAL_CACHE.clear()
        t = _DEAL_CACHE[key] = torch.from_numpy(_deal_order(n, g)).to(dev)
    return t


def plan_ctas(device: torch.device) -> int:
    """Persistent CTAs the attention kernels run on ``device`` (its SM count; PLAN_CTAS
    off the GPU)."""
    if device.type != "cuda":
        return PLAN_CTAS
    from packbalance_b200.ops.gemm import sm_count

    return sm_count(device)


def doc_end_from_start(doc_start: torch.Tensor) -> torch.Tensor:
    t = doc_start.numel()
    idx = torch.arange(t, device=doc_start.device, dtype=torch.int64)
    last = torch.ones(t, device=doc_start.device, dtype=torch.bool)
    if t > 1:
        last[:-1] = doc_start[1:] != doc_start[:-1]
    marks = torch.where(last, idx, torch.full_like(idx, t))
    return torch.flip(torch.cummin(torch.flip(marks, (0,)), dim=0).values, (0,))


def attention_plan(doc_start: torch.Tensor, n_heads: int, n_kv_heads: int,
                   n_ctas: int | None = None) -> dict[str, torch.Tensor]:
    """Cost-ordered work lists: ``fwd`` int32 [nq*H, 3] = (q tile, head, first kv tile);
    ``bwd`` int32 [nk*H, 3] = (kv tile, q head, last q tile), dealt to ``n_ctas``
    persistent CTAs by :func:`_deal_order`.  The GQA heads of a kv head are separate
    backward items; their dK/dV add up in an fp32 accumulator.  Also returns
    ``doc_end`` (last token of each token's document)."""
    dev = doc_start.device
    if n_ctas is None:
        n_ctas = plan_ctas(dev)
    t = doc_start.numel()
    n_tiles = -(-t // TILE)
    tiles = torch.arange(n_tiles, device=dev, dtype=torch.int64)
    ds = doc_start.to(torch.int64)
    kv_lo = ds[tiles * TILE] // TILE
    q_cost = tiles - kv_lo + 1
    order = torch.argsort(q_cost, descending=True, stable=True)
    heads = torch.arange(n_heads, device=dev, dtype=torch.int64)
    fwd = torch.stack(
        [order.repeat_interleave(n_heads), heads.repeat(n_tiles), kv_lo[order].repeat_interleave(n_heads)], dim=1
    ).to(torch.int32).contiguous()
    de = doc_end_from_start(ds)
    last_row = torch.clamp(tiles * TILE + TILE - 1, max=t - 1)
    q_hi = de[last_row] // TILE
    k_cost = q_hi - tiles + 1
    korder = torch.argsort(k_cost, descending=True, stable=True)
    bwd = torch.stack(
        [korder.repeat_interleave(n_heads), heads.repeat(n_tiles), q_hi[korder].repeat_interleave(n_heads)],
        dim=1,
    ).to(torch.int32)
    deal = _deal_tensor(n_tiles * n_heads, n_ctas, dev)
    fwd = fwd[deal].contiguous()
    bwd = bwd[deal].contiguous()
    return {
        "fwd": fwd,
        "bwd": bwd,
        "doc_start": doc_start.to(torch.int32).contiguous(),
        "doc_end": de.to(torch.int32).contiguous(),
    }


ALIGN = 8


def _plan_np(ds: np.ndarray, n_heads: int, n_ctas: int = PLAN_CTAS) -> dict[str, np.ndarray]:
    t = ds.shape[0]
    n_tiles = -(-t // TILE)
    tiles = np.arange(n_tiles, dtype=np.int64)
    kv_lo = ds[tiles * TILE].astype(np.int64) // TILE
    order = np.argsort(-(tiles - kv_lo + 1), kind="stable")
    heads = np.arange(n_heads, dtype=np.int64)
    fwd = np.stack([np.repeat(order, n_heads), np.tile(heads, n_tiles), np.repeat(kv_lo[order], n_heads)], axis=1)
    last = np.ones(t, dtype=bool)
    last[:-1] = ds[1:] != ds[:-1]
    marks = np.where(last, np.arange(t), t)
    de = np.minimum.accumulate(marks[::-1])[::-1]
    q_hi = de[np.minimum(tiles * TILE + TILE - 1, t - 1)] // TILE
    korder = np.argsort(-(q_hi - tiles + 1), kind="stable")
    bwd = np.stack([np.repeat(korder, n_heads), np.tile(heads, n_tiles), np.repeat(q_hi[korder], n_heads)], axis=1)
    deal = _deal_order(n_tiles * n_heads, n_ctas)
    fwd, bwd = fwd[deal], bwd[deal]
    return {"fwd": np.ascontiguousarray(fwd, dtype=np.int32), "bwd": np.ascontiguousarray(bwd, dtype=np.int32),
            "doc_start": ds.astype(np.int32),
            "doc_end": de.astype(np.int32)}


def attention_plan_host(doc_start, n_heads: int, n_ctas: int = PLAN_CTAS) -> dict:
    """:func:`attention_plan` on the host (numpy; CPU tensors out), including the
    ALIGN-padded variant when the token count is not a multiple of ALIGN."""
    ds = np.asarray(doc_start.cpu() if isinstance(doc_start, torch.Tensor) else doc_start).astype(np.int64).reshape(-1)
    plan: dict = {k: torch.from_numpy(v) for k, v in _plan_np(ds, n_heads, n_ctas).items()}
    t = ds.shape[0]
    tp = -(-t // ALIGN) * ALIGN
    if tp != t:
        padded = np.concatenate([ds, np.arange(t, tp, dtype=np.int64)])
        plan["padded"] = {k: torch.from_numpy(v) for k, v in _plan_np(padded, n_heads, n_ctas).items()}
    return plan


def plan_to_device(plan: dict, device: torch.device) -> dict:
    return {k: (plan_to_device(v, device) if isinstance(v, dict) else v.to(device, non_blocking=True))
            for k, v in plan.items()}


def _padded(plan: dict, n_heads: int, n_kv_heads: int, t: int) -> dict:
    """Plan for ``t`` padded up to a multiple of ALIGN tokens (each pad token is its own
    one-token document), cached in the plan."""
    tp = -(-t // ALIGN) * ALIGN
    if tp == t:
        return plan
    if "padded" not in plan:
        ds = plan["doc_start"]
        extra = torch.arange(t, tp, device=ds.device, dtype=torch.int32)
        plan["padded"] = attention_plan(torch.cat([ds, extra]), n_heads, n_kv_heads)
    return plan["padded"]


def _pad_rows(x: torch.Tensor, rows: int) -> torch.Tensor:
    if x.shape[0] == rows:
        return x
    return torch.cat([x, x.new_zeros(rows - x.shape[0], *x.shape[1:])])


def attn_forward_packed(
    qkv: torch.Tensor, plan: dict, n_heads: int, n_kv_heads: int, head_dim: int
) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (out ``[T, H*D]`` bf16, lse ``[H, T]`` fp32 natural log)."""
    t = qkv.shape[0]
    pl = _padded(plan, n_heads, n_kv_heads, t)
    tp = pl["doc_start"].numel()
    qkv_p = _pad_rows(qkv, tp)
    out = torch.empty(tp, n_heads * head_dim, device=qkv.device, dtype=torch.bfloat16)
    o, lse = _native.module().attn_fwd(
        qkv_p, pl["doc_start"], pl["fwd"], n_heads, n_kv_heads, head_dim, 1.0 / math.sqrt(head_dim), out
    )
    if tp != t:
        return o[:t], lse[:, :t].contiguous()
    return o, lse


def attn_backward_packed(
    qkv: torch.Tensor,
    out: torch.Tensor,
    dout: torch.Tensor,
    lse: torch.Tensor,
    plan: dict,
    n_heads: int,
    n_kv_heads: int,
    head_dim: int,
    rope: tuple | None = None,
) -> torch.Tensor:
    """Returns dqkv ``[T, (H + 2 Hkv) * D]`` bf16.  With ``rope = (pos, cos, sin)`` the q
    and k gradients are rotated back to the pre-RoPE frame (the gradient w.r.t. the QKV
    GEMM output); without it they are w.r.t. the rotated q/k."""
    t = qkv.shape[0]
    if _native.deterministic():
        return _attn_backward_fixed_order(qkv, dout, plan["doc_start"][:t], n_heads, n_kv_heads, head_dim, rope)
    pl = _padded(plan, n_heads, n_kv_heads, t)
    tp = pl["doc_start"].numel()
    if tp != t:
        qkv, out, dout = _pad_rows(qkv, tp), _pad_rows(out, tp), _pad_rows(dout, tp)
        lse = torch.cat([lse, lse.new_zeros(lse.shape[0], tp - t)], dim=1)
        if rope is not None:
            rope = (_pad_rows(rope[0], tp), rope[1], rope[2])
    dqkv = torch.empty_like(qkv)
    dq_acc = torch.empty(tp, n_heads * head_dim, device=qkv.device, dtype=torch.float32)
    dkv_acc = torch.empty(tp, 2 * n_kv_heads * head_dim, device=qkv.device, dtype=torch.float32)
    delta = torch.empty(n_heads, tp, device=qkv.device, dtype=torch.float32)
    _native.module().attn_bwd(
        qkv, out, dout.contiguous(), lse.contiguous(), pl["doc_start"], pl["doc_end"], pl["bwd"], n_heads,
        n_kv_heads, head_dim, 1.0 / math.sqrt(head_dim), dqkv, dq_acc, dkv_acc, delta,
        *(rope if rope is not None else (None, None, None)),
    )
    return dqkv[:t] if tp != t else dqkv


def _attn_backward_fixed_order(qkv, dout, doc_start, n_heads, n_kv_heads, head_dim, rope) -> torch.Tensor:
    """Deterministic-mode attention backward: per document, the fp32 causal attention is
    recomputed with PyTorch and differentiated, so no gradient is summed by reduce-adds
    whose order depends on scheduling (the native kernel reduce-adds dQ over key tiles
    and dK/dV over the query heads of a group).  Slow; for the deterministic mode only."""
    t, h, hk, d = qkv.shape[0], n_heads, n_kv_heads, head_dim
    q = qkv[:, : h * d].float().view(t, h, d)
    k = qkv[:, h * d : (h + hk) * d].float().view(t, hk, d)
    v = qkv[:, (h + hk) * d :].float().view(t, hk, d)
    do = dout.float().view(t, h, d)
    dq, dk, dv = torch.zeros_like(q), torch.zeros_like(k), torch.zeros_like(v)
    ds = doc_start.long()
    starts = (ds == torch.arange(t, device=ds.device)).nonzero().flatten().tolist() + [t]
    scale = 1.0 / math.sqrt(d)
    with torch.enable_grad():
        for a, b in zip(starts[:-1], starts[1:]):
            qd = q[a:b].transpose(0, 1).detach().requires_grad_()
            kd = k[a:b].transpose(0, 1).detach().requires_grad_()
            vd = v[a:b].transpose(0, 1).detach().requires_grad_()
            kr, vr = kd.repeat_interleave(h // hk, 0), vd.repeat_interleave(h // hk, 0)
            s = (qd @ kr.transpose(-1, -2)) * scale
            n = b - a
            s = s.masked_fill(torch.ones(n, n, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
            o = s.softmax(-1) @ vr
            gq, gk, gv = torch.autograd.grad(o, (qd, kd, vd), do[a:b].transpose(0, 1))
            dq[a:b], dk[a:b], dv[a:b] = gq.transpose(0, 1), gk.transpose(0, 1), gv.transpose(0, 1)
    if rope is not None:
        from packbalance_b200.ops.reference import rope_reference

        pos, cos, sin = rope
        c, sn = cos[pos.long()][:, None, :], sin[pos.long()][:, None, :]
        dq, dk = rope_reference(dq, c, -sn), rope_reference(dk, c, -sn)  # rotate back: R^T = R(-theta)
    return torch.cat([dq.reshape(t, h * d), dk.reshape(t, hk * d), dv.reshape(t, hk * d)], 1).to(qkv.dtype)


class _VarlenAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, doc_start):
        t, h, d = q.shape
        hk = k.shape[1]
        qkv = torch.cat([q.reshape(t, h * d), k.reshape(t, hk * d), v.reshape(t, hk * d)], dim=1)
        qkv = qkv.to(torch.bfloat16).contiguous()
        plan = attention_plan(doc_start, h, hk)
        o, lse = attn_forward_packed(qkv, plan, h, hk, d)
        ctx.save_for_backward(qkv, o, lse)
        ctx.plan, ctx.dims, ctx.dtype = plan, (t, h, hk, d), q.dtype
        return o.reshape(t, h, d).to(q.dtype)

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse = ctx.saved_tensors
        t, h, hk, d = ctx.dims
        dqkv = attn_backward_packed(qkv, o, do.reshape(t, h * d).to(torch.bfloat16), lse, ctx.plan, h, hk, d)
        dq = dqkv[:, : h * d].reshape(t, h, d).to(ctx.dtype)
        dk = dqkv[:, h * d : (h + hk) * d].reshape(t, hk, d).to(ctx.dtype)
        dv = dqkv[:, (h + hk) * d :].reshape(t, hk, d).to(ctx.dtype)
        return dq, dk, dv, None


def varlen_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, doc_start: torch.Tensor) -> torch.Tensor:
    """Token-major packed attention: q ``[T, H, D]``, k/v ``[T, Hkv, D]``."""
    if q.is_cuda:
        return _VarlenAttention.apply(q, k, v, doc_start)
    return varlen_attention_reference(q, k, v, doc_start)
