"""Plain PyTorch versions of every op: the CPU execution path and the fp32 oracle
that the native kernels are tested against (reference ``kernels/reference.py``)."""

from __future__ import annotations

import torch
import torch.nn.functional as F


def rmsnorm_reference(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    inv = torch.rsqrt(xf.square().mean(dim=-1, keepdim=True) + eps)
    return (xf * inv * weight.float()).to(x.dtype)


def swiglu_reference(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return F.silu(gate) * up


def rope_reference(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Half-split rotation of the last dim; ``cos``/``sin`` broadcast as [..., D/2]."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    c = cos.to(x.dtype)
    s = sin.to(x.dtype)
    return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s), dim=-1)


def chunked_linear_cross_entropy(
    x: torch.Tensor,
    weight: torch.Tensor,
    targets: torch.Tensor,
    *,
    chunk_size: int = 1024,
    ignore_index: int = -100,
    z_loss_coeff: float = 0.0,
) -> torch.Tensor:
    """Summed token cross-entropy of ``x @ weight.T`` without full [T, V] logits.

    Each row chunk is an ordinary autograd graph.  With ``z_loss_coeff`` the loss adds
    ``z * logsumexp**2`` per labelled token.
    """
    x2 = x.reshape(-1, x.shape[-1])
    t1 = targets.reshape(-1)
    if x2.shape[0] != t1.shape[0]:
        raise ValueError(f"x has {x2.shape[0]} rows but targets has {t1.shape[0]}")
    total = x2.new_zeros(())
    for lo in range(0, x2.shape[0], chunk_size):
        logits = x2[lo : lo + chunk_size] @ weight.t()
        y = t1[lo : lo + chunk_size]
        total = total + F.cross_entropy(logits, y, ignore_index=ignore_index, reduction="sum")
        if z_loss_coeff:
            lse = torch.logsumexp(logits.float(), dim=-1)
            total = total + z_loss_coeff * lse[y != ignore_index].square().sum()
    return total


def eager_attention(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, doc_ids: torch.Tensor
) -> torch.Tensor:
    """Exact packed attention, one causal SDPA per document ([B, H, S, D] layout).

    Tokens with a negative document id (padding) get zero output.
    """
    n_heads, n_kv = q.shape[1], k.shape[1]
    if n_kv != n_heads:
        k = k.repeat_interleave(n_heads // n_kv, dim=1)
        v = v.repeat_interleave(n_heads // n_kv, dim=1)
    out = torch.zeros_like(q)
    for b in range(q.shape[0]):
        ids = doc_ids[b]
        for doc in torch.unique(ids).tolist():
            if doc < 0:
                continue
            idx = (ids == doc).nonzero(as_tuple=True)[0]
            out[b : b + 1, :, idx] = F.scaled_dot_product_attention(
                q[b : b + 1, :, idx], k[b : b + 1, :, idx], v[b : b + 1, :, idx], is_causal=True
            )
    return out


def varlen_attention_reference(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, doc_start: torch.Tensor
) -> torch.Tensor:
    """Token-major packed attention: q [T, H, D], k/v [T, Hkv, D]; token ``i`` attends
    to ``j`` iff ``doc_start[i] <= j <= i``.  Computed in fp32 with a dense mask."""
    t, h, d = q.shape
    group = h // k.shape[1]
    kk = k.float().repeat_interleave(group, dim=1)
    vv = v.float().repeat_interleave(group, dim=1)
    pos = torch.arange(t, device=q.device)
    allowed = (pos[None, :] <= pos[:, None]) & (pos[None, :] >= doc_start.long()[:, None])
    scores = torch.einsum("qhd,khd->hqk", q.float(), kk) / d**0.5
    scores = scores.masked_fill(~allowed[None], float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    return torch.einsum("hqk,khd->qhd", probs, vv).to(q.dtype)
