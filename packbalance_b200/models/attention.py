"""Document-masked attention over packed sequences.

The reference builds a FlexAttention ``BlockMask`` per microbatch
(``model/attention.py:25-54``, 7.6 % of its step time).  Here the mask is implicit:
each token carries ``doc_start`` (first token of its document) and token ``q``
attends to ``k`` iff ``doc_start[q] <= k <= q``.  The native sm100 kernel reads
``doc_start`` directly and skips key tiles outside the document; the eager
per-document SDPA loop stays as the CPU path and the oracle.
"""

from __future__ import annotations

import torch

from packbalance_b200.ops.reference import eager_attention

__all__ = ["build_doc_block_mask", "doc_start_from_doc_ids", "eager_attention", "attention_forward"]


def doc_start_from_doc_ids(doc_ids: torch.Tensor) -> torch.Tensor:
    """``doc_start`` (int32) for a 1-D or ``[B, S]`` doc-id tensor, flattened to one
    token stream; rows of a ``[B, S]`` input never share a document."""
    ids = doc_ids.reshape(doc_ids.shape[0], -1) if doc_ids.dim() == 2 else doc_ids.reshape(1, -1)
    rows, s = ids.shape
    pos = torch.arange(s, device=ids.device).expand(rows, s)
    new_run = torch.ones_like(ids, dtype=torch.bool)
    new_run[:, 1:] = ids[:, 1:] != ids[:, :-1]
    starts = torch.where(new_run, pos, torch.zeros_like(pos))
    starts = torch.cummax(starts, dim=1).values
    starts = starts + torch.arange(rows, device=ids.device)[:, None] * s
    return starts.reshape(-1).to(torch.int32)


def build_doc_block_mask(doc_ids: torch.Tensor, n_heads: int = 0, block_size: int = 128) -> torch.Tensor:
    """API-compatible stand-in for the reference's block-mask builder.

    Returns the ``doc_start`` vector that the sm100 kernel consumes; ``n_heads`` and
    ``block_size`` are accepted for signature compatibility.
    """
    return doc_start_from_doc_ids(doc_ids)


def attention_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    doc_ids: torch.Tensor,
    *,
    block_mask=None,
    backend: str = "auto",
    compile_attention: bool = True,
) -> torch.Tensor:
    """Packed attention in ``[B, H, S, D]`` layout (reference signature).

    CUDA tensors with backend ``auto``/``flex``/``sm100`` run the native varlen
    kernel; everything else runs the eager oracle.
    """
    if backend not in ("auto", "flex", "eager", "sm100"):
        raise ValueError(f"unknown attention backend {backend}")
    if backend == "eager" or not q.is_cuda:
        return eager_attention(q, k, v, doc_ids)
    from packbalance_b200.ops.attention import varlen_attention

    b, h, s, d = q.shape
    doc_start = block_mask if isinstance(block_mask, torch.Tensor) else doc_start_from_doc_ids(doc_ids)
    qt = q.transpose(1, 2).reshape(b * s, h, d)
    kt = k.transpose(1, 2).reshape(b * s, k.shape[1], d)
    vt = v.transpose(1, 2).reshape(b * s, v.shape[1], d)
    out = varlen_attention(qt, kt, vt, doc_start.to(q.device))
    out = out.reshape(b, s, h, d).transpose(1, 2)
    valid = (doc_ids.reshape(b, 1, s, 1) >= 0).to(out.dtype)
    return out * valid
