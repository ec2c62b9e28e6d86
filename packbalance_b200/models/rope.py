"""Rotary position embeddings with per-document position ids.

Half-split (not interleaved) rotation, fp32 cos/sin tables up to ``max_seq_len``
held in non-persistent buffers, as in the reference (``model/rope.py:9-42``).  The
same tables feed the native QKV-GEMM RoPE epilogue.
"""

from __future__ import annotations

import torch
from torch import nn

from packbalance_b200.ops.reference import rope_reference


def rope_tables(head_dim: int, max_seq_len: int, theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    angles = torch.outer(torch.arange(max_seq_len, dtype=torch.float32), inv_freq)
    return angles.cos(), angles.sin()


class RotaryEmbedding(nn.Module):
    def __init__(self, head_dim: int, max_seq_len: int, theta: float = 10000.0) -> None:
        super().__init__()
        if head_dim % 2:
            raise ValueError("RoPE requires an even head_dim")
        cos, sin = rope_tables(head_dim, max_seq_len, theta)
        self.register_buffer("cos_cached", cos, persistent=False)
        self.register_buffer("sin_cached", sin, persistent=False)

    def check_positions(self, position_ids: torch.Tensor) -> None:
        if position_ids.numel() and int(position_ids.max()) >= self.cos_cached.shape[0]:
            raise ValueError(
                f"position id {int(position_ids.max())} exceeds RoPE cache ({self.cos_cached.shape[0]})"
            )

    def forward(self, position_ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        self.check_positions(position_ids)
        return self.cos_cached[position_ids], self.sin_cached[position_ids]


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


def apply_rotary_pos_emb(
    q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor]:
    """q/k ``[B, H, S, D]``; cos/sin ``[B, S, D/2]`` (gathered by position)."""
    c = cos.unsqueeze(1)
    s = sin.unsqueeze(1)
    return rope_reference(q, c, s), rope_reference(k, c, s)
