"""In-place RoPE on a packed ``[T, heads * head_dim]`` buffer (forward or inverse).

The training forward applies RoPE inside the QKV GEMM epilogue; this kernel applies
the inverse rotation to dQ / dK after the attention backward."""

from __future__ import annotations

import torch

from packbalance_b200.ops import _native
from packbalance_b200.ops.reference import rope_reference


def rope_inplace(
    x: torch.Tensor, pos: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, n_rope_cols: int, head_dim: int,
    inverse: bool = False,
) -> torch.Tensor:
    if x.is_cuda:
        _native.module().rope_apply(x, pos.to(torch.int32), cos, sin, n_rope_cols, head_dim, inverse)
        return x
    heads = n_rope_cols // head_dim
    view = x[:, :n_rope_cols].reshape(x.shape[0], heads, head_dim)
    c = cos[pos.long()].unsqueeze(1)
    s = sin[pos.long()].unsqueeze(1)
    view.copy_(rope_reference(view, c, -s if inverse else s))
    return x
