"""RMSNorm (reference ``kernels/rmsnorm.py``): native warp-per-row kernels on CUDA with
the weight gradient reduced in the same backward launch pair, torch math on CPU."""

from __future__ import annotations

import torch

from packbalance_b200.ops import _native
from packbalance_b200.ops.reference import rmsnorm_reference


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, eps):
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        y, rstd = _native.module().rmsnorm_fwd(x2, weight.float().contiguous(), float(eps), False)
        ctx.save_for_backward(x2, weight, rstd)
        return y.reshape(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, weight, rstd = ctx.saved_tensors
        dy2 = dy.reshape(x2.shape).contiguous()
        dw = torch.empty(x2.shape[-1], device=x2.device, dtype=torch.float32)
        dx = _native.module().rmsnorm_bwd(dy2, x2, weight.float().contiguous(), rstd, None, None, dw, False)
        return dx.to(dy.dtype).reshape(dy.shape), dw.to(weight.dtype), None


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    if x.is_cuda:
        return _RMSNorm.apply(x, weight, eps)
    return rmsnorm_reference(x, weight, eps)
