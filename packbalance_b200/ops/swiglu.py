"""SwiGLU ``silu(gate) * up`` on separate tensors (reference ``kernels/swiglu.py``).

The training fast path never calls this: SwiGLU runs in the gate|up GEMM epilogue and
its backward in the down-projection dgrad epilogue (``ops/gemm.py``)."""

from __future__ import annotations

import torch

from packbalance_b200.ops import _native
from packbalance_b200.ops.reference import swiglu_reference


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gate, up):
        g, u = gate.contiguous(), up.contiguous()
        ctx.save_for_backward(g, u)
        return _native.module().swiglu_fwd(g, u)

    @staticmethod
    def backward(ctx, dy):
        g, u = ctx.saved_tensors
        dg, du = _native.module().swiglu_bwd(g, u, dy.contiguous())
        return dg, du


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    if gate.is_cuda:
        return _SwiGLU.apply(gate, up)
    return swiglu_reference(gate, up)
