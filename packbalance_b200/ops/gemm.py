"""Python side of the tcgen05 GEMM: tile-width / split-K choice and the Linear
forward / dgrad / wgrad entry points.

Operand conventions (all bf16, unit inner stride, 16-byte aligned rows):

* ``linear_fwd(x[M,K], w[N,K])``      -> x @ w.T        (A K-major, B K-major)
* ``linear_dgrad(dy[M,N], w[N,K])``   -> dy @ w         (A K-major, B MN-major)
* ``linear_wgrad(dy[M,N], x[M,K])``   -> dy.T @ x, fp32 (A MN-major, B MN-major)
"""

from __future__ import annotations

import math

import torch

from packbalance_b200.ops import _native

EPI_BF16, EPI_F32, EPI_ADD_F32, EPI_SWIGLU, EPI_ROPE, EPI_SWIGLU_BWD = 0, 1, 2, 3, 4, 5
EPI_CE_FWD, EPI_CE_BWD = 7, 8

_SM_COUNT: dict[int, int] = {}


def sm_count(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SM_COUNT:
        _SM_COUNT[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SM_COUNT[idx]


# Relative tensor-pipe efficiency of a 128 x BN tile (narrow tiles reload the A tile
# more often per FLOP and issue more, smaller MMAs), measured on the bench shapes.
_TILE_EFF = {256: 1.0, 192: 0.9, 128: 0.75, 64: 0.45}


def pick_bn(m: int, n: int, sms: int, allowed=(256, 192, 128, 64)) -> int:
    """Tile width minimising waves x per-tile time, per-tile time ~ (BN + 64) / eff(BN)."""
    best, best_cost = allowed[0], math.inf
    m_tiles = -(-m // 128)
    for bn in allowed:
        tiles = m_tiles * -(-n // bn)
        cost = -(-tiles // sms) * (bn + 64) / _TILE_EFF[bn]
        if cost < best_cost - 1e-9:
            best, best_cost = bn, cost
    return best


def pick_tiling(m: int, n: int, k: int, sms: int, allowed=(256, 128, 64), max_splits: int = 8) -> tuple[int, int]:
    """(BN, split-K) minimising an estimate of the busiest SM's work: per work unit
    ``BN * (k / splits + 128)`` (the constant models the epilogue), times the number
    of waves.  Splits keep at least 4 k-blocks each.  (Checked against a sweep of the
    100M model's weight-gradient GEMMs on B200: the model's pick was the measured best
    for all four.)"""
    best, best_cost = (allowed[0], 1), math.inf
    m_tiles = -(-m // 128)
    k_blocks = -(-k // 64)
    for bn in allowed:
        tiles = m_tiles * -(-n // bn)
        for s in range(1, max_splits + 1):
            if s > 1 and k_blocks // s < 4:
                break
            cost = -(-(tiles * s) // sms) * bn * (k / s / _TILE_EFF[bn] + 128)
            if cost < best_cost - 1e-9:
                best, best_cost = (bn, s), cost
    return best


def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    out: torch.Tensor,
    m: int,
    n: int,
    k: int,
    *,
    a_mn: bool = False,
    b_mn: bool = False,
    epi: int = EPI_BF16,
    bn: int | None = None,
    splits: int = 1,
    max_ctas: int = 0,
    alpha: float = 1.0,
    aux=None,
    pos=None,
    cos=None,
    sin=None,
    head_dim: int = 0,
    n_rope_cols: int = 0,
    targets=None,
    pmax=None,
    psum=None,
    tlogit=None,
    lse=None,
    row_scale=None,
    z_coeff: float = 0.0,
    ag: list[int] | None = None,
) -> torch.Tensor:
    """Launch the tcgen05 GEMM ``D[m, n] = sum_k A(m, k) B(n, k)`` with epilogue ``epi``.

    ``ag``: fused all-gather of a sharded K-major B (13 ints, built by
    :meth:`packbalance_b200.parallel.sharded.ShardedParameters.gather_spec`): copy warps
    fetch the peer-owned rows of B into this GPU's gathered buffer during the GEMM.

    ``EPI_SWIGLU_BWD``: ``n`` = F, the accumulator is dh; ``aux`` holds the saved
    ``[g | u]`` (bf16 [m, 2F]) and ``out`` receives ``[dg | du]`` (bf16 [m, 2F])."""
    if bn is None:
        # 192-wide tiles only where they run on CTA pairs (K-major B); with an MN-major
        # B they fall back to single CTAs, measured slower than 256-wide pairs
        allowed = (256, 128, 64) if b_mn else (256, 192, 128, 64)
        if epi == EPI_ROPE:
            allowed = tuple(x for x in allowed if x % head_dim == 0)
        bn = pick_bn(m, n, sm_count(a.device), allowed)
    _native.module().gemm_tc(
        a, b, out, m, n, k, a_mn, b_mn, epi, bn, splits, max_ctas, alpha,
        aux, pos, cos, sin, head_dim, n_rope_cols, targets, pmax, psum, tlogit, lse, row_scale, z_coeff,
        ag or [],
    )
    return out


def linear_fwd(x: torch.Tensor, w: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    m, k = x.shape
    n = w.shape[0]
    out = torch.empty(m, n, device=x.device, dtype=out_dtype)
    return gemm(x, w, out, m, n, k, epi=EPI_BF16 if out_dtype == torch.bfloat16 else EPI_F32)


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    m, n = dy.shape
    k = w.shape[1]
    out = torch.empty(m, k, device=dy.device, dtype=out_dtype)
    return gemm(dy, w, out, m, k, n, b_mn=True, epi=EPI_BF16 if out_dtype == torch.bfloat16 else EPI_F32)


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    """``dy.T @ x`` in fp32 into ``out`` (overwritten, or added to when ``accumulate``);
    split-K with TMA reduce-add when the output grid alone cannot fill the GPU."""
    m, n = dy.shape
    k = x.shape[1]
    if out is None:
        out = torch.empty(n, k, device=dy.device, dtype=torch.float32)
    bn, splits = pick_tiling(n, k, m, sm_count(dy.device))
    if _native.deterministic():
        splits = 1  # one writer per output tile: no order-dependent reduce-adds
    if splits == 1 and not accumulate:
        return gemm(dy, x, out, n, k, m, a_mn=True, b_mn=True, epi=EPI_F32, bn=bn)
    if not accumulate:
        out.zero_()
    return gemm(dy, x, out, n, k, m, a_mn=True, b_mn=True, epi=EPI_ADD_F32, bn=bn, splits=splits)


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        wb = w.to(torch.bfloat16).contiguous()
        ctx.save_for_backward(x2, wb)
        ctx.shape, ctx.wdtype, ctx.xdtype = shape, w.dtype, x.dtype
        return linear_fwd(x2, wb).reshape(*shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, wb = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).to(torch.bfloat16).contiguous()
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = linear_dgrad(dy2, wb).reshape(ctx.shape).to(ctx.xdtype)
        if ctx.needs_input_grad[1]:
            dw = linear_wgrad(dy2, x2).to(ctx.wdtype)
        return dx, dw


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w.T`` with bf16 tensor-core math on CUDA (fp32 math on CPU)."""
    if not x.is_cuda:
        return torch.nn.functional.linear(x, w)
    return _Linear.apply(x, w)
