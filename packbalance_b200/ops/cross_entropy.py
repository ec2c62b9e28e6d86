"""LM head + cross-entropy without materialising the full ``[T, V]`` logits.

Reference: ``kernels/fused_ce.py`` (cuBLAS chunk GEMM + Triton online-LSE kernel,
fp32 backward GEMMs).  Here:

* forward: ONE tcgen05 GEMM ``x @ W.T`` whose epilogue reduces each 128 x 256 logits
  tile to per-row (max, sum exp) partials and picks the target logit; a small row
  kernel combines the partials into ``lse`` and the summed loss
  ``lse - logit[target] + z * lse**2`` (labelled rows only).  No logits reach HBM.
* backward, per chunk of rows: a GEMM recomputes the logits and its epilogue writes
  ``dlogits = (softmax * (1 + 2 z lse) - onehot) * dloss`` in bf16 (the only
  materialised chunk), then two GEMMs give ``dx = dlogits @ W`` and
  ``dW (+)= dlogits.T @ x`` with fp32 accumulation.
* optionally (``logits_out`` in the forward, ``logits`` in the backward), the forward
  GEMM also stores the bf16 logits (its statistics are then taken from the rounded
  values) and the backward turns them into dlogits in place with one elementwise pass
  instead of recomputing them: T x V x 2 bytes of HBM for one GEMM of 2 T d V FLOPs,
  the trade the training step makes when the logits are small (the reference's own
  bf16 path also takes the softmax of bf16 logits).

The loss is the *sum* over labelled tokens, like the reference.  CPU tensors run the
chunked PyTorch reference.
"""

from __future__ import annotations

import torch

from packbalance_b200.ops import _native
from packbalance_b200.ops.gemm import EPI_ADD_F32, EPI_CE_BWD, EPI_CE_FWD, EPI_F32, gemm, linear_wgrad, pick_tiling, sm_count
from packbalance_b200.ops.reference import chunked_linear_cross_entropy

CE_TILE = 256
DLOGIT_CHUNK_BYTES = 256 * 1024 * 1024


def lmhead_ce_forward(
    x: torch.Tensor,
    w: torch.Tensor,
    targets: torch.Tensor,
    ignore_index: int = -100,
    z_coeff: float = 0.0,
    ag: list[int] | None = None,
    logits_out: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (summed loss, lse[T]).  ``x`` [T, d] bf16, ``w`` [V, d] bf16.  ``ag``: the
    sharded LM head is fetched inside the GEMM (see :func:`~packbalance_b200.ops.gemm.gemm`).
    ``logits_out`` (bf16 [T, V]): also keep the logits, for :func:`lmhead_ce_backward`."""
    t, d = x.shape
    v = w.shape[0]
    nt = -(-v // CE_TILE)
    pmax = torch.empty(nt, t, device=x.device, dtype=torch.float32)
    psum = torch.empty(nt, t, device=x.device, dtype=torch.float32)
    # written by the one logits tile that holds each row's target column; read only for
    # labelled rows, so it needs no zero fill
    tlogit = torch.empty(t, device=x.device, dtype=torch.float32)
    lse = torch.empty(t, device=x.device, dtype=torch.float32)
    loss = torch.zeros((), device=x.device, dtype=torch.float32)
    tgt = targets.reshape(-1).to(torch.int64).contiguous()
    gemm(x, w, pmax, t, v, d, epi=EPI_CE_FWD, bn=CE_TILE, targets=tgt, pmax=pmax, psum=psum, tlogit=tlogit, ag=ag,
         aux=logits_out)
    _native.module().ce_finalize(pmax, psum, tlogit, tgt, ignore_index, float(z_coeff), lse, loss)
    return loss, lse


def lmhead_ce_backward(
    x: torch.Tensor,
    w: torch.Tensor,
    targets: torch.Tensor,
    lse: torch.Tensor,
    grad_loss: torch.Tensor,
    dw_out: torch.Tensor,
    accumulate_dw: bool,
    ignore_index: int = -100,
    z_coeff: float = 0.0,
    chunk_rows: int | None = None,
    logits: torch.Tensor | None = None,
) -> torch.Tensor:
    """Returns dx [T, d] fp32; writes (or adds) dW into ``dw_out`` [V, d] fp32.
    ``logits``: the forward's kept bf16 logits (overwritten with dlogits)."""
    t, d = x.shape
    v = w.shape[0]
    tgt = targets.reshape(-1).to(torch.int64).contiguous()
    scale = torch.empty(t, device=x.device, dtype=torch.float32)
    _native.module().ce_row_scale(tgt, ignore_index, grad_loss.reshape(()).float().contiguous(), scale)
    sms = sm_count(x.device)
    if logits is not None:
        _native.module().ce_dlogits(logits, lse, tgt, scale, float(z_coeff))
        dx = torch.empty(t, d, device=x.device, dtype=torch.float32)
        bn, splits = pick_tiling(t, d, v, sms)
        if _native.deterministic():
            splits = 1
        if splits > 1:
            dx.zero_()
            gemm(logits, w, dx, t, d, v, b_mn=True, epi=EPI_ADD_F32, bn=bn, splits=splits)
        else:
            gemm(logits, w, dx, t, d, v, b_mn=True, epi=EPI_F32, bn=bn)
        linear_wgrad(logits, x, dw_out, accumulate=accumulate_dw)
        return dx
    if chunk_rows is None:
        chunk_rows = max(128, (DLOGIT_CHUNK_BYTES // (2 * v)) // 128 * 128)
    chunk_rows = min(chunk_rows, t)
    dx = torch.empty(t, d, device=x.device, dtype=torch.float32)
    dlog = torch.empty(chunk_rows, v, device=x.device, dtype=torch.bfloat16)
    for i, r0 in enumerate(range(0, t, chunk_rows)):
        r1 = min(t, r0 + chunk_rows)
        rows = r1 - r0
        dl = dlog[:rows]
        gemm(x[r0:r1], w, dl, rows, v, d, epi=EPI_CE_BWD, bn=CE_TILE, targets=tgt[r0:r1], lse=lse[r0:r1],
             row_scale=scale[r0:r1], z_coeff=z_coeff)
        bn, splits = pick_tiling(rows, d, v, sms)
        if _native.deterministic():
            splits = 1
        if splits > 1:
            dx[r0:r1].zero_()
            gemm(dl, w, dx[r0:r1], rows, d, v, b_mn=True, epi=EPI_ADD_F32, bn=bn, splits=splits)
        else:
            gemm(dl, w, dx[r0:r1], rows, d, v, b_mn=True, epi=EPI_F32, bn=bn)
        linear_wgrad(dl, x[r0:r1], dw_out, accumulate=accumulate_dw or i > 0)
    return dx


class _FusedLinearCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, targets, chunk_size, ignore_index, z_coeff):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
        wb = weight.to(torch.bfloat16).contiguous()
        loss, lse = lmhead_ce_forward(x2, wb, targets, ignore_index, z_coeff)
        ctx.save_for_backward(x2, wb, targets, lse)
        ctx.meta = (shape, x.dtype, weight.dtype, chunk_size, ignore_index, z_coeff)
        return loss

    @staticmethod
    def backward(ctx, grad):
        x2, wb, targets, lse = ctx.saved_tensors
        shape, xdt, wdt, chunk, ignore_index, z = ctx.meta
        dw = torch.empty(wb.shape, device=wb.device, dtype=torch.float32)
        dx = lmhead_ce_backward(x2, wb, targets, lse, grad, dw, False, ignore_index, z)
        return dx.reshape(shape).to(xdt), dw.to(wdt), None, None, None, None


def linear_cross_entropy(
    x: torch.Tensor,
    weight: torch.Tensor,
    targets: torch.Tensor,
    *,
    chunk_size: int = 1024,
    ignore_index: int = -100,
    z_loss_coeff: float = 0.0,
) -> torch.Tensor:
    """Summed CE of ``x @ weight.T`` against ``targets`` (reference signature)."""
    if x.is_cuda:
        return _FusedLinearCE.apply(x, weight, targets, chunk_size, ignore_index, z_loss_coeff)
    return chunked_linear_cross_entropy(
        x, weight, targets, chunk_size=chunk_size, ignore_index=ignore_index, z_loss_coeff=z_loss_coeff
    )
