"""Native (sm_100a) forward/backward of :class:`LlamaForCausalLM`.

Three autograd nodes per step instead of a graph of small ops:

* ``_Embed``    fp32 gather of the embedding rows; backward scatter-adds into the
                embedding gradient (which the tied LM head wrote first).
* ``_Decoder``  one whole pre-norm decoder layer per node.  Forward launches:
                RMSNorm -> QKV GEMM (+RoPE epilogue) -> varlen attention ->
                O-proj GEMM (+residual epilogue) -> RMSNorm -> gate|up GEMM
                (+SwiGLU epilogue) -> down GEMM (+residual epilogue).
                Backward: down dgrad (+SwiGLU-backward epilogue) and wgrad,
                gate|up dgrad / wgrad, RMSNorm backward (+residual gradient), O-proj
                dgrad / wgrad, attention backward, inverse RoPE, QKV dgrad / wgrad,
                RMSNorm backward.  Weight gradients go straight into the flat fp32
                gradient buffer; the layer then tells the data-parallel engine its
                gradients are final so their all-reduce can start.
* ``_Head``     final RMSNorm + fused LM-head cross-entropy (summed loss).

The residual stream is fp32 (as under the reference's autocast); GEMM operands are
bf16 (activations rounded once at their producer, weights from the bf16 shadow).
"""

from __future__ import annotations

import math

import torch

from packbalance_b200.models.llama import CausalLMOutput
from packbalance_b200.ops import _native
from packbalance_b200.ops.attention import attention_plan, attn_backward_packed, attn_forward_packed
from packbalance_b200.ops.cross_entropy import lmhead_ce_backward, lmhead_ce_forward
from packbalance_b200.ops.gemm import (
    EPI_BF16,
    EPI_F32,
    EPI_RESID,
    EPI_ROPE,
    EPI_SWIGLU,
    EPI_SWIGLU_BWD,
    gemm,
)
from packbalance_b200.ops.rope import rope_inplace
from packbalance_b200.parallel.flat import FlatParameters


class StepContext:
    """Per-forward data shared by the layer nodes (positions, attention plan, and a
    side channel carrying the bf16 copy of each residual gradient)."""

    def __init__(self, model, flat: FlatParameters, pos: torch.Tensor, plan: dict) -> None:
        self.model = model
        self.cfg = model.cfg
        self.flat = flat
        self.pos = pos
        self.plan = plan
        rot = model.model.rotary
        self.cos = rot.cos_cached
        self.sin = rot.sin_cached
        self._bf16_of: tuple[torch.Tensor, torch.Tensor] | None = None

    def stash_bf16(self, g32: torch.Tensor, g16: torch.Tensor) -> None:
        self._bf16_of = (g32, g16)

    def bf16_of(self, g32: torch.Tensor) -> torch.Tensor:
        if self._bf16_of is not None and self._bf16_of[0] is g32:
            return self._bf16_of[1]
        return g32.to(torch.bfloat16)


def _write_grad(flat: FlatParameters, params, fn) -> None:
    """Call ``fn(grad_view, accumulate)`` for a group of adjacent params."""
    acc = flat.claim(*params)
    fn(flat.grad_of(*params), acc)


class _Embed(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight, sc: StepContext):
        ctx.sc = sc
        ctx.ids = ids
        ctx.weight = weight
        return _native.module().embedding_fwd(ids, weight)

    @staticmethod
    def backward(ctx, dx):
        sc = ctx.sc
        flat = sc.flat
        w = ctx.weight
        acc = flat.claim(w)
        _native.module().embedding_bwd(ctx.ids, dx.contiguous(), flat.grad_of(w), acc)
        flat.ready(flat.slot(w).offset)
        return None, None, None


class _Decoder(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w_in, wq, wk, wv, wo, w_post, wg, wu, wd, sc: StepContext):
        cfg = sc.cfg
        flat = sc.flat
        t, d = x.shape
        h, hk, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        nqkv = (h + 2 * hk) * hd
        F = cfg.d_ff
        C = _native.module()
        xn1, rstd1 = C.rmsnorm_fwd(x, w_in, cfg.norm_eps, True)
        qkv = torch.empty(t, nqkv, device=x.device, dtype=torch.bfloat16)
        gemm(xn1, flat.shadow_of(wq, wk, wv), qkv, t, nqkv, d, epi=EPI_ROPE, pos=sc.pos, cos=sc.cos, sin=sc.sin,
             head_dim=hd, n_rope_cols=(h + hk) * hd)
        o, lse = attn_forward_packed(qkv, sc.plan, h, hk, hd)
        x1 = torch.empty_like(x)
        gemm(o, flat.shadow_of(wo), x1, t, d, h * hd, epi=EPI_RESID, res=x)
        xn2, rstd2 = C.rmsnorm_fwd(x1, w_post, cfg.norm_eps, True)
        hmid = torch.empty(t, F, device=x.device, dtype=torch.bfloat16)
        gu = torch.empty(t, 2 * F, device=x.device, dtype=torch.bfloat16)
        gemm(xn2, flat.shadow_of(wg, wu), hmid, t, 2 * F, d, epi=EPI_SWIGLU, aux=gu)
        x2 = torch.empty_like(x)
        gemm(hmid, flat.shadow_of(wd), x2, t, d, F, epi=EPI_RESID, res=x1)
        ctx.sc = sc
        ctx.params = (w_in, wq, wk, wv, wo, w_post, wg, wu, wd)
        ctx.saved = (x, xn1, rstd1, qkv, o, lse, x1, xn2, rstd2, gu, hmid)
        return x2

    @staticmethod
    def backward(ctx, dx2):
        sc = ctx.sc
        cfg = sc.cfg
        flat = sc.flat
        C = _native.module()
        w_in, wq, wk, wv, wo, w_post, wg, wu, wd = ctx.params
        x, xn1, rstd1, qkv, o, lse, x1, xn2, rstd2, gu, hmid = ctx.saved
        ctx.saved = None
        t, d = x.shape
        h, hk, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        nqkv = (h + 2 * hk) * hd
        F = cfg.d_ff
        dx2 = dx2.contiguous()
        dx2b = sc.bf16_of(dx2)
        # MLP: dh -> (SwiGLU backward epilogue) -> dg|du
        dgu = torch.empty(t, 2 * F, device=x.device, dtype=torch.bfloat16)
        gemm(dx2b, flat.shadow_of(wd), dgu, t, F, d, b_mn=True, epi=EPI_SWIGLU_BWD, aux=gu, aux2=dgu)
        _write_grad(flat, (wd,), lambda g, acc: gemm(dx2b, hmid, g, d, F, t, a_mn=True, b_mn=True, epi=EPI_F32, beta=acc))
        dxn2 = torch.empty(t, d, device=x.device, dtype=torch.float32)
        gemm(dgu, flat.shadow_of(wg, wu), dxn2, t, d, 2 * F, b_mn=True, epi=EPI_F32)
        _write_grad(
            flat, (wg, wu), lambda g, acc: gemm(dgu, xn2, g, 2 * F, d, t, a_mn=True, b_mn=True, epi=EPI_F32, beta=acc)
        )
        dx1b = torch.empty(t, d, device=x.device, dtype=torch.bfloat16)
        acc = flat.claim(w_post)
        dx1 = C.rmsnorm_bwd(dxn2, x1, w_post, rstd2, dx2, dx1b, flat.grad_of(w_post).view(-1), acc)
        # attention
        do = torch.empty(t, h * hd, device=x.device, dtype=torch.bfloat16)
        gemm(dx1b, flat.shadow_of(wo), do, t, h * hd, d, b_mn=True, epi=EPI_BF16)
        _write_grad(flat, (wo,), lambda g, acc: gemm(dx1b, o, g, d, h * hd, t, a_mn=True, b_mn=True, epi=EPI_F32, beta=acc))
        dqkv = attn_backward_packed(qkv, o, do, lse, sc.plan, h, hk, hd)
        rope_inplace(dqkv, sc.pos, sc.cos, sc.sin, (h + hk) * hd, hd, inverse=True)
        dxn1 = torch.empty(t, d, device=x.device, dtype=torch.float32)
        gemm(dqkv, flat.shadow_of(wq, wk, wv), dxn1, t, d, nqkv, b_mn=True, epi=EPI_F32)
        _write_grad(
            flat, (wq, wk, wv), lambda g, acc: gemm(dqkv, xn1, g, nqkv, d, t, a_mn=True, b_mn=True, epi=EPI_F32, beta=acc)
        )
        dxb = torch.empty(t, d, device=x.device, dtype=torch.bfloat16)
        acc = flat.claim(w_in)
        dx = C.rmsnorm_bwd(dxn1, x, w_in, rstd1, dx1, dxb, flat.grad_of(w_in).view(-1), acc)
        sc.stash_bf16(dx, dxb)
        flat.ready(flat.slot(w_in).offset)
        return (dx,) + (None,) * 10


class _Head(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w_norm, w_lm, labels, sc: StepContext):
        cfg = sc.cfg
        C = _native.module()
        xf, rstd = C.rmsnorm_fwd(x, w_norm, cfg.norm_eps, True)
        loss, lse = lmhead_ce_forward(xf, sc.flat.shadow_of(w_lm), labels, -100, cfg.z_loss_coeff)
        ctx.sc = sc
        ctx.saved = (x, xf, rstd, lse, labels)
        ctx.params = (w_norm, w_lm)
        return loss

    @staticmethod
    def backward(ctx, grad):
        sc = ctx.sc
        cfg = sc.cfg
        flat = sc.flat
        x, xf, rstd, lse, labels = ctx.saved
        ctx.saved = None
        w_norm, w_lm = ctx.params
        acc = flat.claim(w_lm)
        dxf = lmhead_ce_backward(
            xf, flat.shadow_of(w_lm), labels, lse, grad, flat.grad_of(w_lm), acc, -100, cfg.z_loss_coeff
        )
        dxb = torch.empty(x.shape, device=x.device, dtype=torch.bfloat16)
        acc = flat.claim(w_norm)
        dx = _native.module().rmsnorm_bwd(dxf, x, w_norm, rstd, None, dxb, flat.grad_of(w_norm).view(-1), acc)
        sc.stash_bf16(dx, dxb)
        flat.ready(min(flat.slot(w_norm).offset, flat.slot(w_lm).offset) if sc.model.lm_head is not None
                   else flat.slot(w_norm).offset)
        return dx, None, None, None, None


def _ensure_flat(model) -> FlatParameters:
    if model.flat is None:
        model.flat = FlatParameters(model)
    model.flat.refresh_shadow()
    return model.flat


def fused_causal_lm_forward(model, input_ids, labels, position_ids, doc_start) -> CausalLMOutput:
    cfg = model.cfg
    flat = _ensure_flat(model)
    ids = input_ids.reshape(-1).contiguous()
    pos = position_ids.reshape(-1)
    model.model.rotary.check_positions(pos) if not torch.cuda.is_current_stream_capturing() else None
    pos32 = pos.to(torch.int32).contiguous()
    doc_start = doc_start.reshape(-1).to(device=ids.device, dtype=torch.int32).contiguous()
    plan = attention_plan(doc_start, cfg.n_heads, cfg.n_kv_heads)
    sc = StepContext(model, flat, pos32, plan)
    m = model.model
    x = _Embed.apply(ids, m.embed_tokens.weight, sc)
    for layer in m.layers:
        a, mlp = layer.self_attn, layer.mlp
        x = _Decoder.apply(
            x, layer.input_layernorm.weight, a.q_proj.weight, a.k_proj.weight, a.v_proj.weight, a.o_proj.weight,
            layer.post_attention_layernorm.weight, mlp.gate_proj.weight, mlp.up_proj.weight, mlp.down_proj.weight, sc,
        )
    shape = input_ids.shape
    if labels is not None:
        loss = _Head.apply(x, m.norm.weight, model.lm_head_weight, labels.reshape(-1).contiguous(), sc)
        return CausalLMOutput(loss=loss, hidden_states=None)
    xf, _ = _native.module().rmsnorm_fwd(x, m.norm.weight, cfg.norm_eps, True)
    w = flat.shadow_of(model.lm_head_weight)
    logits = torch.empty(xf.shape[0], cfg.vocab_size, device=xf.device, dtype=torch.bfloat16)
    gemm(xf, w, logits, xf.shape[0], cfg.vocab_size, cfg.d_model, epi=EPI_BF16)
    return CausalLMOutput(
        logits=logits.float().reshape(*shape, cfg.vocab_size), hidden_states=xf.float().reshape(*shape, cfg.d_model)
    )


__all__ = ["fused_causal_lm_forward", "StepContext", "math"]
