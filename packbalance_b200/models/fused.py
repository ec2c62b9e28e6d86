"""Native (sm_100a) forward/backward of :class:`LlamaForCausalLM`.

Autograd nodes per step instead of a graph of small ops:

* ``_Embed``    fp32 gather of the embedding rows; backward scatter-adds into the
                embedding gradient (which the tied LM head wrote first).
* ``_Decoder``  one whole pre-norm decoder layer.  The residual stream is carried
                between layers as a pair ``(x, delta)`` with ``x`` fp32 and ``delta``
                the bf16 output of the last projection; the sum ``x + delta`` is formed
                inside the next fused add+RMSNorm kernel, so no GEMM epilogue reads the
                residual.  Forward launches: add+RMSNorm -> QKV GEMM (+RoPE epilogue)
                -> varlen attention -> O-proj GEMM -> add+RMSNorm -> gate|up GEMM
                (+SwiGLU epilogue) -> down GEMM.  Backward: down dgrad, SwiGLU
                backward, gate|up dgrad, RMSNorm backward (+residual gradient), O-proj
                dgrad, attention backward (+inverse RoPE), QKV dgrad, RMSNorm backward;
                the weight-gradient GEMMs (split-K, fp32) write straight into the flat
                gradient buffer, after which the layer tells the data-parallel engine
                that its gradients are final.
* ``_Head``     final add+RMSNorm + fused LM-head cross-entropy (summed loss).

The gradient of ``x + delta`` reaches a layer twice, as the fp32 gradient of ``x``
and as the bf16 gradient of ``delta``: the bf16 copy is produced by the RMSNorm
backward kernel and feeds the bf16 GEMMs directly.
"""

from __future__ import annotations

import torch

from packbalance_b200.models.llama import CausalLMOutput
from packbalance_b200.ops import _native
from packbalance_b200.ops.attention import attention_plan, attn_backward_packed, attn_forward_packed
from packbalance_b200.ops.cross_entropy import lmhead_ce_backward, lmhead_ce_forward
from packbalance_b200.ops.gemm import EPI_BF16, EPI_F32, EPI_ROPE, EPI_SWIGLU, EPI_SWIGLU_BWD, gemm, linear_wgrad
from packbalance_b200.parallel.flat import FlatParameters


class StepContext:
    """Per-forward data shared by the layer nodes (positions, attention plan, RoPE tables)."""

    def __init__(self, model, flat: FlatParameters, pos: torch.Tensor, plan: dict) -> None:
        self.model = model
        self.cfg = model.cfg
        self.flat = flat
        self.pos = pos
        self.plan = plan
        rot = model.model.rotary
        self.cos = rot.cos_cached
        self.sin = rot.sin_cached
        # reference flag (model/llama.py:153-163): recompute each layer in its backward
        self.checkpoint = bool(model.model.gradient_checkpointing and model.training)


_WGRAD_STREAMS: dict[int, torch.cuda.Stream] = {}
# Weight gradients go to a side stream only while a CUDA graph is being captured: in a
# graph the fork/join costs nothing at run time; eagerly, the host-side stream and
# allocator bookkeeping per GEMM costs more than the overlap gains.
ASYNC_WGRAD = False


def _dev_index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def _wgrad_stream(device: torch.device) -> torch.cuda.Stream | None:
    if device.type != "cuda":
        return None
    idx = _dev_index(device)
    if idx not in _WGRAD_STREAMS:
        _WGRAD_STREAMS[idx] = torch.cuda.Stream(device=idx)
    return _WGRAD_STREAMS[idx]


def _wgrad(flat: FlatParameters, params, dy: torch.Tensor, x: torch.Tensor) -> None:
    """Weight gradient ``dy.T @ x`` of a group of adjacent params into the flat buffer,
    on a side stream: the weight gradients of a layer depend on nothing the rest of the
    backward pass computes, so they fill the SMs the dgrad / attention kernels leave idle
    (wave tails).  The layer joins the side stream before it reports its gradients."""
    acc = flat.claim(*params)
    ws = _wgrad_stream(dy.device) if ASYNC_WGRAD else None
    if ws is None:
        linear_wgrad(dy, x, flat.grad_of(*params), accumulate=acc)
        return
    ws.wait_stream(torch.cuda.current_stream(dy.device))
    with torch.cuda.stream(ws):
        linear_wgrad(dy, x, flat.grad_of(*params), accumulate=acc)
    dy.record_stream(ws)
    x.record_stream(ws)


def _join_wgrads(device: torch.device) -> None:
    ws = _WGRAD_STREAMS.get(_dev_index(device)) if ASYNC_WGRAD and device.type == "cuda" else None
    if ws is not None:
        torch.cuda.current_stream(device).wait_stream(ws)


class _Embed(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight, sc: StepContext):
        ctx.sc = sc
        ctx.ids = ids
        ctx.weight = weight
        return sc.flat.embedding(ids, weight)

    @staticmethod
    def backward(ctx, dx):
        flat = ctx.sc.flat
        w = ctx.weight
        acc = flat.claim(w)
        _native.module().embedding_bwd(ctx.ids, dx.contiguous(), flat.grad_of(w), acc)
        flat.ready_after(w)
        return None, None, None


def _layer_forward(x_prev, delta_prev, params, sc: StepContext):
    """One decoder layer forward; returns (x1, mlp_out, saved activations)."""
    w_in, wq, wk, wv, wo, w_post, wg, wu, wd = params
    cfg = sc.cfg
    flat = sc.flat
    C = _native.module()
    t, d = x_prev.shape
    h, hk, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    nqkv = (h + 2 * hk) * hd
    F = cfg.d_ff
    x, xn1, rstd1 = C.add_rmsnorm_fwd(x_prev, delta_prev, w_in, cfg.norm_eps, True)
    qkv = torch.empty(t, nqkv, device=x.device, dtype=torch.bfloat16)
    ag = flat.gather_spec(wq, wk, wv)  # sharded weights: fetched inside this GEMM
    gemm(xn1, flat.shadow_of(wq, wk, wv), qkv, t, nqkv, d, epi=EPI_ROPE, pos=sc.pos, cos=sc.cos, sin=sc.sin,
         head_dim=hd, n_rope_cols=(h + hk) * hd, ag=ag)
    o, lse = attn_forward_packed(qkv, sc.plan, h, hk, hd)
    attn_out = torch.empty(t, d, device=x.device, dtype=torch.bfloat16)
    gemm(o, flat.shadow_of(wo), attn_out, t, d, h * hd, epi=EPI_BF16)
    x1, xn2, rstd2 = C.add_rmsnorm_fwd(x, attn_out, w_post, cfg.norm_eps, True)
    hmid = torch.empty(t, F, device=x.device, dtype=torch.bfloat16)
    gu = torch.empty(t, 2 * F, device=x.device, dtype=torch.bfloat16)
    ag = flat.gather_spec(wg, wu)
    gemm(xn2, flat.shadow_of(wg, wu), hmid, t, 2 * F, d, epi=EPI_SWIGLU, aux=gu, ag=ag)
    mlp_out = torch.empty(t, d, device=x.device, dtype=torch.bfloat16)
    gemm(hmid, flat.shadow_of(wd), mlp_out, t, d, F, epi=EPI_BF16)
    return x1, mlp_out, (x, xn1, rstd1, qkv, o, lse, x1, xn2, rstd2, gu, hmid)


class _Decoder(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_prev, delta_prev, w_in, wq, wk, wv, wo, w_post, wg, wu, wd, sc: StepContext):
        params = (w_in, wq, wk, wv, wo, w_post, wg, wu, wd)
        x1, mlp_out, saved = _layer_forward(x_prev, delta_prev, params, sc)
        ctx.sc = sc
        ctx.has_delta = delta_prev is not None
        ctx.params = params
        if sc.checkpoint:
            # activation checkpointing: keep only the layer inputs, recompute in backward
            ctx.saved = None
            ctx.inputs = (x_prev, delta_prev)
        else:
            ctx.saved = saved
        return x1, mlp_out

    @staticmethod
    def backward(ctx, dx2, dx2b):
        sc = ctx.sc
        cfg = sc.cfg
        flat = sc.flat
        C = _native.module()
        w_in, wq, wk, wv, wo, w_post, wg, wu, wd = ctx.params
        flat.backward_begin(wq, wk, wv, wo, wg, wu, wd)
        if ctx.saved is None:  # checkpointed: recompute this layer's activations
            ctx.saved = _layer_forward(*ctx.inputs, ctx.params, sc)[2]
            ctx.inputs = None
        x, xn1, rstd1, qkv, o, lse, x1, xn2, rstd2, gu, hmid = ctx.saved
        ctx.saved = None
        t, d = x.shape
        h, hk, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        nqkv = (h + 2 * hk) * hd
        F = cfg.d_ff
        dev = x.device
        dx2 = dx2.contiguous()
        dx2b = dx2b.contiguous() if dx2b is not None else dx2.to(torch.bfloat16)
        # one zero fill for the layer's weight gradients (adjacent in the flat buffer), then
        # every weight-gradient writer of the layer accumulates
        flat.prezero(wq, wk, wv, wo, w_post, wg, wu, wd)
        # MLP
        # down-projection dgrad with the SwiGLU backward in its epilogue: [dg | du]
        dgu = torch.empty(t, 2 * F, device=dev, dtype=torch.bfloat16)
        gemm(dx2b, flat.shadow_of(wd), dgu, t, F, d, b_mn=True, epi=EPI_SWIGLU_BWD, aux=gu)
        _wgrad(flat, (wd,), dx2b, hmid)
        dxn2 = torch.empty(t, d, device=dev, dtype=torch.float32)
        gemm(dgu, flat.shadow_of(wg, wu), dxn2, t, d, 2 * F, b_mn=True, epi=EPI_F32)
        _wgrad(flat, (wg, wu), dgu, xn2)
        dx1b = torch.empty(t, d, device=dev, dtype=torch.bfloat16)
        dx1 = C.rmsnorm_bwd(dxn2, x1, w_post, rstd2, dx2, dx1b, flat.grad_of(w_post).view(-1), flat.claim(w_post))
        # attention
        do = torch.empty(t, h * hd, device=dev, dtype=torch.bfloat16)
        gemm(dx1b, flat.shadow_of(wo), do, t, h * hd, d, b_mn=True, epi=EPI_BF16)
        _wgrad(flat, (wo,), dx1b, o)
        dqkv = attn_backward_packed(qkv, o, do, lse, sc.plan, h, hk, hd, rope=(sc.pos, sc.cos, sc.sin))
        dxn1 = torch.empty(t, d, device=dev, dtype=torch.float32)
        gemm(dqkv, flat.shadow_of(wq, wk, wv), dxn1, t, d, nqkv, b_mn=True, epi=EPI_F32)
        _wgrad(flat, (wq, wk, wv), dqkv, xn1)
        dxb = torch.empty(t, d, device=dev, dtype=torch.bfloat16)
        dx = C.rmsnorm_bwd(dxn1, x, w_in, rstd1, dx1, dxb, flat.grad_of(w_in).view(-1), flat.claim(w_in))
        _join_wgrads(dev)
        flat.ready_after(w_in)
        return (dx, dxb if ctx.has_delta else None) + (None,) * 10


# The LM head can keep its bf16 logits for the backward (one elementwise pass instead
# of recomputing the logits GEMM) while they take at most this many bytes.  Off by
# default: on B200 at 8192 x 768 x 32000 the forward GEMM becomes store-bound
# (396 -> 607 us) and the backward gains only 132 us (1104 -> 972 us), so recomputing
# is faster (bench_kernels --cases lmhead).
LOGITS_KEEP_BYTES = 0


class _Head(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_prev, delta_prev, w_norm, w_lm, labels, sc: StepContext):
        cfg = sc.cfg
        C = _native.module()
        x, xf, rstd = C.add_rmsnorm_fwd(x_prev, delta_prev, w_norm, cfg.norm_eps, True)
        ag = sc.flat.gather_spec(w_lm)
        t = xf.shape[0]
        keep = t * cfg.vocab_size * 2 <= LOGITS_KEEP_BYTES and cfg.vocab_size % 8 == 0
        logits = torch.empty(t, cfg.vocab_size, device=xf.device, dtype=torch.bfloat16) if keep else None
        loss, lse = lmhead_ce_forward(xf, sc.flat.shadow_of(w_lm), labels, -100, cfg.z_loss_coeff, ag=ag,
                                      logits_out=logits)
        ctx.sc = sc
        ctx.has_delta = delta_prev is not None
        ctx.logits = logits
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
        dxf = lmhead_ce_backward(
            xf, flat.shadow_of(w_lm), labels, lse, grad, flat.grad_of(w_lm), flat.claim(w_lm), -100, cfg.z_loss_coeff,
            logits=ctx.logits,
        )
        ctx.logits = None
        dxb = torch.empty(x.shape, device=x.device, dtype=torch.bfloat16)
        dx = _native.module().rmsnorm_bwd(dxf, x, w_norm, rstd, None, dxb, flat.grad_of(w_norm).view(-1),
                                          flat.claim(w_norm))
        flat.ready_after(w_norm)
        return dx, (dxb if ctx.has_delta else None), None, None, None, None


def _ensure_flat(model):
    """The model's parameter buffers: :class:`FlatParameters` (single GPU, DDP) or the
    sharded layout of :mod:`packbalance_b200.parallel.sharded` (same interface)."""
    if model.flat is None:
        model.flat = FlatParameters(model)
    model.flat.refresh_shadow()
    return model.flat


def fused_causal_lm_forward(model, input_ids, labels, position_ids, doc_start, attn_plan=None) -> CausalLMOutput:
    cfg = model.cfg
    flat = _ensure_flat(model)
    ids = input_ids.reshape(-1).contiguous()
    pos32 = position_ids.reshape(-1).to(torch.int32).contiguous()
    if attn_plan is not None:
        plan = attn_plan  # built on the host with the batch
    else:
        doc_start = doc_start.reshape(-1).to(device=ids.device, dtype=torch.int32).contiguous()
        plan = attention_plan(doc_start, cfg.n_heads, cfg.n_kv_heads)
    sc = StepContext(model, flat, pos32, plan)
    m = model.model
    x = _Embed.apply(ids, m.embed_tokens.weight, sc)
    delta = None
    for layer in m.layers:
        a, mlp = layer.self_attn, layer.mlp
        x, delta = _Decoder.apply(
            x, delta, layer.input_layernorm.weight, a.q_proj.weight, a.k_proj.weight, a.v_proj.weight,
            a.o_proj.weight, layer.post_attention_layernorm.weight, mlp.gate_proj.weight, mlp.up_proj.weight,
            mlp.down_proj.weight, sc,
        )
    shape = input_ids.shape
    if labels is not None:
        loss = _Head.apply(x, delta, m.norm.weight, model.lm_head_weight, labels.reshape(-1).contiguous(), sc)
        return CausalLMOutput(loss=loss, hidden_states=None)
    _, xf, _ = _native.module().add_rmsnorm_fwd(x, delta, m.norm.weight, cfg.norm_eps, True)
    w = flat.shadow_of(model.lm_head_weight)
    logits = torch.empty(xf.shape[0], cfg.vocab_size, device=xf.device, dtype=torch.bfloat16)
    gemm(xf, w, logits, xf.shape[0], cfg.vocab_size, cfg.d_model, epi=EPI_BF16)
    return CausalLMOutput(
        logits=logits.float().reshape(*shape, cfg.vocab_size), hidden_states=xf.float().reshape(*shape, cfg.d_model)
    )
