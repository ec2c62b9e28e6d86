"""Llama-style decoder for packed-sequence training.

Architecture and parameter names follow the reference (``model/llama.py:36-290``):
pre-norm RMSNorm, GQA attention with RoPE on per-document positions, SwiGLU MLP,
tied embeddings by default, N(0, init_std) init with residual projections scaled by
1/sqrt(2 * n_layers).  ``forward`` returns the *summed* token cross-entropy (plus
z-loss) when labels are given, otherwise logits.

Two execution paths share the same parameters:

* CPU tensors (and ``attention_backend="eager"``): plain PyTorch modules, the
  numerics oracle.
* CUDA tensors: :mod:`packbalance_b200.models.fused`, one autograd node per decoder
  layer built from the native sm100 kernels (tcgen05 GEMMs with RoPE / SwiGLU /
  residual epilogues, varlen document attention, fused LM-head cross-entropy).
  Weight gradients are written straight into the flat fp32 gradient buffer that the
  parameter ``.grad`` tensors alias.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from packbalance_b200.config import ModelConfig
from packbalance_b200.models.attention import attention_forward, doc_start_from_doc_ids
from packbalance_b200.models.rope import RotaryEmbedding, apply_rotary_pos_emb
from packbalance_b200.ops.reference import (
    chunked_linear_cross_entropy,
    rmsnorm_reference,
    swiglu_reference,
)


@dataclass
class CausalLMOutput:
    loss: torch.Tensor | None = None
    logits: torch.Tensor | None = None
    hidden_states: torch.Tensor | None = None


class RMSNorm(nn.Module):
    def __init__(self, d_model: int, eps: float, use_fused: bool = True) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d_model))
        self.eps = eps
        self.use_fused = use_fused

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.is_cuda and self.use_fused:
            from packbalance_b200.ops.rmsnorm import rmsnorm

            return rmsnorm(x, self.weight, self.eps)
        return rmsnorm_reference(x, self.weight, self.eps)


class LlamaMLP(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(cfg.d_model, cfg.d_ff, bias=False)
        self.up_proj = nn.Linear(cfg.d_model, cfg.d_ff, bias=False)
        self.down_proj = nn.Linear(cfg.d_ff, cfg.d_model, bias=False)
        self.use_fused = cfg.use_fused_swiglu

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        gate, up = self.gate_proj(x), self.up_proj(x)
        if x.is_cuda and self.use_fused:
            from packbalance_b200.ops.swiglu import swiglu

            hidden = swiglu(gate, up)
        else:
            hidden = swiglu_reference(gate, up)
        return self.down_proj(hidden)


class LlamaAttention(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.n_heads = cfg.n_heads
        self.n_kv_heads = cfg.n_kv_heads
        self.head_dim = cfg.head_dim
        self.q_proj = nn.Linear(cfg.d_model, cfg.n_heads * self.head_dim, bias=False)
        self.k_proj = nn.Linear(cfg.d_model, cfg.n_kv_heads * self.head_dim, bias=False)
        self.v_proj = nn.Linear(cfg.d_model, cfg.n_kv_heads * self.head_dim, bias=False)
        self.o_proj = nn.Linear(cfg.n_heads * self.head_dim, cfg.d_model, bias=False)
        self.attention_backend = cfg.attention_backend
        self.compile_attention = cfg.compile_attention

    def forward(self, hidden, cos, sin, doc_ids, block_mask=None) -> torch.Tensor:
        b, s, _ = hidden.shape
        q = self.q_proj(hidden).view(b, s, self.n_heads, self.head_dim).transpose(1, 2)
        k = self.k_proj(hidden).view(b, s, self.n_kv_heads, self.head_dim).transpose(1, 2)
        v = self.v_proj(hidden).view(b, s, self.n_kv_heads, self.head_dim).transpose(1, 2)
        q, k = apply_rotary_pos_emb(q, k, cos, sin)
        out = attention_forward(
            q, k, v, doc_ids, block_mask=block_mask, backend=self.attention_backend,
            compile_attention=self.compile_attention,
        )
        return self.o_proj(out.transpose(1, 2).reshape(b, s, -1))


class LlamaDecoderLayer(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.input_layernorm = RMSNorm(cfg.d_model, cfg.norm_eps, cfg.use_fused_rmsnorm)
        self.self_attn = LlamaAttention(cfg)
        self.post_attention_layernorm = RMSNorm(cfg.d_model, cfg.norm_eps, cfg.use_fused_rmsnorm)
        self.mlp = LlamaMLP(cfg)

    def forward(self, hidden, cos, sin, doc_ids, block_mask=None) -> torch.Tensor:
        hidden = hidden + self.self_attn(self.input_layernorm(hidden), cos, sin, doc_ids, block_mask)
        return hidden + self.mlp(self.post_attention_layernorm(hidden))


class LlamaModel(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.layers = nn.ModuleList(LlamaDecoderLayer(cfg) for _ in range(cfg.n_layers))
        self.norm = RMSNorm(cfg.d_model, cfg.norm_eps, cfg.use_fused_rmsnorm)
        self.rotary = RotaryEmbedding(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
        self.gradient_checkpointing = False

    def forward(self, input_ids, position_ids, doc_ids, block_mask=None) -> torch.Tensor:
        """Reference-path decoder stack (final norm applied)."""
        hidden = self.embed_tokens(input_ids)
        cos, sin = self.rotary(position_ids)
        for layer in self.layers:
            if self.gradient_checkpointing and self.training:
                hidden = torch.utils.checkpoint.checkpoint(
                    layer, hidden, cos, sin, doc_ids, block_mask, use_reentrant=False
                )
            else:
                hidden = layer(hidden, cos, sin, doc_ids, block_mask)
        return self.norm(hidden)


class LlamaForCausalLM(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.model = LlamaModel(cfg)
        self.lm_head = None if cfg.tie_embeddings else nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        self.apply(self._init_weights)
        self._scale_residual_projections()
        # Flat fp32/bf16/grad buffers that the native path works on; attached by
        # parallel.flat.FlatParameters (lazily on the first CUDA forward).
        self.flat = None
        # False forces the module path on CUDA too (used under torch FSDP2).
        self.native = True

    @property
    def lm_head_weight(self) -> torch.Tensor:
        return self.model.embed_tokens.weight if self.lm_head is None else self.lm_head.weight

    def _init_weights(self, module: nn.Module) -> None:
        if isinstance(module, (nn.Linear, nn.Embedding)):
            nn.init.normal_(module.weight, mean=0.0, std=self.cfg.init_std)

    def _scale_residual_projections(self) -> None:
        std = self.cfg.init_std / math.sqrt(2 * self.cfg.n_layers)
        for layer in self.model.layers:
            nn.init.normal_(layer.self_attn.o_proj.weight, mean=0.0, std=std)
            nn.init.normal_(layer.mlp.down_proj.weight, mean=0.0, std=std)

    def gradient_checkpointing_enable(self) -> None:
        self.model.gradient_checkpointing = True

    def gradient_checkpointing_disable(self) -> None:
        self.model.gradient_checkpointing = False

    def uses_native_path(self, input_ids: torch.Tensor) -> bool:
        return input_ids.is_cuda and self.native and self.cfg.attention_backend != "eager"

    def forward(
        self,
        input_ids: torch.Tensor,
        labels: torch.Tensor | None = None,
        position_ids: torch.Tensor | None = None,
        doc_ids: torch.Tensor | None = None,
        block_mask=None,
        doc_start: torch.Tensor | None = None,
        attn_plan: dict | None = None,
    ) -> CausalLMOutput:
        """Reference signature plus ``doc_start`` (first token of each token's document)
        and ``attn_plan`` (the attention work lists of
        :func:`packbalance_b200.ops.attention.attention_plan_host`, already on the
        device), both optional and used only by the native path."""
        if input_ids.dim() == 1:
            input_ids = input_ids.unsqueeze(0)
            labels = labels.unsqueeze(0) if labels is not None else None
            position_ids = position_ids.unsqueeze(0) if position_ids is not None else None
            doc_ids = doc_ids.unsqueeze(0) if doc_ids is not None else None
        if position_ids is None:
            position_ids = torch.arange(input_ids.shape[1], device=input_ids.device).expand_as(input_ids)
        if doc_ids is None:
            doc_ids = torch.zeros_like(input_ids)
        if self.uses_native_path(input_ids):
            from packbalance_b200.models.fused import fused_causal_lm_forward

            if doc_start is None and attn_plan is None:
                doc_start = (
                    block_mask if isinstance(block_mask, torch.Tensor) else doc_start_from_doc_ids(doc_ids)
                )
            return fused_causal_lm_forward(self, input_ids, labels, position_ids, doc_start, attn_plan)
        hidden = self.model(input_ids, position_ids, doc_ids, block_mask)
        if labels is None:
            return CausalLMOutput(logits=hidden @ self.lm_head_weight.t(), hidden_states=hidden)
        loss = chunked_linear_cross_entropy(
            hidden,
            self.lm_head_weight,
            labels,
            chunk_size=self.cfg.ce_chunk_size,
            ignore_index=-100,
            z_loss_coeff=self.cfg.z_loss_coeff,
        )
        return CausalLMOutput(loss=loss, hidden_states=hidden)

    @torch.no_grad()
    def generate(
        self,
        input_ids: torch.Tensor,
        max_new_tokens: int = 32,
        temperature: float = 0.0,
        top_k: int | None = None,
    ) -> torch.Tensor:
        """Greedy or temperature/top-k sampling; recomputes the prefix each token."""
        was_training = self.training
        self.eval()
        ids = input_ids
        try:
            for _ in range(max_new_tokens):
                if ids.shape[1] >= self.cfg.max_seq_len:
                    break
                pos = torch.arange(ids.shape[1], device=ids.device).expand_as(ids)
                logits = self.forward(ids, position_ids=pos, doc_ids=torch.zeros_like(ids)).logits
                last = logits[:, -1, :].float()
                if temperature <= 0:
                    nxt = last.argmax(dim=-1, keepdim=True)
                else:
                    last = last / temperature
                    if top_k is not None:
                        kth = torch.topk(last, min(top_k, last.shape[-1])).values[:, -1:]
                        last = last.masked_fill(last < kth, float("-inf"))
                    nxt = torch.multinomial(F.softmax(last, dim=-1), num_samples=1)
                ids = torch.cat([ids, nxt.to(ids.dtype)], dim=1)
            return ids
        finally:
            self.train(was_training)


def count_parameters(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())
