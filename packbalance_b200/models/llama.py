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
from packbalance_b200.models.rope import RotaryEmbedding
from packbalance_b200.ops.reference import (
    chunked_linear_cross_entropy,
    rmsnorm_reference,
    rope_reference,
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


class KVCache:
    """Keys and values of every layer for incremental decoding.

    ``k`` / ``v``: ``[n_layers, B, capacity, n_kv_heads, head_dim]`` (keys stored after
    RoPE); ``length`` tokens of each row are valid.  A decode pass appends the new
    tokens of every layer at ``length`` and then advances ``length`` once.
    """

    def __init__(self, cfg: ModelConfig, batch: int, capacity: int, dtype: torch.dtype,
                 device: torch.device) -> None:
        shape = (cfg.n_layers, batch, capacity, cfg.n_kv_heads, cfg.head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.length = 0

    @property
    def capacity(self) -> int:
        return self.k.shape[2]

    def extend(self, layer: int, k_new: torch.Tensor, v_new: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Store ``[B, n, KV, D]`` keys/values of ``layer`` after the valid prefix and
        return that layer's keys and values up to and including them."""
        end = self.length + k_new.shape[1]
        if end > self.capacity:
            raise ValueError(f"KV cache full: {end} > {self.capacity} tokens")
        self.k[layer, :, self.length:end] = k_new
        self.v[layer, :, self.length:end] = v_new
        return self.k[layer, :, :end], self.v[layer, :, :end]


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

    def _rotated_heads(self, hidden: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
        """q | k | v from one projection (the three weights stacked, as the native QKV
        GEMM stores them), RoPE applied to the q and k heads together.  Token-major
        ``[B, S, heads, D]`` results; ``cos`` / ``sin`` are ``[B, S, D/2]``."""
        h, kv = self.n_heads, self.n_kv_heads
        w = torch.cat((self.q_proj.weight, self.k_proj.weight, self.v_proj.weight))
        heads = F.linear(hidden, w).unflatten(-1, (h + 2 * kv, self.head_dim))
        qk = rope_reference(heads[:, :, : h + kv], cos.unsqueeze(2), sin.unsqueeze(2))
        return qk[:, :, :h], qk[:, :, h:], heads[:, :, h + kv:]

    def forward(self, hidden, cos, sin, doc_ids, block_mask=None, cache: tuple[KVCache, int] | None = None):
        """Packed-sequence attention (``doc_ids`` separate the documents), or, with
        ``cache=(kv_cache, layer)``, the next tokens of each row attending to the
        cached prefix and causally to each other."""
        q, k, v = self._rotated_heads(hidden, cos, sin)
        if cache is None:
            out = attention_forward(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), doc_ids,
                                    block_mask=block_mask, backend=self.attention_backend,
                                    compile_attention=self.compile_attention).transpose(1, 2)
        else:
            kv_cache, layer = cache
            past = kv_cache.length
            k_all, v_all = kv_cache.extend(layer, k, v)
            n, total = q.shape[1], k_all.shape[1]
            visible = torch.arange(total, device=q.device)[None, :] <= past + torch.arange(n, device=q.device)[:, None]
            out = F.scaled_dot_product_attention(q.transpose(1, 2), k_all.transpose(1, 2), v_all.transpose(1, 2),
                                                 attn_mask=visible, enable_gqa=True).transpose(1, 2)
        return self.o_proj(out.flatten(2))


class LlamaDecoderLayer(nn.Module):
    """Pre-norm block: ``x + attn(norm(x))`` then ``+ mlp(norm(.))``."""

    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.input_layernorm = RMSNorm(cfg.d_model, cfg.norm_eps, cfg.use_fused_rmsnorm)
        self.self_attn = LlamaAttention(cfg)
        self.post_attention_layernorm = RMSNorm(cfg.d_model, cfg.norm_eps, cfg.use_fused_rmsnorm)
        self.mlp = LlamaMLP(cfg)

    def forward(self, hidden, cos, sin, doc_ids, block_mask=None, cache: tuple[KVCache, int] | None = None):
        mixed = self.self_attn(self.input_layernorm(hidden), cos, sin, doc_ids, block_mask, cache)
        residual = hidden + mixed
        return residual + self.mlp(self.post_attention_layernorm(residual))


class LlamaModel(nn.Module):
    def __init__(self, cfg: ModelConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.layers = nn.ModuleList(LlamaDecoderLayer(cfg) for _ in range(cfg.n_layers))
        self.norm = RMSNorm(cfg.d_model, cfg.norm_eps, cfg.use_fused_rmsnorm)
        self.rotary = RotaryEmbedding(cfg.head_dim, cfg.max_seq_len, cfg.rope_theta)
        self.gradient_checkpointing = False

    def forward(self, input_ids, position_ids, doc_ids, block_mask=None, kv_cache: KVCache | None = None):
        """Decoder stack on the module path (final norm applied).  With ``kv_cache``
        the tokens continue the cached rows: their positions start at the cache
        length, and the cache grows by their count."""
        if kv_cache is not None:
            position_ids = kv_cache.length + torch.arange(input_ids.shape[1], device=input_ids.device)
            position_ids = position_ids.expand_as(input_ids)
        cos, sin = self.rotary(position_ids)
        hidden = self.embed_tokens(input_ids)
        recompute = self.gradient_checkpointing and self.training and kv_cache is None
        for i, layer in enumerate(self.layers):
            if recompute:
                hidden = torch.utils.checkpoint.checkpoint(layer, hidden, cos, sin, doc_ids, block_mask,
                                                           use_reentrant=False)
            else:
                hidden = layer(hidden, cos, sin, doc_ids, block_mask,
                               None if kv_cache is None else (kv_cache, i))
        if kv_cache is not None:
            kv_cache.length += input_ids.shape[1]
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
        return self._head(hidden, labels)

    def _head(self, hidden: torch.Tensor, labels: torch.Tensor | None) -> CausalLMOutput:
        """Module-path head: the summed chunked cross-entropy (+ z-loss) against
        ``labels``, or the logits when there are none."""
        out = CausalLMOutput(hidden_states=hidden)
        if labels is not None:
            out.loss = chunked_linear_cross_entropy(hidden, self.lm_head_weight, labels,
                                                    chunk_size=self.cfg.ce_chunk_size, ignore_index=-100,
                                                    z_loss_coeff=self.cfg.z_loss_coeff)
        else:
            out.logits = F.linear(hidden, self.lm_head_weight)
        return out

    @staticmethod
    def _pick_next(logits: torch.Tensor, temperature: float, top_k: int | None) -> torch.Tensor:
        """``[B, V]`` fp32 logits -> ``[B, 1]`` token ids: argmax when ``temperature <=
        0``, else a draw from softmax(logits / temperature), restricted to the
        ``top_k`` largest logits when given."""
        if temperature <= 0:
            return logits.argmax(dim=-1, keepdim=True)
        scaled = logits / temperature
        if top_k is None:
            return torch.multinomial(scaled.softmax(dim=-1), 1)
        best, where = scaled.topk(min(top_k, scaled.shape[-1]), dim=-1)
        return where.gather(-1, torch.multinomial(best.softmax(dim=-1), 1))

    @torch.no_grad()
    def generate(
        self,
        input_ids: torch.Tensor,
        max_new_tokens: int = 32,
        temperature: float = 0.0,
        top_k: int | None = None,
    ) -> torch.Tensor:
        """Continue every row of ``input_ids`` ``[B, S]`` by up to ``max_new_tokens``
        tokens, never past ``max_seq_len`` in total.

        The prompt runs through the decoder once and fills a :class:`KVCache`; each
        further token is a one-token pass that attends to the cache, so a sequence
        of n new tokens costs O(n) token passes instead of re-running the prefix
        every step.  Runs on the module path (any device)."""
        budget = min(max_new_tokens, self.cfg.max_seq_len - input_ids.shape[1])
        if budget <= 0:
            return input_ids
        was_training = self.training
        self.eval()
        try:
            w = self.lm_head_weight
            cache = KVCache(self.cfg, input_ids.shape[0], input_ids.shape[1] + budget, w.dtype, w.device)
            pieces = [input_ids]
            step_ids = input_ids
            for i in range(budget):
                hidden = self.model(step_ids, None, None, kv_cache=cache)
                logits = F.linear(hidden[:, -1], w).float()
                step_ids = self._pick_next(logits, temperature, top_k).to(input_ids.dtype)
                pieces.append(step_ids)
            return torch.cat(pieces, dim=1)
        finally:
            self.train(was_training)


def count_parameters(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())
