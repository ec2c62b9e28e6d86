"""Analytical per-document FLOP model used by the packers and the scheduler.

The formula is the reference's (``data/cost.py:23-130``) so that pack costs,
schedules and MFU agree between the two frameworks:

    cost(doc of length L) = (2 * P_lin + 8 * n_layers * d_model) * L
                            + 2 * n_layers * d_model * L**2

where ``P_lin`` counts every matmul weight touched per token (QKV, O, SwiGLU and the
LM head).  A padded row of ``S`` slots is charged ``S`` tokens and a dense ``S**2``
attention term.  Training FLOPs are 3x the forward cost.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from packbalance_b200.config import ModelConfig


@dataclass(frozen=True)
class FlopModel:
    vocab_size: int
    d_model: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    d_ff: int

    @classmethod
    def from_config(cls, cfg: ModelConfig) -> FlopModel:
        return cls(cfg.vocab_size, cfg.d_model, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.d_ff)

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    @property
    def d_kv(self) -> int:
        return self.n_kv_heads * self.head_dim

    @property
    def attn_params_per_layer(self) -> int:
        d = self.d_model
        return d * (d + 2 * self.d_kv) + d * d

    @property
    def mlp_params_per_layer(self) -> int:
        return 3 * self.d_model * self.d_ff

    @property
    def linear_params(self) -> int:
        """Matmul weights used per token, LM head included."""
        per_layer = self.attn_params_per_layer + self.mlp_params_per_layer
        return self.n_layers * per_layer + self.vocab_size * self.d_model

    @property
    def embedding_params(self) -> int:
        return self.vocab_size * self.d_model

    @property
    def total_params(self) -> int:
        norm_params = (2 * self.n_layers + 1) * self.d_model
        blocks = self.n_layers * (self.attn_params_per_layer + self.mlp_params_per_layer)
        return self.embedding_params + blocks + norm_params

    @property
    def linear_flops_per_token(self) -> float:
        return 2.0 * self.linear_params

    @property
    def elementwise_flops_per_token(self) -> float:
        return 8.0 * self.n_layers * self.d_model

    @property
    def attention_flops_coeff(self) -> float:
        return 2.0 * self.n_layers * self.d_model

    @property
    def _per_token(self) -> float:
        return self.linear_flops_per_token + self.elementwise_flops_per_token

    def doc_cost(self, length: int | np.ndarray) -> float | np.ndarray:
        """Forward FLOPs of one document (vectorised over ``length``)."""
        n = np.asarray(length, dtype=np.float64)
        return self._per_token * n + self.attention_flops_coeff * n * n

    def pack_cost(self, lengths: list[int] | np.ndarray) -> float:
        n = np.asarray(lengths, dtype=np.float64)
        if n.size == 0:
            return 0.0
        return float(self._per_token * n.sum() + self.attention_flops_coeff * np.dot(n, n))

    def padded_batch_cost(self, lengths: list[int] | np.ndarray, pad_len: int) -> float:
        rows = float(len(lengths))
        return float(
            self._per_token * rows * pad_len + self.attention_flops_coeff * rows * pad_len * pad_len
        )

    def train_flops(self, lengths: list[int] | np.ndarray) -> float:
        return 3.0 * self.pack_cost(lengths)

    def useful_tokens_per_step(self, lengths: list[int] | np.ndarray) -> int:
        return int(np.asarray(lengths, dtype=np.int64).sum())

    # --- additions: hardware FLOPs actually executed by the sm100 kernels ---
    def matmul_train_flops(self, tokens: int) -> float:
        """fwd+bwd matmul FLOPs (6 * P_lin * tokens), what the GEMM kernels execute."""
        return 6.0 * self.linear_params * tokens

    def attention_train_flops(self, lengths: list[int] | np.ndarray) -> float:
        """fwd+bwd FLOPs of exact causal document attention (QK^T, PV; bwd = 2.5x fwd)."""
        n = np.asarray(lengths, dtype=np.float64)
        causal_pairs = float((n * (n + 1) / 2).sum())
        fwd = 4.0 * self.n_layers * self.n_heads * self.head_dim * causal_pairs
        return 3.5 * fwd


def cost_stats(costs: list[float] | np.ndarray) -> dict[str, float]:
    c = np.asarray(costs, dtype=np.float64)
    if c.size == 0:
        return {"mean": 0.0, "std": 0.0, "cv": 0.0, "p50": 0.0, "p99": 0.0, "max": 0.0}
    mean = float(c.mean())
    std = float(c.std())
    return {
        "mean": mean,
        "std": std,
        "cv": std / mean if mean else 0.0,
        "p50": float(np.percentile(c, 50)),
        "p99": float(np.percentile(c, 99)),
        "max": float(c.max()),
    }
