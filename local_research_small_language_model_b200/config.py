"""ModelConfig with the reference's field names and defaults (model/config.py:7-48)."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class ModelConfig:
    vocab_size: int = 32000
    n_layer: int = 12
    n_embd: int = 768
    n_head: int = 12
    n_kv_head: int = 4
    head_dim: int = 64
    ffn_dim: int = 2048
    forecast_heads: int = 4
    forecast_dim: int = 64
    context_length: int = 1024
    rope_theta: float = 10000.0
    norm_eps: float = 1e-6
    tie_embeddings: bool = True
    initializer_range: float = 0.02
    attention_backend: str = "b200_forecast"
    sparse_mode: str = "forecast"
    block_size: int = 32
    top_k_blocks: int = 4
    num_queries_per_kv: int = 3
    # decode-time causal rule of the selector: "reference" (the reference's
    # literal behaviour, see ops.RULES) or "absolute"
    selector_rule: str = "reference"
    # when decode scores the current block: "after_append" (SparseAttention and
    # ForecastOffloadAttention, model/attention/sparse.py:133-139) or
    # "before_append" (AsyncForecastOffloadAttention.prefetch,
    # model/attention/async_offload.py:241-260)
    selection_timing: str = "after_append"

    def __post_init__(self):
        assert self.n_embd == self.n_head * self.head_dim, (
            f"n_embd ({self.n_embd}) must equal n_head ({self.n_head}) * head_dim ({self.head_dim})")
        assert self.n_head % self.n_kv_head == 0, (
            f"n_head ({self.n_head}) must be divisible by n_kv_head ({self.n_kv_head})")
        self.num_queries_per_kv = self.n_head // self.n_kv_head
