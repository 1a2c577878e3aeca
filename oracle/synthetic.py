"""Seeded synthetic inputs shared by the golden generator, the tests and bench.py.

TEST INFRASTRUCTURE ONLY (see oracle/sparda_oracle.py).  Nothing in the product
package imports this module.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class SmallModelConfig:
    """Field names follow model/config.py:7-48 of the reference."""
    vocab_size: int = 512
    n_layer: int = 3
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
    block_size: int = 64
    top_k_blocks: int = 8


def state_shapes(cfg) -> dict:
    """Parameter shapes keyed by the reference's state-dict names
    (model/model.py:16-50, model/transformer.py:50-74, model/attention/base.py:49-52,
    model/forecast.py:23-27)."""
    c, qd, kd = cfg.n_embd, cfg.n_head * cfg.head_dim, cfg.n_kv_head * cfg.head_dim
    fd = cfg.forecast_heads * cfg.forecast_dim
    shapes = {"embeddings.weight": (cfg.vocab_size, c)}
    for i in range(cfg.n_layer):
        p = f"layers.{i}."
        shapes.update({
            p + "attn_norm.weight": (c,),
            p + "attention.wq.weight": (qd, c),
            p + "attention.wk.weight": (kd, c),
            p + "attention.wv.weight": (kd, c),
            p + "attention.wo.weight": (c, qd),
            p + "forecast.wf.weight": (fd, c),
            p + "ffn_norm.weight": (c,),
            p + "ffn.w_gate.weight": (cfg.ffn_dim, c),
            p + "ffn.w_up.weight": (cfg.ffn_dim, c),
            p + "ffn.w_down.weight": (c, cfg.ffn_dim),
        })
    shapes["final_norm.weight"] = (c,)
    return shapes


def model_state(cfg, seed: int = 0, std: float = 0.02) -> dict:
    """Random-init weights, N(0, std) for matrices and 1 + N(0, 0.1) for norm
    gains, drawn from numpy's PCG64 in sorted key order (so any consumer can
    regenerate them without torch's RNG)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name in sorted(state_shapes(cfg)):
        shape = state_shapes(cfg)[name]
        if name.endswith("norm.weight"):
            out[name] = (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32)
        else:
            out[name] = (std * rng.standard_normal(shape)).astype(np.float32)
    return out


def normal(shape, seed: int, scale: float = 1.0, dtype=np.float32) -> np.ndarray:
    """Seeded N(0, scale^2) array (numpy PCG64)."""
    return (scale * np.random.default_rng(seed).standard_normal(shape)).astype(dtype)
