"""Drop-in forecast modules (model/forecast.py) backed by the sm_100a kernels."""

from __future__ import annotations

from typing import Tuple

import torch
import torch.nn as nn

from . import ops


class ForecastProjection(nn.Module):
    """model/forecast.py:11-40: wf = Linear(n_embd, forecast_heads*forecast_dim)."""

    def __init__(self, config):
        super().__init__()
        self.n_embd = config.n_embd
        self.forecast_heads = config.forecast_heads
        self.forecast_dim = config.forecast_dim
        self.wf = nn.Linear(self.n_embd, self.forecast_heads * self.forecast_dim, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, t, _ = x.shape
        return self.wf(x).view(b, t, self.forecast_heads, self.forecast_dim)


class KVBlockCompressor(nn.Module):
    """KVBlockCompressor (model/forecast.py:43-78) on the compressor kernel.

    forward(k [B,T,H,D]) -> fp32 block prototypes [B,N_b,H,D].  The projection
    is the identity when head_dim == forecast_dim, as in the reference; other
    geometries apply a bias-free Linear after the kernel.
    """

    def __init__(self, block_size: int = 32, head_dim: int = 64, forecast_dim: int = 64):
        super().__init__()
        self.block_size = block_size
        self.head_dim = head_dim
        self.forecast_dim = forecast_dim
        self.proj = nn.Linear(head_dim, forecast_dim, bias=False) if head_dim != forecast_dim else nn.Identity()

    def forward(self, k: torch.Tensor) -> torch.Tensor:
        reps = ops.compress_blocks(k, self.block_size)
        return self.proj(reps)


class ForecastBlockSelector(nn.Module):
    """ForecastBlockSelector (model/forecast.py:81-130) on the fp32 selector kernel.

    forward(forecast [B,Tq,H,D], block_reps [B,N_b,H,D], top_k, is_causal) ->
    (scores [B,H,Tq,N_b] fp32, topk_indices [B,H,Tq,min(top_k,N_b)] int64).
    Equal scores (the -inf of masked blocks included) are ordered by ascending
    block index.
    """

    def __init__(self, block_size: int = 32, forecast_dim: int = 64):
        super().__init__()
        self.block_size = block_size
        self.forecast_dim = forecast_dim

    def forward(self, forecast: torch.Tensor, block_reps: torch.Tensor, top_k: int,
                is_causal: bool = True, q_offset: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
        return ops.select_blocks(forecast, block_reps, top_k, self.block_size, is_causal, q_offset)
