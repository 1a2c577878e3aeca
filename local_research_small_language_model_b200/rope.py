"""RoPE tables with the reference's layout and growth rule (model/rope.py:8-98).

The tables are fp32 [max_seq_len, head_dim/2]; the B200 decode kernel applies
the rotation itself (fused into the KV append), with the reference's rounding
sequence.  ``apply_rotary_emb`` is kept for the prefill path.
"""

from __future__ import annotations

from typing import Tuple

import torch
import torch.nn as nn


def precompute_rope_freqs(head_dim: int, max_seq_len: int, theta: float = 10000.0):
    """model/rope.py:8-23."""
    assert head_dim % 2 == 0, "head_dim must be even for RoPE"
    dim_indices = torch.arange(0, head_dim, 2).float()
    inv_freq = 1.0 / (theta ** (dim_indices / head_dim))
    t = torch.arange(max_seq_len).float()
    freqs = torch.outer(t, inv_freq)
    return torch.cos(freqs), torch.sin(freqs)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1 = x[..., : x.shape[-1] // 2]
    x2 = x[..., x.shape[-1] // 2:]
    return torch.cat((-x2, x1), dim=-1)


def apply_rotary_emb(xq, xk, cos, sin, offset: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """model/rope.py:34-65."""
    seq_len = xq.shape[1]
    cos_seq = cos[offset: offset + seq_len, :]
    sin_seq = sin[offset: offset + seq_len, :]
    cos_seq = torch.cat([cos_seq, cos_seq], dim=-1).unsqueeze(0).unsqueeze(2).type_as(xq)
    sin_seq = torch.cat([sin_seq, sin_seq], dim=-1).unsqueeze(0).unsqueeze(2).type_as(xq)
    return (xq * cos_seq) + (rotate_half(xq) * sin_seq), (xk * cos_seq) + (rotate_half(xk) * sin_seq)


class RotaryEmbedding(nn.Module):
    """model/rope.py:68-98: caches cos/sin up to max_seq_len, doubling on demand."""

    def __init__(self, head_dim: int, max_seq_len: int = 4096, theta: float = 10000.0):
        super().__init__()
        self.head_dim = head_dim
        self.theta = theta
        self.max_seq_len = max_seq_len
        cos, sin = precompute_rope_freqs(head_dim, max_seq_len, theta)
        self.register_buffer("cos", cos, persistent=False)
        self.register_buffer("sin", sin, persistent=False)

    def _extend_cache(self, seq_len: int, device: torch.device):
        if seq_len > self.max_seq_len:
            self.max_seq_len = max(seq_len, self.max_seq_len * 2)
            cos, sin = precompute_rope_freqs(self.head_dim, self.max_seq_len, self.theta)
            self.cos = cos.to(device)
            self.sin = sin.to(device)

    def _apply(self, fn, *args, **kwargs):
        """Module.to(dtype) would cast the tables too (the reference's buffers
        become e.g. bf16 under model.to(torch.bfloat16)).  They stay fp32 here:
        the fused decode kernel reads fp32 tables and rounds each entry to the
        activation dtype, and apply_rotary_emb casts with type_as, so results
        equal the reference's cast tables while the kernel never sees a 16-bit
        buffer where it expects fp32."""
        super()._apply(fn, *args, **kwargs)
        if self.cos.dtype != torch.float32 or self.sin.dtype != torch.float32:
            cos, sin = precompute_rope_freqs(self.head_dim, self.max_seq_len, self.theta)
            self.cos = cos.to(self.cos.device)
            self.sin = sin.to(self.sin.device)
        return self

    def ensure(self, seq_len: int) -> None:
        """Grows the tables so positions < seq_len are covered."""
        self._extend_cache(seq_len, self.cos.device)

    def forward(self, xq, xk, offset: int = 0):
        total = offset + xq.shape[1]
        if total > self.max_seq_len:
            self._extend_cache(total, xq.device)
        if xq.is_cuda and xq.shape[-1] % 16 == 0:
            from . import ops  # the fused kernel (sd_rope_qk), same rounding sequence
            return ops.rope_qk(xq, xk, self.cos, self.sin, offset)
        return apply_rotary_emb(xq, xk, self.cos, self.sin, offset=offset)
