"""Block-major KV cache for the B200 path (replaces model/attention/base.py:11-32).

Storage per layer:
  k_store, v_store  [B, H, Tcap, D]  activation dtype; one (head, block) tile of
                    block_size x D is contiguous (8 KB at 64 x 64 bf16), so the
                    decode kernel stages a block with one bulk copy;
  proto_sum         [B, H, NBcap, D] fp32 running block sums of K, so the
                    compressor (model/forecast.py:57-78) is never re-run over
                    the whole cache: prototype = proto_sum / block_size;
  len_dev           int32 on the device, tokens cached so far (read by the
                    fused decode kernel, which makes CUDA-graph replay possible).
Tcap is max_seq_len rounded up to a whole block.  ``k`` and ``v`` return views
in the reference's [B, T, H, D] layout.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import ops


class B200KVCache:
    def __init__(self, max_batch_size: int, max_seq_len: int, n_kv_head: int, head_dim: int,
                 device: torch.device, dtype: torch.dtype, block_size: int = 64,
                 len_dev: Optional[torch.Tensor] = None):
        self.block_size = block_size
        self.max_batch_size = max_batch_size
        self.max_seq_len = max_seq_len
        self.n_kv_head = n_kv_head
        self.head_dim = head_dim
        self.tcap = ops.num_blocks(max_seq_len, block_size) * block_size
        self.nbcap = self.tcap // block_size
        self.k_store = torch.zeros(max_batch_size, n_kv_head, self.tcap, head_dim, device=device, dtype=dtype)
        self.v_store = torch.zeros_like(self.k_store)
        self.proto_sum = torch.zeros(max_batch_size, n_kv_head, self.nbcap, head_dim, device=device,
                                     dtype=torch.float32)
        self.len_dev = len_dev if len_dev is not None else torch.zeros(1, dtype=torch.int32, device=device)
        self.current_len = 0

    @property
    def k(self) -> torch.Tensor:
        return self.k_store.permute(0, 2, 1, 3)

    @property
    def v(self) -> torch.Tensor:
        return self.v_store.permute(0, 2, 1, 3)

    def update(self, xk: torch.Tensor, xv: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Appends xk, xv [B,T,H,D]; returns the cached [B,current_len,H,D] views
        (KVCache.update, model/attention/base.py:19-29)."""
        t = xk.shape[1]
        if self.current_len + t > self.tcap:
            raise ValueError(f"cache overflow: {self.current_len} + {t} > {self.tcap}")
        ops.kv_append(xk, xv, self.k_store, self.v_store, self.proto_sum, self.current_len, self.block_size)
        self.advance(t)
        return self.k[:, :self.current_len], self.v[:, :self.current_len]

    def advance(self, t: int, device: bool = True) -> None:
        """Bumps the host length and, unless the caller bumps a shared length
        array itself, the device length."""
        self.current_len += t
        if device:
            self.len_dev.add_(t)

    def prototypes(self) -> torch.Tensor:
        """Block prototypes [B, N_b, H, D] fp32 of the cached tokens."""
        nb = ops.num_blocks(self.current_len, self.block_size)
        return (self.proto_sum[:, :, :nb] / self.block_size).permute(0, 2, 1, 3)

    def reset(self) -> None:
        self.current_len = 0
        self.len_dev.zero_()
