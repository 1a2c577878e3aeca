"""Offloaded KV cache for the B200 path (OffloadedKVCache and
AsyncOffloadedKVCache, model/attention/offload.py:23-128 and
model/attention/async_offload.py:28-112).

The authoritative K/V rows live in pinned host memory, block-major
[B, Hkv, Tcap, D] (the reference keeps [B, T, Hkv, D]), and the GPU reads and
writes them directly through unified addressing: the decode kernel writes each
new token through to the host copy, and the prefetch kernel copies the blocks
the next step needs into device slots.  Block indices never travel to the host
(the reference calls ``.to("cpu")`` on them, async_offload.py:78).

Device state per layer:
  slot_k, slot_v  [B, Hkv, (2 + kslots) * 64, D]: slot 0 = sink block 0, slot 1 =
                  the block being appended to, slots 2.. = staged blocks
                  (kslots = top_k, or cache_blocks for an LRU block cache);
  slot_block      int32 [B, Hkv, 2 * kslots + 1]: which block each slot holds
                  (-1 empty), then 0 once the sink is loaded, then the
                  position each slot was last used at;
  cand / cand_slot  the forecast candidates of the next step and their slots;
  proto_sum       fp32 running block sums (selection never reads the host);
  stats           int64 [3]: blocks wanted, hits, bytes copied host -> device.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import ops


def _check_device_mapped(t: torch.Tensor, device: torch.device) -> None:
    """The kernels dereference the host store's own address on the GPU: check
    that the pinned allocation is mapped there at the same address."""
    from cuda.bindings import runtime as rt
    with torch.cuda.device(device):
        err, attrs = rt.cudaPointerGetAttributes(t.data_ptr())
    if err != rt.cudaError_t.cudaSuccess or int(attrs.devicePointer) != t.data_ptr():
        raise RuntimeError("pinned host memory is not mapped at the same address on the GPU "
                           f"({err}); offloaded caches need unified addressing")


class B200OffloadKVCache:
    def __init__(self, max_batch_size: int, max_seq_len: int, n_kv_head: int, head_dim: int,
                 gpu_device: torch.device, dtype: torch.dtype = torch.bfloat16, pin_memory: bool = True,
                 transfer_stream: Optional[torch.cuda.Stream] = None, block_size: int = 64, top_k: int = 8,
                 len_dev: Optional[torch.Tensor] = None, cache_blocks: Optional[int] = None):
        gpu_device = torch.device(gpu_device)
        if gpu_device.type != "cuda":
            raise ValueError("the B200 offloaded cache needs a CUDA device")
        if not pin_memory:
            raise ValueError("the GPU reads the host store directly: it must be pinned")
        if block_size != 64 or head_dim != 64:
            raise NotImplementedError("offloaded caches use 64-token blocks and head_dim 64")
        self.max_batch_size = max_batch_size
        self.max_seq_len = max_seq_len
        self.n_kv_head = n_kv_head
        self.head_dim = head_dim
        self.gpu_device = gpu_device
        self.dtype = dtype
        self.block_size = block_size
        # device slots for selected blocks besides the sink and the current
        # block: top_k of them by default (each step's candidates); more make
        # the slots a block cache with least-recently-used replacement
        self.top_k = top_k
        self.kslots = top_k if cache_blocks is None else int(cache_blocks)
        if not top_k <= self.kslots <= 32:
            raise ValueError(f"cache_blocks must be in [top_k, 32], got {self.kslots}")
        self.tcap = ops.num_blocks(max_seq_len, block_size) * block_size
        self.nbcap = self.tcap // block_size
        shape = (max_batch_size, n_kv_head, self.tcap, head_dim)
        self.host_k = torch.zeros(shape, dtype=dtype, pin_memory=True)
        self.host_v = torch.zeros(shape, dtype=dtype, pin_memory=True)
        for t in (self.host_k, self.host_v):
            _check_device_mapped(t, gpu_device)
        s = (2 + self.kslots) * block_size
        self.slot_k = torch.zeros(max_batch_size, n_kv_head, s, head_dim, device=gpu_device, dtype=dtype)
        self.slot_v = torch.zeros_like(self.slot_k)
        # per (sequence, kv head): the block in each slot, the sink flag, the
        # position each slot was last used at
        self.slot_block = torch.full((max_batch_size, n_kv_head, 2 * self.kslots + 1), -1, dtype=torch.int32,
                                     device=gpu_device)
        self.cand_slot = torch.full((max_batch_size, n_kv_head, top_k), -1, dtype=torch.int32, device=gpu_device)
        self.cand = (torch.full((max_batch_size, n_kv_head, top_k), -1, dtype=torch.int32, device=gpu_device),
                     torch.zeros(max_batch_size, n_kv_head, top_k, dtype=torch.float32, device=gpu_device))
        self.proto_sum = torch.zeros(max_batch_size, n_kv_head, self.nbcap, head_dim, device=gpu_device,
                                     dtype=torch.float32)
        self.len_dev = len_dev if len_dev is not None else torch.zeros(1, dtype=torch.int32, device=gpu_device)
        self.stats = torch.zeros(3, dtype=torch.int64, device=gpu_device)
        self.transfer_stream = transfer_stream or torch.cuda.Stream(device=gpu_device)
        self.prefetch_event = torch.cuda.Event()
        self.prefetched = False   # a prefetch for the next decode step is in flight
        self.has_cand = False     # ... and it staged forecast candidates
        self.current_len = 0
        self.total_transfer_calls = 0

    # -- reference-compatible views and accounting
    @property
    def cpu_k(self) -> torch.Tensor:
        """Host store in the reference's [B, T, H, D] layout (a view)."""
        return self.host_k.permute(0, 2, 1, 3)

    @property
    def cpu_v(self) -> torch.Tensor:
        return self.host_v.permute(0, 2, 1, 3)

    @property
    def total_bytes_transferred(self) -> int:
        return int(self.stats[2].item())

    def hit_rate(self) -> float:
        wanted, hits = (int(x) for x in self.stats[:2].tolist())
        return hits / wanted if wanted else 0.0

    def get_full_cpu_kv(self) -> Tuple[torch.Tensor, torch.Tensor]:
        return self.cpu_k[:, :self.current_len], self.cpu_v[:, :self.current_len]

    def prototypes(self) -> torch.Tensor:
        return self.proto_sum / self.block_size

    # -- writes
    def update(self, xk: torch.Tensor, xv: torch.Tensor) -> int:
        """Prefill of an empty cache with xk, xv [B, T, H, D] (device tensors):
        host store, running block sums, the sink slot and the current-block
        slot.  Decode steps append through the fused kernel instead."""
        t = xk.shape[1]
        if self.current_len != 0:
            raise NotImplementedError("appending a prompt to a non-empty offloaded cache")
        if t > self.tcap:
            raise ValueError(f"cache overflow: {t} > {self.tcap}")
        bs = self.block_size
        tt = ops.num_blocks(t, bs) * bs
        b, _, h, d = xk.shape
        tmp_k = torch.zeros(b, h, tt, d, device=self.gpu_device, dtype=self.dtype)
        tmp_v = torch.zeros_like(tmp_k)
        self.proto_sum.zero_()
        ops.kv_append(xk.to(self.gpu_device), xv.to(self.gpu_device), tmp_k, tmp_v, self.proto_sum, 0, bs)
        self.host_k[:, :, :t].copy_(tmp_k[:, :, :t])
        self.host_v[:, :, :t].copy_(tmp_v[:, :, :t])
        curr = t // bs  # block the next token lands in
        if curr >= 1:
            self.slot_k[:, :, :bs].copy_(tmp_k[:, :, :bs])
            self.slot_v[:, :, :bs].copy_(tmp_v[:, :, :bs])
            self.slot_block[:, :, self.kslots] = 0
        n = t - curr * bs
        if n:
            self.slot_k[:, :, bs:bs + n].copy_(tmp_k[:, :, curr * bs:t])
            self.slot_v[:, :, bs:bs + n].copy_(tmp_v[:, :, curr * bs:t])
        torch.cuda.current_stream(self.gpu_device).synchronize()
        self.advance(t)
        return self.current_len

    def advance(self, t: int, device: bool = True) -> None:
        self.current_len += t
        if device:
            ops.advance_len(self.len_dev, t)

    def reset(self) -> None:
        self.current_len = 0
        self.len_dev.zero_()
        self.proto_sum.zero_()
        self.slot_block.fill_(-1)
        self.stats.zero_()
        self.prefetched = False
        self.total_transfer_calls = 0

    # -- transfers (reference API)
    def transfer_selected_blocks(self, block_indices: torch.Tensor, block_size: int, non_blocking: bool = True
                                 ) -> Tuple[torch.Tensor, torch.Tensor, int]:
        """offload.py:83-123: the listed blocks [B, H, S] gathered from the host
        store into device tensors [B, H, S*block_size, D]; the gather kernel
        reads the pinned rows directly, so indices stay on the device."""
        idx = block_indices.to(self.gpu_device)
        kh = self.host_k[:, :, :self.current_len]
        vh = self.host_v[:, :, :self.current_len]
        gk, gv = ops.gather_kv_blocks(kh, vh, idx, block_size, device=self.gpu_device)
        nbytes = (gk.numel() + gv.numel()) * gk.element_size()
        self.stats[2] += nbytes
        self.total_transfer_calls += 1
        return gk, gv, nbytes

    def async_transfer_selected_blocks(self, block_indices: torch.Tensor, block_size: int,
                                       stream: Optional[torch.cuda.Stream] = None):
        """async_offload.py:55-112: the same gather on the transfer stream;
        returns (gpu_k, gpu_v, event, bytes)."""
        s = stream or self.transfer_stream
        s.wait_stream(torch.cuda.current_stream(self.gpu_device))
        with torch.cuda.stream(s):
            gk, gv, nbytes = self.transfer_selected_blocks(block_indices, block_size)
            ev = torch.cuda.Event()
            ev.record(s)
        return gk, gv, ev, nbytes

    # -- forecast-guided prefetch
    def issue_prefetch(self, forecast: Optional[torch.Tensor], rule: str, top_k: int,
                       stream: Optional[torch.cuda.Stream] = None, timing_events=None) -> None:
        """For the next decode step: candidates from the forecast (if any) and
        the staging of the wanted blocks, on ``stream`` (default: the transfer
        stream, ordered after the current stream's work).  timing_events: an
        optional (start, end) pair of CUDA events recorded around that work."""
        s = stream or self.transfer_stream
        cur = torch.cuda.current_stream(self.gpu_device)
        if s is not cur:
            s.wait_stream(cur)
        with torch.cuda.stream(s):
            if timing_events is not None:
                timing_events[0].record(s)
            if forecast is not None:
                ops.decode_candidates(forecast, self.proto_sum, self.len_dev, self.n_kv_head, self.block_size, top_k,
                                      rule, out=self.cand)
                ops.offload_prefetch(self, self.cand[0])
            else:
                ops.offload_prefetch(self, None)
            if timing_events is not None:
                timing_events[1].record(s)
            self.prefetch_event.record(s)
        self.prefetched = True
        self.has_cand = forecast is not None
        self.total_transfer_calls += 1
