"""Drop-in attention backend (model/attention/base.py, model/attention/sparse.py)
whose hot path runs on the sm_100a kernels of libspardab200.so."""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .cache import B200KVCache
from .offload import B200OffloadKVCache
from .forecast import ForecastBlockSelector, KVBlockCompressor
from .rope import apply_rotary_emb


class _RopeQK(torch.autograd.Function):
    """RoPE of q and k (ops.rope_qk, model/rope.py:34-65) with its backward for
    training: the rotation's transpose is the rotation by the negated angle,
    i.e. the same kernel with -sin (sin is the same for both halves of a head,
    so rotate_half commutes with it)."""

    @staticmethod
    def forward(ctx, xq, xk, cos, sin):
        ctx.save_for_backward(cos, sin)
        ctx.shapes = (xq.shape, xk.shape)
        return ops.rope_qk(xq, xk, cos, sin, 0)

    @staticmethod
    def backward(ctx, gq, gk):
        cos, sin = ctx.saved_tensors
        if gq is None:
            gq = torch.zeros(ctx.shapes[0], dtype=gk.dtype, device=gk.device)
        if gk is None:
            gk = torch.zeros(ctx.shapes[1], dtype=gq.dtype, device=gq.device)
        dq, dk = ops.rope_qk(gq, gk, cos, -sin, 0)
        return dq, dk, None, None


class _SparseAttentionCore(torch.autograd.Function):
    """Block-sparse prefill attention (ops.prefill_attention) with its backward
    (ops.prefill_attention_backward, fp32) for training: the gradients autograd
    takes through the reference's masked / chunked SDPA (sparse.py:185-364).
    The block lists and per-row top-k are indices and carry no gradient, as in
    the reference, where only topk's indices build the mask."""

    @staticmethod
    def forward(ctx, q, k, v, lists, counts, topk, block_size, causal):
        ctx.save_for_backward(q, k, v, lists, counts, topk)
        ctx.block_size, ctx.causal = block_size, causal
        return ops.prefill_attention(q, k, v, lists, counts, block_size, topk, causal)

    @staticmethod
    def backward(ctx, gout):
        q, k, v, lists, counts, topk = ctx.saved_tensors
        dq, dk, dv = ops.prefill_attention_backward(q, k, v, gout, lists, counts, ctx.block_size, topk, ctx.causal)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None, None, None, None


class BaseAttention(nn.Module):
    """model/attention/base.py:35-52: owns wq, wk, wv, wo (same state-dict keys)."""

    def __init__(self, config, layer_idx: int):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.n_head = config.n_head
        self.n_kv_head = config.n_kv_head
        self.head_dim = config.head_dim
        self.n_embd = config.n_embd
        self.num_queries_per_kv = config.n_head // config.n_kv_head
        self.wq = nn.Linear(self.n_embd, self.n_head * self.head_dim, bias=False)
        self.wk = nn.Linear(self.n_embd, self.n_kv_head * self.head_dim, bias=False)
        self.wv = nn.Linear(self.n_embd, self.n_kv_head * self.head_dim, bias=False)
        self.wo = nn.Linear(self.n_head * self.head_dim, self.n_embd, bias=False)


class B200SparseAttention(BaseAttention):
    """Forecast-guided block-sparse GQA attention (SparseAttention,
    model/attention/sparse.py:65-439) on B200 kernels.

    Same constructor, state-dict keys and forward signature as the reference.
    Decode (T == 1 with a cache) on a B200KVCache runs one fused kernel per
    layer (RoPE + append + compressor update + selection + attention); any
    other cache object with the reference's ``update``/``current_len`` API runs
    the unfused kernels.  ``rule`` picks the decode-time causal rule of the
    selector (see ops.RULES); the default reproduces the reference.
    """

    def __init__(self, config, layer_idx: int, mode: Optional[str] = None, rule: Optional[str] = None,
                 selection_timing: Optional[str] = None):
        super().__init__(config, layer_idx)
        self.block_size = config.block_size
        self.top_k_blocks = config.top_k_blocks
        if mode is not None:
            self.mode = mode
        elif config.attention_backend in ("static_sparse", "static"):
            self.mode = "static"
        elif getattr(config, "sparse_mode", "forecast") == "static":
            self.mode = "static"
        else:
            self.mode = "forecast"
        self.rule = rule or getattr(config, "selector_rule", "reference")
        if self.rule not in ops.RULES:
            raise ValueError(f"unknown selector rule {self.rule!r}")
        self.selection_timing = selection_timing or getattr(config, "selection_timing", "after_append")
        if self.selection_timing not in ("after_append", "before_append"):
            raise ValueError(f"unknown selection timing {self.selection_timing!r}")
        self.compressor = KVBlockCompressor(self.block_size, self.head_dim, config.forecast_dim)
        self.selector = ForecastBlockSelector(self.block_size, config.forecast_dim)
        self._packed = None
        self._packed_key = None
        self.last_profile = {}

    @property
    def before_append(self) -> bool:
        return self.selection_timing == "before_append"

    # -- fused projection weight [wq; wk; wv], rebuilt when any weight changes
    def qkv_weight(self) -> torch.Tensor:
        key = tuple((w.data_ptr(), w._version, w.dtype) for w in (self.wq.weight, self.wk.weight, self.wv.weight))
        if self._packed is None or self._packed_key != key:
            with torch.no_grad():
                self._packed = torch.cat([self.wq.weight, self.wk.weight, self.wv.weight], dim=0).contiguous()
            self._packed_key = key
        return self._packed

    def forward(self, x: torch.Tensor, rotary_emb, kv_cache=None, mask: Optional[torch.Tensor] = None,
                is_causal: bool = True, forecast_vector: Optional[torch.Tensor] = None, **kwargs):
        if kwargs.get("return_attn_weights", False):
            raise NotImplementedError("return_attn_weights is a training/test feature of the reference backend")
        b, t, _ = x.shape
        if kv_cache is not None and t == 1:
            if isinstance(kv_cache, B200KVCache):
                return self._decode_fused(x, rotary_emb, kv_cache, forecast_vector)
            if isinstance(kv_cache, B200OffloadKVCache):
                return self._decode_offload(x, rotary_emb, kv_cache, forecast_vector)
            return self._decode_generic(x, rotary_emb, kv_cache, forecast_vector)
        return self._prefill(x, rotary_emb, kv_cache, mask, is_causal, forecast_vector, **kwargs)

    def _decode_fused(self, x, rotary_emb, cache: B200KVCache, forecast_vector):
        b = x.shape[0]
        if cache.current_len >= cache.tcap:
            raise ValueError(f"cache full: {cache.current_len} tokens of {cache.tcap}")
        if rotary_emb.cos.shape[0] < cache.tcap:
            rotary_emb._extend_cache(cache.tcap, x.device)
        qkv = F.linear(x.view(b, self.n_embd), self.qkv_weight())
        if qkv.dtype != cache.k_store.dtype:
            qkv = qkv.to(cache.k_store.dtype)
        f = forecast_vector if (self.mode == "forecast" and forecast_vector is not None) else None
        out = ops.decode_layer(qkv, f, rotary_emb.cos, rotary_emb.sin, cache.len_dev, cache.k_store,
                               cache.v_store, cache.proto_sum, self.n_head, self.n_kv_head, self.block_size,
                               self.top_k_blocks, self.rule, select_before_append=self.before_append)
        cache.advance(1, device=not getattr(cache, "shared_len", False))
        return self.wo(out.to(x.dtype)).view(b, 1, self.n_embd)

    # -- offloaded caches (model/attention/async_offload.py:170-519)
    def prefetch(self, forecast_vector: Optional[torch.Tensor], offload_cache, timing_events=None) -> bool:
        """Called by layer L with its forecast to stage layer L+1's blocks
        (this layer's) on the cache's transfer stream while layer L computes
        (async_offload.py:170-294).  Returns False when there is nothing to do."""
        if not isinstance(offload_cache, B200OffloadKVCache) or offload_cache.current_len == 0:
            return False
        f = forecast_vector if self.mode == "forecast" else None
        offload_cache.issue_prefetch(f, self.rule, self.top_k_blocks, timing_events=timing_events)
        return True

    def offload_ready(self, cache: B200OffloadKVCache, f: Optional[torch.Tensor]) -> None:
        """Orders the current stream after this step's prefetch, issuing it
        here (synchronously in stream order) when none is in flight or the one
        in flight was for the other selection mode (async_offload.py:392-460)."""
        cur = torch.cuda.current_stream(cache.gpu_device)
        if cache.prefetched:
            cur.wait_event(cache.prefetch_event)
            if cache.has_cand == (f is not None):
                return
        cache.issue_prefetch(f, self.rule, self.top_k_blocks, stream=cur)

    def _decode_offload(self, x, rotary_emb, cache: B200OffloadKVCache, forecast_vector):
        b = x.shape[0]
        if cache.current_len >= cache.tcap:
            raise ValueError(f"cache full: {cache.current_len} tokens of {cache.tcap}")
        if rotary_emb.cos.shape[0] < cache.tcap:
            rotary_emb._extend_cache(cache.tcap, x.device)
        qkv = F.linear(x.view(b, self.n_embd), self.qkv_weight())
        if qkv.dtype != cache.slot_k.dtype:
            qkv = qkv.to(cache.slot_k.dtype)
        f = forecast_vector if (self.mode == "forecast" and forecast_vector is not None) else None
        self.offload_ready(cache, f)
        out = ops.decode_layer_offload(qkv, f, rotary_emb.cos, rotary_emb.sin, cache, self.n_head, self.rule,
                                       cand=cache.cand if f is not None else None,
                                       select_before_append=self.before_append)
        cache.prefetched = False
        cache.advance(1, device=not getattr(cache, "shared_len", False))
        return self.wo(out.to(x.dtype)).view(b, 1, self.n_embd)

    def _decode_generic(self, x, rotary_emb, cache, forecast_vector):
        b = x.shape[0]
        xq = self.wq(x).view(b, 1, self.n_head, self.head_dim)
        xk = self.wk(x).view(b, 1, self.n_kv_head, self.head_dim)
        xv = self.wv(x).view(b, 1, self.n_kv_head, self.head_dim)
        xq, xk = rotary_emb(xq, xk, offset=cache.current_len)
        k_all, v_all = cache.update(xk, xv)
        seq_len_k = cache.current_len
        f = forecast_vector if (self.mode == "forecast" and forecast_vector is not None) else None
        reps = self.compressor(k_all) if f is not None else None
        sel, cnt = ops.decode_select(f, reps, seq_len_k, b, self.n_kv_head, self.head_dim, self.block_size,
                                     self.top_k_blocks, self.rule, device=x.device)
        out = ops.decode_attention(xq[:, 0], k_all.transpose(1, 2), v_all.transpose(1, 2), sel, cnt, seq_len_k,
                                   self.block_size)
        return self.wo(out.reshape(b, 1, self.n_head * self.head_dim).to(x.dtype))

    def _prefill(self, x, rotary_emb, kv_cache, mask, is_causal, forecast_vector, **kwargs):
        """Sequence prefill (sparse.py:412-439): the masked path for T <= 8192,
        the chunked path above (or when ``use_chunked_gather`` is passed)."""
        if mask is not None:
            raise NotImplementedError("explicit additive masks are not supported by the B200 backend")
        b, t, _ = x.shape
        xq = self.wq(x).view(b, t, self.n_head, self.head_dim)
        xk = self.wk(x).view(b, t, self.n_kv_head, self.head_dim)
        xv = self.wv(x).view(b, t, self.n_kv_head, self.head_dim)
        out = self.prefill_core(xq, xk, xv, rotary_emb, kv_cache, is_causal, forecast_vector, **kwargs)
        return self.wo(out.reshape(b, t, self.n_head * self.head_dim).to(x.dtype))

    def block_lists(self, xk: torch.Tensor, f: Optional[torch.Tensor], is_causal: bool, chunked: bool):
        """The prefill's key-block lists (sparse.py:185-364): compressor +
        selector on the RoPE'd keys xk [B,T,Hkv,D] and forecast f (or None),
        then the per-q-block lists of the masked path (dense, forecast or
        static window) or of the chunked path.  Returns (lists, counts,
        per-row top-k or None, causal) for ops.prefill_attention."""
        b, t = xk.shape[0], xk.shape[1]
        bs, kk = self.block_size, self.top_k_blocks
        nb = ops.num_blocks(t, bs)
        topk = None
        if chunked:
            causal = True  # the chunked path always clears future blocks (sparse.py:330-346)
            if f is not None:
                _, topk = ops.select_blocks(f, self.compressor(xk), kk, bs, False, return_scores=False)
                mode = "chunked_forecast"
            else:
                mode = "chunked_static"
            row_topk = None
        else:
            causal = is_causal
            if nb <= 2 or (self.mode == "forecast" and (f is None or self.layer_idx == 0)):
                mode = "dense"
            elif self.mode == "forecast":
                _, topk = ops.select_blocks(f, self.compressor(xk), kk, bs, is_causal, return_scores=False)
                mode = "masked_forecast"
            else:
                mode = "masked_static"
            row_topk = topk
        lists, counts = ops.prefill_lists(mode, b, self.n_kv_head, t, bs, kk, topk, causal, device=xk.device)
        return lists, counts, row_topk, causal

    def prefill_core(self, xq, xk, xv, rotary_emb, kv_cache, is_causal, forecast_vector, **kwargs):
        """Prefill from the q/k/v projections [B,T,H,D] (any strides with an
        innermost stride of 1, e.g. views of one packed projection): RoPE,
        cache write, compressor, selector, block lists and block-sparse
        attention.  Returns the attention output [B,T,Hq,D] before wo.

        While autograd records and q, k or v needs a gradient, RoPE and the
        attention core run as autograd functions with CUDA backward kernels
        (training without a cache, as the reference's trainer does)."""
        b, t = xq.shape[0], xq.shape[1]
        grad = torch.is_grad_enabled() and (xq.requires_grad or xk.requires_grad or xv.requires_grad)
        if grad and kv_cache is not None:
            raise NotImplementedError("gradients through a KV cache are not supported: train without a cache")
        offset = kv_cache.current_len if kv_cache is not None else 0
        if offset:
            # the reference uses seq_len for both queries and keys here
            # (sparse.py:413-430), so a prompt cannot extend a filled cache
            raise NotImplementedError("prefill into a non-empty cache")
        rotary_emb.ensure(t)
        if grad:
            xq, xk = _RopeQK.apply(xq, xk, rotary_emb.cos, rotary_emb.sin)
        else:
            xq, xk = ops.rope_qk(xq, xk, rotary_emb.cos, rotary_emb.sin, 0)
        if isinstance(kv_cache, B200OffloadKVCache):
            kv_cache.update(xk, xv)  # host store + block sums + slots; attend over the prompt itself
            kh, vh = xk.transpose(1, 2), xv.transpose(1, 2)
        elif kv_cache is not None:
            k_all, v_all = kv_cache.update(xk, xv)
            if isinstance(kv_cache, B200KVCache):
                kh, vh = kv_cache.k_store[:, :, :t], kv_cache.v_store[:, :, :t]
            else:
                kh, vh = k_all.transpose(1, 2), v_all.transpose(1, 2)
        else:
            kh, vh = xk.transpose(1, 2), xv.transpose(1, 2)
        f = forecast_vector if (self.mode == "forecast" and forecast_vector is not None) else None
        lists, counts, row_topk, causal = self.block_lists(
            xk.detach(), f.detach() if f is not None else None, is_causal,
            kwargs.get("use_chunked_gather", t > 8192))
        if grad:
            return _SparseAttentionCore.apply(xq, kh, vh, lists, counts, row_topk, self.block_size, causal)
        return ops.prefill_attention(xq, kh, vh, lists, counts, self.block_size, row_topk, causal)
