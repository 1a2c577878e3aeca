"""SparDA model driver on the B200 attention backend.

The caller side of the hot path: SparDAResearchModel (model/model.py:14-191)
and TransformerBlock (model/transformer.py:54-131) with the reference's module
tree and state-dict keys, so reference checkpoints load unchanged, wired to
B200SparseAttention.  Embedding, RMSNorm, SwiGLU and the tied head stay on
PyTorch/cuBLAS.  ``DecodeEngine`` captures a whole greedy decode step (all
layers, LM head and argmax) in one CUDA graph.
"""

from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .attention import B200SparseAttention
from .cache import B200KVCache
from .offload import B200OffloadKVCache
from .config import ModelConfig
from .forecast import ForecastProjection
from .rope import RotaryEmbedding


def _records_grad(x: torch.Tensor, module: nn.Module) -> bool:
    """Whether autograd is recording a graph that needs the gradient of x or of
    one of the module's parameters.  The packed projections and the RMSNorm /
    SwiGLU kernels have no backward, so such calls take the layer-by-layer
    path, whose attention core has CUDA backward kernels."""
    return torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in module.parameters()))


class RMSNorm(nn.Module):
    """model/norm.py:7-21."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        # the library's kernel has no backward: while autograd records a graph
        # that needs x's or the gain's gradient, the differentiable formula runs
        if x.is_cuda and x.dtype == self.weight.dtype and not _records_grad(x, self):
            c = x.shape[-1]
            return ops.rmsnorm(x.reshape(-1, c), self.weight, self.eps).view(x.shape)
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).type_as(x) * self.weight


class TiedEmbedding(nn.Module):
    """model/embeddings.py:8-32."""

    def __init__(self, vocab_size: int, n_embd: int, initializer_range: float = 0.02):
        super().__init__()
        self.vocab_size = vocab_size
        self.n_embd = n_embd
        self.weight = nn.Parameter(torch.empty(vocab_size, n_embd))
        nn.init.normal_(self.weight, mean=0.0, std=initializer_range)

    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        return F.embedding(ids, self.weight)

    def project(self, h: torch.Tensor) -> torch.Tensor:
        return F.linear(h, self.weight)


class SwiGLU(nn.Module):
    """model/transformer.py:18-31."""

    def __init__(self, n_embd: int, ffn_dim: int):
        super().__init__()
        self.w_gate = nn.Linear(n_embd, ffn_dim, bias=False)
        self.w_up = nn.Linear(n_embd, ffn_dim, bias=False)
        self.w_down = nn.Linear(ffn_dim, n_embd, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.w_down(F.silu(self.w_gate(x)) * self.w_up(x))


class TransformerBlock(nn.Module):
    """model/transformer.py:54-131 with the B200 attention backend.

    Decode on a B200KVCache uses one GEMM for [wq; wk; wv; wf] (the forecast
    of layer L is computed from the same normalised input as L's q/k/v,
    transformer.py:104-107) followed by the fused decode kernel."""

    def __init__(self, config: ModelConfig, layer_idx: int):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.attn_norm = RMSNorm(config.n_embd, eps=config.norm_eps)
        self.attention = B200SparseAttention(config, layer_idx)
        self.forecast = ForecastProjection(config)
        self.ffn_norm = RMSNorm(config.n_embd, eps=config.norm_eps)
        self.ffn = SwiGLU(config.n_embd, config.ffn_dim)
        self._packed = None
        self._packed_key = None
        # optional instrumentation of the fused decode kernel: {"start", "end"}
        # timing events (external=True so they survive graph capture) and
        # {"sel", "cnt"} buffers receiving the selected block lists
        self.probe = None

    def packed_weight(self) -> torch.Tensor:
        ws = (self.attention.wq.weight, self.attention.wk.weight, self.attention.wv.weight, self.forecast.wf.weight)
        key = tuple((w.data_ptr(), w._version, w.dtype) for w in ws)
        if self._packed is None or self._packed_key != key:
            with torch.no_grad():
                self._packed = torch.cat(ws, dim=0).contiguous()
            self._packed_key = key
        return self._packed

    def packed_ffn_weight(self) -> torch.Tensor:
        ws = (self.ffn.w_gate.weight, self.ffn.w_up.weight)
        key = tuple((w.data_ptr(), w._version, w.dtype) for w in ws)
        if getattr(self, "_ffn_packed", None) is None or self._ffn_key != key:
            with torch.no_grad():
                self._ffn_packed = torch.cat(ws, dim=0).contiguous()
            self._ffn_key = key
        return self._ffn_packed

    def swiglu_weight(self) -> torch.Tensor:
        """[w_gate; w_up] interleaved in 64-row groups for the fused SwiGLU
        epilogue, rebuilt when either weight changes."""
        ws = (self.ffn.w_gate.weight, self.ffn.w_up.weight)
        key = tuple((w.data_ptr(), w._version, w.dtype) for w in ws)
        if getattr(self, "_swiglu_w", None) is None or self._swiglu_key != key:
            with torch.no_grad():
                self._swiglu_w = ops.swiglu_weight(*ws)
            self._swiglu_key = key
        return self._swiglu_w

    def tc_projections(self, x2: torch.Tensor) -> bool:
        """Whether the decode step's projections run on this library's fused
        tensor-core kernel (sd_linear): opt-in (`use_tc_linear = True`), for
        16-bit activations and weights with widths that tile by 64 x 128.  The
        default is cuBLAS with the library's RMSNorm and SwiGLU kernels, which
        measured faster for the 64-row decode batch."""
        cfg = self.config
        return (getattr(self, "use_tc_linear", False) and x2.is_cuda and x2.dtype in (torch.bfloat16, torch.float16)
                and self.attn_norm.weight.dtype == x2.dtype and x2.stride(-1) == 1 and cfg.n_embd % 128 == 0
                and cfg.ffn_dim % 64 == 0 and cfg.n_embd <= 1024)

    def _ffn_decode(self, x2: torch.Tensor, attn_out: torch.Tensor, tc: bool) -> torch.Tensor:
        """x + wo(attn); then h + w_down(silu(w_gate(n)) * w_up(n)) with n =
        ffn_norm(h) (transformer.py:118-129)."""
        a = self.attention
        if tc:
            h = ops.linear(attn_out, a.wo.weight, epilogue="residual", res=x2)
            g = ops.linear(h, self.swiglu_weight(), self.ffn_norm.weight, self.ffn_norm.eps, epilogue="swiglu")
            return ops.linear(g, self.ffn.w_down.weight, epilogue="residual", res=h, out=h)
        x2 = torch.addmm(x2, attn_out, a.wo.weight.t())
        gu = F.linear(self.ffn_norm(x2), self.packed_ffn_weight())
        return torch.addmm(x2, ops.silu_mul(gu), self.ffn.w_down.weight.t())

    def forward(self, x, rotary_emb, kv_cache=None, mask=None, is_causal=True, prev_layer_forecast=None,
                next_layer_block=None, next_kv_cache=None):
        b, t, c = x.shape
        if isinstance(kv_cache, (B200KVCache, B200OffloadKVCache)) and t == 1:
            # decode step: 8 launches per layer by default (norm, [wq;wk;wv;wf]
            # GEMM, fused attention kernel, wo GEMM with the residual add folded
            # into addmm, norm, [w_gate;w_up] GEMM, SwiGLU gate kernel, w_down
            # addmm); with use_tc_linear 5, all of this library (RMSNorm +
            # [wq;wk;wv;wf], attention, wo + residual, RMSNorm + [w_gate;w_up] +
            # SwiGLU gate, w_down + residual).
            a = self.attention
            x2 = x.view(b, c)
            tc = self.tc_projections(x2)
            if tc:
                proj = ops.linear(x2, self.packed_weight(), self.attn_norm.weight, self.attn_norm.eps)
            else:
                proj = F.linear(self.attn_norm(x2), self.packed_weight())
            nq = (a.n_head + 2 * a.n_kv_head) * a.head_dim
            current_forecast = proj[:, nq:].view(b, 1, self.config.forecast_heads, self.config.forecast_dim)
            if kv_cache.current_len >= kv_cache.tcap:
                raise ValueError(f"cache full: {kv_cache.current_len} tokens of {kv_cache.tcap}")
            if rotary_emb.cos.shape[0] < kv_cache.tcap:
                rotary_emb._extend_cache(kv_cache.tcap, x.device)
            f = prev_layer_forecast if (a.mode == "forecast" and prev_layer_forecast is not None) else None
            probe = self.probe
            # the next layer's forecast candidates only need this layer's forecast
            # and the next layer's (unchanged until its own step) running sums:
            # compute them on the side stream while this layer's attention and
            # FFN run on the main stream
            side = getattr(self, "side_stream", None)
            next_cand = None
            if getattr(self, "chain_next", False) and next_layer_block is not None \
                    and isinstance(next_kv_cache, B200KVCache) and isinstance(kv_cache, B200KVCache) \
                    and next_layer_block.attention.mode == "forecast" \
                    and next_layer_block.attention.rule == a.rule \
                    and next_layer_block.attention.top_k_blocks == a.top_k_blocks \
                    and a.top_k_blocks <= 32 \
                    and next_layer_block.attention.block_size == a.block_size \
                    and next_kv_cache.proto_sum.shape == kv_cache.proto_sum.shape:
                # this layer's kernel ends by computing the next layer's
                # candidates: no side stream, no extra launch
                nc = next_kv_cache
                if getattr(nc, "cand", None) is None:
                    nc.cand = (torch.empty(b, a.n_kv_head, a.top_k_blocks, dtype=torch.int32, device=x.device),
                               torch.empty(b, a.n_kv_head, a.top_k_blocks, dtype=torch.float32, device=x.device))
                next_cand = (nc.proto_sum, proj[:, nq:], nc.cand)
                nc.cand_ready = True
                nc.cand_event = None
            elif next_layer_block is not None and isinstance(next_kv_cache, B200OffloadKVCache):
                # offloaded next layer: candidates + host -> device staging of
                # its blocks on the transfer stream (transformer.py:110-115)
                ev = (probe["cstart"], probe["cend"]) if probe is not None and "cstart" in probe else None
                next_layer_block.attention.prefetch(current_forecast, next_kv_cache, timing_events=ev)
            elif side is not None and next_layer_block is not None and isinstance(next_kv_cache, B200KVCache) \
                    and next_layer_block.attention.mode == "forecast":
                na = next_layer_block.attention
                nc = next_kv_cache
                if getattr(nc, "cand", None) is None:
                    nc.cand = (torch.empty(b, na.n_kv_head, na.top_k_blocks, dtype=torch.int32, device=x.device),
                               torch.empty(b, na.n_kv_head, na.top_k_blocks, dtype=torch.float32, device=x.device))
                    nc.cand_event = torch.cuda.Event()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    if probe is not None and "cstart" in probe:
                        probe["cstart"].record(side)
                    ops.decode_candidates(current_forecast, nc.proto_sum, nc.len_dev, na.n_kv_head, na.block_size,
                                          na.top_k_blocks, na.rule, out=nc.cand)
                    if probe is not None and "cend" in probe:
                        probe["cend"].record(side)
                    nc.cand_event.record(side)
                nc.cand_ready = True
            if isinstance(kv_cache, B200OffloadKVCache):
                if probe is not None and "wstart" in probe:
                    probe["wstart"].record()
                a.offload_ready(kv_cache, f)
                if probe is not None and "wend" in probe:
                    probe["wend"].record()
                if probe is not None:
                    probe["start"].record()
                out = ops.decode_layer_offload(proj[:, :nq], f, rotary_emb.cos, rotary_emb.sin, kv_cache, a.n_head,
                                               a.rule, sel_out=probe["sel"] if probe is not None else None,
                                               cnt_out=probe["cnt"] if probe is not None else None,
                                               cand=kv_cache.cand if f is not None else None,
                                               select_before_append=a.before_append)
                if probe is not None:
                    probe["end"].record()
                kv_cache.prefetched = False
                kv_cache.advance(1, device=not getattr(kv_cache, "shared_len", False))
                return self._ffn_decode(x2, out, tc).view(b, 1, c), current_forecast
            cand = None
            if getattr(kv_cache, "cand_ready", False):
                if kv_cache.cand_event is not None:
                    torch.cuda.current_stream().wait_event(kv_cache.cand_event)  # join the side stream
                cand = kv_cache.cand if f is not None else None
            kv_cache.cand_ready = False
            if probe is not None:
                probe["start"].record()
            out = ops.decode_layer(proj[:, :nq], f, rotary_emb.cos, rotary_emb.sin, kv_cache.len_dev,
                                   kv_cache.k_store, kv_cache.v_store, kv_cache.proto_sum, a.n_head, a.n_kv_head,
                                   a.block_size, a.top_k_blocks, a.rule,
                                   sel_out=probe["sel"] if probe is not None else None,
                                   cnt_out=probe["cnt"] if probe is not None else None, cand=cand,
                                   next_cand=next_cand, select_before_append=a.before_append)
            if probe is not None:
                probe["end"].record()
            kv_cache.advance(1, device=not getattr(kv_cache, "shared_len", False))
            return self._ffn_decode(x2, out, tc).view(b, 1, c), current_forecast
        elif x.is_cuda and mask is None and isinstance(self.attention, B200SparseAttention) \
                and not _records_grad(x, self):
            # prompt: one GEMM for [wq; wk; wv; wf], the attention core on views
            # of it, the residual adds folded into addmm, and the SwiGLU gate
            # on one [w_gate; w_up] GEMM (transformer.py:76-131 in 6 launches
            # around the attention core instead of 12)
            a = self.attention
            x2 = x.reshape(b * t, c)
            normed = self.attn_norm(x2)
            proj = F.linear(normed, self.packed_weight())
            nq, nk = a.n_head * a.head_dim, a.n_kv_head * a.head_dim
            current_forecast = proj[:, nq + 2 * nk:].view(b, t, self.config.forecast_heads,
                                                          self.config.forecast_dim)
            if next_layer_block is not None and next_kv_cache is not None and \
                    hasattr(next_layer_block.attention, "prefetch"):
                next_layer_block.attention.prefetch(forecast_vector=current_forecast, offload_cache=next_kv_cache)
            p3 = proj.view(b, t, -1)
            out = a.prefill_core(p3[..., :nq].unflatten(-1, (a.n_head, a.head_dim)),
                                 p3[..., nq:nq + nk].unflatten(-1, (a.n_kv_head, a.head_dim)),
                                 p3[..., nq + nk:nq + 2 * nk].unflatten(-1, (a.n_kv_head, a.head_dim)),
                                 rotary_emb, kv_cache, is_causal, prev_layer_forecast)
            x2 = torch.addmm(x2, out.reshape(b * t, nq).to(x2.dtype), a.wo.weight.t())
            gu = F.linear(self.ffn_norm(x2), self.packed_ffn_weight())
            x2 = torch.addmm(x2, ops.silu_mul(gu), self.ffn.w_down.weight.t())
            return x2.view(b, t, c), current_forecast
        else:
            normed = self.attn_norm(x)
            current_forecast = self.forecast(normed)
            if next_layer_block is not None and next_kv_cache is not None and \
                    hasattr(next_layer_block.attention, "prefetch"):
                next_layer_block.attention.prefetch(forecast_vector=current_forecast, offload_cache=next_kv_cache)
            x = x + self.attention(normed, rotary_emb=rotary_emb, kv_cache=kv_cache, mask=mask,
                                   is_causal=is_causal, forecast_vector=prev_layer_forecast)
        x = x + self.ffn(self.ffn_norm(x))
        return x, current_forecast


class SparDAB200Model(nn.Module):
    """model/model.py:14-157 with B200 attention."""

    def __init__(self, config: ModelConfig):
        super().__init__()
        self.config = config
        self.embeddings = TiedEmbedding(config.vocab_size, config.n_embd, config.initializer_range)
        self.rotary_emb = RotaryEmbedding(config.head_dim, config.context_length, config.rope_theta)
        self.layers = nn.ModuleList([TransformerBlock(config, i) for i in range(config.n_layer)])
        self.final_norm = RMSNorm(config.n_embd, eps=config.norm_eps)
        self.apply(self._init_weights)
        self._lens: Optional[torch.Tensor] = None

    def _init_weights(self, module: nn.Module):
        if isinstance(module, nn.Linear):
            nn.init.normal_(module.weight, mean=0.0, std=self.config.initializer_range)
        elif isinstance(module, nn.Embedding):
            nn.init.normal_(module.weight, mean=0.0, std=self.config.initializer_range)

    def allocate_caches(self, batch: int, max_seq_len: int, dtype: Optional[torch.dtype] = None,
                        device=None, overlap_selection: bool = True, offload: bool = False,
                        selection: Optional[str] = None, cache_blocks: Optional[int] = None) -> List:
        """One cache per layer, sharing one device length array so a decode
        step bumps all lengths with a single launch.  With
        ``overlap_selection`` layer L+1's candidates for each decode step are
        computed ahead of its kernel (by default at the end of layer L's fused
        kernel).  With ``offload``
        the K/V rows live in pinned host memory (B200OffloadKVCache) and the
        side stream also stages layer L+1's selected blocks into device slots.
        ``selection`` overrides ``overlap_selection``: "kernel" (each fused
        kernel scores its own blocks), "side-stream" (layer L+1's candidates on
        a side stream during layer L) or "chain" (layer L's fused kernel ends
        by computing layer L+1's candidates).  ``cache_blocks`` (offload only):
        device slots per (sequence, kv head) for selected blocks, top_k..32;
        more than top_k keep blocks resident across steps with
        least-recently-used replacement."""
        if selection is None:
            selection = "chain" if overlap_selection else "kernel"
        if selection not in ("kernel", "side-stream", "chain"):
            raise ValueError(f"unknown selection mode {selection!r}")
        cfg = self.config
        device = device or self.embeddings.weight.device
        dtype = dtype or self.embeddings.weight.dtype
        self._lens = torch.zeros(cfg.n_layer, dtype=torch.int32, device=device)
        caches = []
        side = torch.cuda.Stream(device=device) if torch.device(device).type == "cuda" else None
        for i in range(cfg.n_layer):
            if offload:
                c = B200OffloadKVCache(batch, max_seq_len, cfg.n_kv_head, cfg.head_dim, device, dtype,
                                       transfer_stream=side, block_size=cfg.block_size, top_k=cfg.top_k_blocks,
                                       len_dev=self._lens[i:i + 1], cache_blocks=cache_blocks)
            else:
                c = B200KVCache(batch, max_seq_len, cfg.n_kv_head, cfg.head_dim, device, dtype, cfg.block_size,
                                len_dev=self._lens[i:i + 1])
            c.shared_len = True
            caches.append(c)
        self.rotary_emb._extend_cache(caches[0].tcap, device)
        for layer in self.layers:
            layer.chain_next = selection == "chain" and not offload
            layer.side_stream = None
        if (selection == "side-stream" or offload) and side is not None:
            for layer in self.layers:
                layer.side_stream = side
        return caches

    def forward(self, input_ids: torch.Tensor, targets: Optional[torch.Tensor] = None,
                kv_caches: Optional[List] = None, return_forecasts: bool = False) -> Dict[str, torch.Tensor]:
        b, t = input_ids.shape
        x = self.embeddings.embed(input_ids)
        forecasts = []
        prev = None
        for i, layer in enumerate(self.layers):
            cache = kv_caches[i] if kv_caches is not None else None
            nxt = self.layers[i + 1] if i + 1 < len(self.layers) else None
            ncache = kv_caches[i + 1] if (kv_caches is not None and i + 1 < len(kv_caches)) else None
            x, cur = layer(x=x, rotary_emb=self.rotary_emb, kv_cache=cache, mask=None, is_causal=True,
                           prev_layer_forecast=prev, next_layer_block=nxt, next_kv_cache=ncache)
            if return_forecasts:
                forecasts.append(cur)
            prev = cur
        if kv_caches is not None and t == 1 and getattr(kv_caches[0], "shared_len", False) and \
                kv_caches[0].len_dev.data_ptr() == self._lens.data_ptr():
            ops.advance_len(self._lens, 1)
        if t == 1 and kv_caches is not None and self.layers[-1].tc_projections(x.view(b, -1)) \
                and self.config.vocab_size % 128 == 0:
            # final RMSNorm + tied LM head in one tensor-core launch (model.py:141-142)
            logits = ops.linear(x.view(b, -1), self.embeddings.weight, self.final_norm.weight,
                                self.final_norm.eps).view(b, 1, -1)
        else:
            logits = self.embeddings.project(self.final_norm(x))
        out = {"logits": logits}
        if return_forecasts:
            out["forecasts"] = forecasts
        if targets is not None:
            out["loss"] = F.cross_entropy(logits.view(-1, self.config.vocab_size), targets.view(-1),
                                          ignore_index=-100)
        return out


class DecodeEngine:
    """Greedy decode step of a SparDAB200Model captured in one CUDA graph.

    ``ids`` (device, [B,1] int64) feeds the step; the graph writes the argmax
    tokens to ``next_ids`` and copies them into ``ids`` so replays chain.
    Cache lengths live on the device; the engine keeps the host copies in step.
    """

    def __init__(self, model: SparDAB200Model, caches: List[B200KVCache], batch: int):
        self.model, self.caches, self.batch = model, caches, batch
        dev = model.embeddings.weight.device
        self.ids = torch.zeros(batch, 1, dtype=torch.long, device=dev)
        self.next_ids = torch.zeros(batch, 1, dtype=torch.long, device=dev)
        self.graph = None

    def _body(self):
        out = self.model(self.ids, kv_caches=self.caches)
        ops.argmax_rows(out["logits"][:, -1, :], out=self.next_ids)
        self.ids.copy_(self.next_ids)

    def _snapshot(self):
        bs = self.caches[0].block_size
        j = self.caches[0].current_len // bs
        return [c.proto_sum[:, :, j].clone() for c in self.caches], j

    def _restore(self, snap):
        rows, j = snap
        for c, r in zip(self.caches, rows):
            c.proto_sum[:, :, j].copy_(r)
            c.current_len -= 1
        self.model._lens.sub_(1)

    @torch.no_grad()
    def capture(self) -> None:
        """Warm-up (whose cache writes are rolled back) and graph capture."""
        snap = self._snapshot()
        saved = self.ids.clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._body()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self._restore(snap)
        self.ids.copy_(saved)
        self.graph = torch.cuda.CUDAGraph()
        host_lens = [c.current_len for c in self.caches]
        with torch.cuda.graph(self.graph):
            self._body()
        for c, n in zip(self.caches, host_lens):  # capture ran no kernels
            c.current_len = n
        torch.cuda.synchronize()

    def step(self) -> torch.Tensor:
        self.graph.replay()
        for c in self.caches:
            c.current_len += 1
        return self.next_ids
