"""Torch-tensor wrappers over the C ABI.  Every op requires CUDA tensors: there
is no CPU path.  Each wrapper validates shapes, allocates its outputs with the
caching allocator and launches on the current CUDA stream."""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch

from . import _lib as L

_DT = {torch.float32: L.SD_DTYPE_F32, torch.bfloat16: L.SD_DTYPE_BF16, torch.float16: L.SD_DTYPE_F16}
RULES = {"reference": L.SD_RULE_REFERENCE, "absolute": L.SD_RULE_ABSOLUTE}

_err_bufs = {}


def rule_code(rule: str, select_before_append: bool = False) -> int:
    """SD_RULE_* of a rule name, with SD_SELECT_BEFORE_APPEND or-ed in on request."""
    try:
        code = RULES[rule]
    except KeyError:
        raise ValueError(f"unknown selector rule {rule!r}") from None
    return code | (L.SD_SELECT_BEFORE_APPEND if select_before_append else 0)


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32, bfloat16 or float16") from None


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("the B200 kernels need CUDA tensors (this library has no CPU path)")


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _inner1(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def error_buffer(device) -> torch.Tensor:
    """Per-device int32 word the kernels set when a bounded wait expires."""
    device = torch.device(device)
    key = device.index if device.index is not None else torch.cuda.current_device()
    buf = _err_bufs.get(key)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", key))
        _err_bufs[key] = buf
    return buf


def check_device_errors(device=None) -> None:
    """Synchronises and raises if any kernel reported a device-side timeout."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    buf = error_buffer(device)
    if int(buf.item()) != 0:
        code = int(buf.item())
        buf.zero_()
        raise L.SparDAError(f"a kernel gave up a bounded wait (device error code {code})")


def num_blocks(t: int, bs: int) -> int:
    return (t + bs - 1) // bs


# ---------------------------------------------------------------- K1 compressor
def compress_blocks(k: torch.Tensor, block_size: int) -> torch.Tensor:
    """KVBlockCompressor.forward (model/forecast.py:57-78): k [B,T,H,D] ->
    fp32 prototypes [B,N_b,H,D] (zero-padded block sum / block_size)."""
    _cuda(k)
    k = _inner1(k)
    b, t, h, d = k.shape
    reps = torch.empty(b, num_blocks(t, block_size), h, d, dtype=torch.float32, device=k.device)
    L.call("sd_compress_blocks", k.data_ptr(), dtype_code(k), b, t, h, d, k.stride(0), k.stride(1), k.stride(2),
           block_size, reps.data_ptr(), _stream(k))
    return reps


# ---------------------------------------------------------------- K2 selector
def select_blocks(forecast: torch.Tensor, reps: torch.Tensor, top_k: int, block_size: int,
                  is_causal: bool = True, q_offset: int = 0,
                  return_scores: bool = True) -> Tuple[Optional[torch.Tensor], torch.Tensor]:
    """ForecastBlockSelector.forward (model/forecast.py:89-130) in fp32.
    forecast [B,Tq,H,D], reps [B,N_b,H,D] -> (scores [B,H,Tq,N_b] fp32, idx [B,H,Tq,k] int64)."""
    _cuda(forecast, reps)
    b, tq, h, d = forecast.shape
    if reps.shape[0] != b or reps.shape[2] != h or reps.shape[3] != d:
        raise AssertionError(f"Mismatch: forecast_heads ({h}) != n_kv_head ({reps.shape[2]})")
    forecast = _inner1(forecast)
    reps = _inner1(reps.float())
    nb = reps.shape[1]
    k = min(top_k, nb)
    scores = torch.empty(b, h, tq, nb, dtype=torch.float32, device=forecast.device) if return_scores else None
    idx = torch.empty(b, h, tq, k, dtype=torch.int64, device=forecast.device)
    L.call("sd_select_blocks", forecast.data_ptr(), dtype_code(forecast), b, tq, h, d, forecast.stride(0),
           forecast.stride(1), forecast.stride(2), reps.data_ptr(), nb, reps.stride(0), reps.stride(1),
           reps.stride(2), top_k, block_size, int(bool(is_causal)), int(q_offset),
           scores.data_ptr() if scores is not None else None, idx.data_ptr(), _stream(forecast))
    return scores, idx


def topk_rows(scores: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """torch.topk(scores, k, dim=-1) (largest, sorted) with ties in ascending index order."""
    _cuda(scores)
    s = _inner1(scores.float())
    n = s.shape[-1]
    flat = s.reshape(-1, n)
    idx = torch.empty(flat.shape[0], k, dtype=torch.int64, device=s.device)
    vals = torch.empty(flat.shape[0], k, dtype=torch.float32, device=s.device)
    L.call("sd_topk_rows", flat.data_ptr(), flat.shape[0], n, flat.stride(0), k, idx.data_ptr(), vals.data_ptr(),
           _stream(s))
    return vals.view(*s.shape[:-1], k), idx.view(*s.shape[:-1], k)


# ---------------------------------------------------------------- K4 gather
def gather_kv_blocks(k: torch.Tensor, v: torch.Tensor, block_indices: torch.Tensor,
                     block_size: int, device: Optional[torch.device] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """gather_kv_blocks (model/attention/sparse.py:19-62): k, v [B,H,T,D],
    indices [B,H,S] -> [B,H,S*block_size,D].  k and v may also be pinned host
    tensors (an offloaded cache): the kernel on ``device`` then reads the
    selected rows straight from host memory."""
    if k.dim() != 4 or tuple(k.shape) != tuple(v.shape) or block_indices.dim() != 3 \
            or tuple(block_indices.shape[:2]) != tuple(k.shape[:2]):
        raise ValueError(f"k, v must be [B, H, T, D] alike and the indices [B, H, S], got {tuple(k.shape)}, "
                         f"{tuple(v.shape)}, {tuple(block_indices.shape)}")
    if not k.is_cuda or not v.is_cuda:
        if not (k.is_pinned() and v.is_pinned()) or device is None:
            raise ValueError("host K/V must be pinned, and the gather needs a target device")
        if k.stride() != v.stride() or k.dtype != v.dtype or k.stride(-1) != 1:
            raise ValueError("pinned host K/V must share dtype and strides, innermost stride 1")
        _cuda(block_indices)
        out_dev = torch.device(device)
    else:
        _cuda(block_indices)
        if k.stride() != v.stride() or k.dtype != v.dtype:
            k, v = k.contiguous(), v.contiguous()
        k, v = _inner1(k), _inner1(v)
        if k.stride() != v.stride():
            k, v = k.contiguous(), v.contiguous()
        out_dev = k.device
    b, h, t, d = k.shape
    idx = block_indices.to(torch.int64).contiguous()
    s = idx.shape[-1]
    ko = torch.empty(b, h, s * block_size, d, dtype=k.dtype, device=out_dev)
    vo = torch.empty_like(ko)
    L.call("sd_gather_kv_blocks", k.data_ptr(), v.data_ptr(), dtype_code(k), b, h, t, d, k.stride(0), k.stride(1),
           k.stride(2), idx.data_ptr(), s, block_size, ko.data_ptr(), vo.data_ptr(),
           torch.cuda.current_stream(out_dev).cuda_stream)
    return ko, vo


# ---------------------------------------------------------------- K3 + K7 decode
def decode_select(forecast: Optional[torch.Tensor], reps: Optional[torch.Tensor], seq_len_k: int, batch: int,
                  n_kv_head: int, head_dim: int, block_size: int, top_k: int,
                  rule: str = "reference", device=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Selected-block list of a decode step (model/attention/sparse.py:108-154).
    forecast [B,1,H,D] or [B,H,D] (or None: static window); reps [B,N_b,H,D] fp32.
    Returns sel int32 [B,H,MS] (ascending, -1 padded) and cnt int32 [B,H]."""
    nb = num_blocks(seq_len_k, block_size)
    ms = min(nb, top_k + 2)
    if forecast is not None:
        if reps is None or reps.dim() != 4 or reps.shape[0] < batch or reps.shape[1] < nb \
                or tuple(reps.shape[2:]) != (n_kv_head, head_dim) or forecast.numel() != batch * n_kv_head * head_dim:
            raise ValueError(f"forecast must hold [{batch}, {n_kv_head}, {head_dim}] and reps be "
                             f"[>={batch}, >={nb}, {n_kv_head}, {head_dim}], got "
                             f"{tuple(forecast.shape)} and {None if reps is None else tuple(reps.shape)}")
    dev = forecast.device if forecast is not None else (reps.device if reps is not None else device)
    _cuda(forecast, reps)
    sel = torch.empty(batch, n_kv_head, ms, dtype=torch.int32, device=dev)
    cnt = torch.empty(batch, n_kv_head, dtype=torch.int32, device=dev)
    if forecast is not None:
        f = _inner1(forecast.reshape(batch, n_kv_head, head_dim) if forecast.dim() == 4 else forecast)
        r = _inner1(reps.float())
        fargs = (f.data_ptr(), dtype_code(f), f.stride(0), f.stride(1))
        rargs = (r.data_ptr(), r.stride(0), r.stride(1), r.stride(2))
    else:
        fargs = (None, L.SD_DTYPE_F32, 0, 0)
        rargs = (None, 0, 0, 0)
    L.call("sd_decode_select", *fargs, *rargs, batch, n_kv_head, head_dim, seq_len_k, block_size, top_k,
           RULES[rule], sel.data_ptr(), cnt.data_ptr(), ms, torch.cuda.current_stream(dev).cuda_stream)
    return sel, cnt


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, sel: torch.Tensor,
                     cnt: torch.Tensor, seq_len_k: int, block_size: int,
                     scale: Optional[float] = None) -> torch.Tensor:
    """Block-sparse GQA decode attention (model/attention/sparse.py:156-181).
    q [B,Hq,D]; caches [B,Hkv,Tcap,D] views (any strides with inner 1, same for K
    and V); sel/cnt from decode_select.  Returns [B,Hq,D] in q's dtype."""
    if q.dim() != 3 or k_cache.dim() != 4 or tuple(k_cache.shape) != tuple(v_cache.shape):
        raise ValueError(f"q must be [B, Hq, D] and the caches [B, Hkv, Tcap, D] alike, got {tuple(q.shape)}, "
                         f"{tuple(k_cache.shape)}, {tuple(v_cache.shape)}")
    b, hq, d = q.shape
    hkv, tcap = k_cache.shape[1], k_cache.shape[2]
    if k_cache.shape[0] < b or k_cache.shape[3] != d or hq % hkv or not 0 < seq_len_k <= tcap:
        raise ValueError(f"caches {tuple(k_cache.shape)} do not fit q {tuple(q.shape)} at length {seq_len_k}")
    if sel.dim() != 3 or tuple(sel.shape[:2]) != (b, hkv) or tuple(cnt.shape) != (b, hkv):
        raise ValueError(f"sel must be [{b}, {hkv}, ms] and cnt [{b}, {hkv}], got {tuple(sel.shape)}, "
                         f"{tuple(cnt.shape)}")
    _cuda(q, k_cache, v_cache, sel, cnt)
    if k_cache.stride() != v_cache.stride():
        raise ValueError("K and V caches must share strides")
    q = _inner1(q)
    if q.dtype != k_cache.dtype:
        q = q.to(k_cache.dtype)
    sel = sel.to(torch.int32).contiguous()
    cnt = cnt.to(torch.int32).contiguous()
    out = torch.empty(b, hq, d, dtype=k_cache.dtype, device=q.device)
    sc = 1.0 / math.sqrt(d) if scale is None else scale
    L.call("sd_decode_attention", q.data_ptr(), dtype_code(k_cache), b, hq, hkv, d, q.stride(0), q.stride(1),
           k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), tcap,
           sel.data_ptr(), cnt.data_ptr(), sel.shape[-1], seq_len_k, block_size, sc, out.data_ptr(), out.stride(0),
           out.stride(1), error_buffer(q.device).data_ptr(), _stream(q))
    return out


def kv_append(xk: torch.Tensor, xv: torch.Tensor, k_store: torch.Tensor, v_store: torch.Tensor,
              proto_sum: torch.Tensor, start: int, block_size: int) -> None:
    """Writes xk, xv [B,T,H,D] into the head-major stores [B,H,Tcap,D] at
    positions start.. and refreshes the block sums [B,H,NBcap,D] they touch."""
    if xk.dim() != 4 or tuple(xk.shape) != tuple(xv.shape) or tuple(k_store.shape) != tuple(v_store.shape) \
            or k_store.dim() != 4 or proto_sum.dim() != 4:
        raise ValueError(f"xk, xv must be [B, T, H, D] alike and the stores [B, H, Tcap, D] alike, got "
                         f"{tuple(xk.shape)}, {tuple(xv.shape)}, {tuple(k_store.shape)}, {tuple(v_store.shape)}")
    b_, t_, h_, d_ = xk.shape
    if k_store.shape[0] < b_ or k_store.shape[1] != h_ or k_store.shape[3] != d_ or \
            proto_sum.shape[0] < b_ or proto_sum.shape[1] != h_ or proto_sum.shape[3] != d_ or \
            proto_sum.dtype != torch.float32 or not (proto_sum.is_contiguous() and k_store.is_contiguous()
                                                     and v_store.is_contiguous()):
        raise ValueError(f"stores {tuple(k_store.shape)} / sums {tuple(proto_sum.shape)} do not fit "
                         f"[{b_}, {t_}, {h_}, {d_}] rows (contiguous stores, fp32 sums)")
    _cuda(xk, xv, k_store, v_store, proto_sum)
    xk, xv = _inner1(xk.to(k_store.dtype)), _inner1(xv.to(v_store.dtype))
    b, t, h, d = xk.shape
    L.call("sd_kv_append", xk.data_ptr(), xv.data_ptr(), dtype_code(k_store), b, t, h, d, xk.stride(0),
           xk.stride(1), xk.stride(2), xv.stride(0), xv.stride(1), xv.stride(2), k_store.data_ptr(),
           v_store.data_ptr(), proto_sum.data_ptr(), k_store.shape[2], proto_sum.shape[2], start, block_size,
           _stream(xk))


def _rope_tables(cos: torch.Tensor, sin: torch.Tensor, head_dim: int, need: int) -> None:
    """The fused decode kernels read fp32 tables [max_pos, head_dim / 2] at the
    new token's position; anything else would be read as fp32 and past its end."""
    for tb in (cos, sin):
        if tb.dtype != torch.float32 or not tb.is_contiguous() or tb.dim() != 2 or tb.shape[1] != head_dim // 2:
            raise TypeError(f"RoPE tables must be contiguous fp32 [max_pos, {head_dim // 2}], got "
                            f"{tb.dtype} {tuple(tb.shape)}")
    if cos.shape != sin.shape or cos.shape[0] < need:
        raise ValueError(f"RoPE tables cover {cos.shape[0]} positions; the cache needs {need}")


def decode_layer(qkv: torch.Tensor, forecast: Optional[torch.Tensor], rope_cos: torch.Tensor,
                 rope_sin: torch.Tensor, cur_len: torch.Tensor, k_store: torch.Tensor, v_store: torch.Tensor,
                 proto_sum: torch.Tensor, n_head: int, n_kv_head: int, block_size: int, top_k: int,
                 rule: str = "reference", scale: Optional[float] = None,
                 out: Optional[torch.Tensor] = None, sel_out: Optional[torch.Tensor] = None,
                 cnt_out: Optional[torch.Tensor] = None,
                 cand: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                 next_cand: Optional[Tuple[torch.Tensor, torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]] = None,
                 select_before_append: bool = False) -> torch.Tensor:
    """Fused decode layer: RoPE + append + compressor update + selection +
    attention (model/attention/sparse.py:366-410 + :99-183 for T == 1).
    next_cand (optional) = (next layer's proto_sum, next layer's forecast
    rows [B,Hkv*D] (activation dtype), (cand_idx, cand_val) out): the kernel
    also computes the next layer's candidates for its coming step.
    qkv [B,(Hq+2Hkv)*D] (pre-RoPE projections), forecast [B,Hkv,D] or None.
    sel_out [B,Hkv,cap] / cnt_out [B,Hkv] int32 (optional) receive each
    (sequence, kv head)'s selected block list.  cand (optional) is the
    (cand_idx, cand_val) pair decode_candidates produced for this step.
    select_before_append: score the current block with its sum before this
    step's token (AsyncForecastOffloadAttention's prefetch timing,
    async_offload.py:241-260) instead of after the append (sparse.py:133-139).
    Returns [B,Hq*D]."""
    _cuda(qkv, forecast, rope_cos, rope_sin, cur_len, k_store, v_store, proto_sum)
    _rope_tables(rope_cos, rope_sin, k_store.shape[-1], k_store.shape[2])
    b = qkv.shape[0]
    d = k_store.shape[-1]
    qkv = _inner1(qkv)
    if out is None:
        out = torch.empty(b, n_head * d, dtype=k_store.dtype, device=qkv.device)
    if forecast is not None:
        f = forecast.reshape(b, n_kv_head * d)
        f = _inner1(f)
        fargs = (f.data_ptr(), dtype_code(f), f.stride(0))
    else:
        fargs = (None, dtype_code(k_store), 0)
    if next_cand is not None:
        # the kernel indexes the next layer's sums with this layer's geometry
        nproto, nfc, (nci, ncv) = next_cand
        _cuda(nproto, nfc, nci, ncv)
        if nproto.shape != proto_sum.shape or nproto.dtype != torch.float32 or not nproto.is_contiguous():
            raise ValueError(f"next layer's block sums {tuple(nproto.shape)} must match this layer's "
                             f"{tuple(proto_sum.shape)} (fp32, contiguous)")
        if nfc.reshape(b, -1).shape[1] != n_kv_head * d or nfc.dtype != qkv.dtype:
            raise ValueError(f"next layer's forecast rows must hold {n_kv_head * d} values of {qkv.dtype}")
        if top_k > 32:
            raise ValueError("chained candidates support top_k <= 32")
        for tt in (nci, ncv):
            if tuple(tt.shape) != (b, n_kv_head, top_k) or not tt.is_contiguous():
                raise ValueError(f"candidate outputs must be contiguous [{b}, {n_kv_head}, {top_k}]")
    sc = 1.0 / math.sqrt(d) if scale is None else scale
    L.call("sd_decode_layer", qkv.data_ptr(), dtype_code(qkv), qkv.stride(0), *fargs, rope_cos.data_ptr(),
           rope_sin.data_ptr(), rope_cos.shape[0], cur_len.data_ptr(), k_store.data_ptr(), v_store.data_ptr(),
           proto_sum.data_ptr(), b, n_head, n_kv_head, d, k_store.shape[2], proto_sum.shape[2], block_size, top_k,
           rule_code(rule, select_before_append), sc, out.data_ptr(), out.stride(0),
           cand[0].data_ptr() if cand is not None else None,
           cand[1].data_ptr() if cand is not None else None,
           sel_out.data_ptr() if sel_out is not None else None,
           cnt_out.data_ptr() if cnt_out is not None else None,
           sel_out.shape[-1] if sel_out is not None else 0,
           error_buffer(qkv.device).data_ptr(), *_next_args(next_cand, b, d), _stream(qkv))
    return out


def _next_args(next_cand, b: int, d: int):
    if next_cand is None:
        return (None, None, 0, None, None)
    proto, fc, (ci, cv) = next_cand
    fc = _inner1(fc.reshape(b, -1))
    return (proto.data_ptr(), fc.data_ptr(), fc.stride(0), ci.data_ptr(), cv.data_ptr())


def decode_candidates(forecast: torch.Tensor, proto_sum: torch.Tensor, cur_len: torch.Tensor, n_kv_head: int,
                      block_size: int, top_k: int, rule: str = "reference",
                      out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                      scale: Optional[float] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Top-k candidate blocks for a layer's next decode step, over every cached
    block but the current one (sd_decode_candidates).  forecast [B,Hkv,D] (or
    [B,1,Hkv,D]) rows; proto_sum [B,Hkv,NBcap,D]; cur_len device int32.
    Returns (cand_idx int32, cand_val fp32) [B,Hkv,top_k]."""
    _cuda(forecast, proto_sum, cur_len)
    b = forecast.shape[0]
    d = proto_sum.shape[-1]
    f = _inner1(forecast.reshape(b, n_kv_head * d))
    if out is None:
        out = (torch.empty(b, n_kv_head, top_k, dtype=torch.int32, device=forecast.device),
               torch.empty(b, n_kv_head, top_k, dtype=torch.float32, device=forecast.device))
    sc = 1.0 / math.sqrt(d) if scale is None else scale
    L.call("sd_decode_candidates", f.data_ptr(), dtype_code(f), f.stride(0), proto_sum.data_ptr(), b, n_kv_head, d,
           proto_sum.shape[2], cur_len.data_ptr(), block_size, top_k, RULES[rule], sc, out[0].data_ptr(),
           out[1].data_ptr(), _stream(forecast))
    return out



# ---------------------------------------------------------------- offloaded caches
def offload_prefetch(cache, cand_idx: Optional[torch.Tensor] = None) -> None:
    """Stages the blocks the next decode step of an offloaded layer attends to
    (sd_offload_prefetch): the candidates cand_idx [B,Hkv,top_k] (forecast
    steps) or the static window / every block, copied from the pinned host
    store into the cache's device slots unless already resident."""
    _cuda(cache.slot_k, cache.len_dev)
    b, h, _, d = cache.slot_k.shape
    L.call("sd_offload_prefetch", cache.host_k.data_ptr(), cache.host_v.data_ptr(), dtype_code(cache.slot_k), b, h,
           d, cache.tcap, cache.slot_k.data_ptr(), cache.slot_v.data_ptr(), cache.kslots, cache.len_dev.data_ptr(),
           cache.block_size, cache.top_k, cand_idx.data_ptr() if cand_idx is not None else None,
           cache.slot_block.data_ptr(), cache.cand_slot.data_ptr(), cache.stats.data_ptr(),
           torch.cuda.current_stream(cache.slot_k.device).cuda_stream)


def decode_layer_offload(qkv: torch.Tensor, forecast: Optional[torch.Tensor], rope_cos: torch.Tensor,
                         rope_sin: torch.Tensor, cache, n_head: int, rule: str = "reference",
                         scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                         sel_out: Optional[torch.Tensor] = None, cnt_out: Optional[torch.Tensor] = None,
                         cand: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                         select_before_append: bool = False) -> torch.Tensor:
    """decode_layer on an offloaded cache (sd_decode_layer_offload): the new
    token is written to the current-block slot and through to the host store;
    attention reads the sink, current and prefetched slots.  Forecast steps
    need ``cand`` (and the slots offload_prefetch assigned to it)."""
    _cuda(qkv, forecast, rope_cos, rope_sin, cache.slot_k)
    _rope_tables(rope_cos, rope_sin, cache.slot_k.shape[-1], cache.tcap)
    b = qkv.shape[0]
    d = cache.slot_k.shape[-1]
    hkv = cache.n_kv_head
    qkv = _inner1(qkv)
    if out is None:
        out = torch.empty(b, n_head * d, dtype=cache.slot_k.dtype, device=qkv.device)
    if forecast is not None:
        f = _inner1(forecast.reshape(b, hkv * d))
        fargs = (f.data_ptr(), dtype_code(f), f.stride(0))
    else:
        fargs = (None, dtype_code(cache.slot_k), 0)
    sc = 1.0 / math.sqrt(d) if scale is None else scale
    L.call("sd_decode_layer_offload", qkv.data_ptr(), dtype_code(qkv), qkv.stride(0), *fargs, rope_cos.data_ptr(),
           rope_sin.data_ptr(), rope_cos.shape[0], cache.len_dev.data_ptr(), cache.host_k.data_ptr(),
           cache.host_v.data_ptr(), cache.tcap, cache.slot_k.data_ptr(), cache.slot_v.data_ptr(), cache.kslots,
           cache.proto_sum.data_ptr(), b, n_head, hkv, d, cache.nbcap, cache.block_size, cache.top_k,
           rule_code(rule, select_before_append),
           sc, out.data_ptr(), out.stride(0),
           cand[0].data_ptr() if cand is not None else None,
           cand[1].data_ptr() if cand is not None else None,
           cache.cand_slot.data_ptr() if cand is not None else None,
           sel_out.data_ptr() if sel_out is not None else None,
           cnt_out.data_ptr() if cnt_out is not None else None,
           sel_out.shape[-1] if sel_out is not None else 0,
           error_buffer(qkv.device).data_ptr(), _stream(qkv))
    return out

# ---------------------------------------------------------------- prefill
LIST_MODES = {"dense": 0, "masked_forecast": 1, "masked_static": 2, "chunked_forecast": 3, "chunked_static": 4}


def prefill_lists(mode: str, batch: int, n_kv_head: int, seq_len: int, block_size: int, top_k: int,
                  topk: Optional[torch.Tensor] = None, causal: bool = True, device=None
                  ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-(sequence, kv head, 64-token query block) block lists of the prefill
    paths (model/attention/sparse.py:185-364); see SD_LIST_* in the C header.
    topk [B,H,T,k] int64 for the *_forecast modes.  Returns (lists [B,H,NQ,cap]
    int32 ascending and -1 padded, counts [B,H,NQ] int32)."""
    nb = num_blocks(seq_len, block_size)
    cap = min(nb, top_k + 2) if mode.startswith("chunked") else (nb if mode != "masked_static" else top_k + 2)
    dev = topk.device if topk is not None else device
    lists = torch.empty(batch, n_kv_head, nb, cap, dtype=torch.int32, device=dev)
    counts = torch.empty(batch, n_kv_head, nb, dtype=torch.int32, device=dev)
    if topk is not None:
        _cuda(topk)
        topk = topk.to(torch.int64).contiguous()
    L.call("sd_prefill_lists", LIST_MODES[mode], int(bool(causal)), batch, n_kv_head, seq_len, block_size, top_k,
           topk.data_ptr() if topk is not None else None, topk.shape[-1] if topk is not None else 0,
           lists.data_ptr(), counts.data_ptr(), cap, torch.cuda.current_stream(dev).cuda_stream)
    return lists, counts


def _check_prefill_shapes(q, k, v, lists, counts, topk, block_size, dout=None):
    """Shapes the prefill kernels index by, checked before any launch: q (and
    dout) [B,T,Hq,D]; k, v [>=B, Hkv, >=T, D] (cache views may hold more
    sequences or positions); lists [B,Hkv,NQ,cap] and counts [B,Hkv,NQ] int32
    contiguous (NQ = ceil(T / block_size)); topk [B,Hkv,T,k]."""
    if q.dim() != 4:
        raise ValueError(f"q must be [B, T, Hq, D], got {tuple(q.shape)}")
    b, t, hq, d = q.shape
    if dout is not None and tuple(dout.shape) != tuple(q.shape):
        raise ValueError(f"dout must have q's shape {tuple(q.shape)}, got {tuple(dout.shape)}")
    if k.dim() != 4 or tuple(k.shape) != tuple(v.shape) or k.shape[0] < b or k.shape[2] < t or k.shape[3] != d:
        raise ValueError(f"k and v must be [>={b}, Hkv, >={t}, {d}], got {tuple(k.shape)} and {tuple(v.shape)}")
    hkv = k.shape[1]
    if hq % hkv:
        raise ValueError(f"query heads ({hq}) must be a multiple of kv heads ({hkv})")
    nq = num_blocks(t, block_size)
    if lists.dim() != 4 or tuple(lists.shape[:3]) != (b, hkv, nq) or tuple(counts.shape) != (b, hkv, nq):
        raise ValueError(f"lists must be [{b}, {hkv}, {nq}, cap] and counts [{b}, {hkv}, {nq}], got "
                         f"{tuple(lists.shape)} and {tuple(counts.shape)}")
    if lists.dtype != torch.int32 or counts.dtype != torch.int32 or not lists.is_contiguous() \
            or not counts.is_contiguous():
        raise ValueError("lists and counts must be contiguous int32 (as prefill_lists returns them)")
    if topk is not None and (topk.dim() != 4 or tuple(topk.shape[:3]) != (b, hkv, t)):
        raise ValueError(f"topk must be [{b}, {hkv}, {t}, k], got {tuple(topk.shape)}")


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, lists: torch.Tensor, counts: torch.Tensor,
                      block_size: int, topk: Optional[torch.Tensor] = None, causal: bool = True,
                      scale: Optional[float] = None) -> torch.Tensor:
    """Block-sparse GQA prefill attention over prefill_lists' lists.
    q [B,T,Hq,D]; k, v [B,Hkv,T,D] views (same strides); topk [B,H,T,k] for
    per-row membership (masked forecast mode).  Returns [B,T,Hq,D]."""
    _check_prefill_shapes(q, k, v, lists, counts, topk, block_size)
    _cuda(q, k, v, lists, counts, topk)
    b, t, hq, d = q.shape
    hkv = k.shape[1]
    if k.stride() != v.stride():
        k, v = k.contiguous(), v.contiguous()
    q, k, v = _inner1(q), _inner1(k), _inner1(v)
    if k.stride() != v.stride():
        k, v = k.contiguous(), v.contiguous()
    if q.dtype != k.dtype:
        q = q.to(k.dtype)
    out = torch.empty(b, t, hq, d, dtype=k.dtype, device=q.device)
    tk = topk.to(torch.int64).contiguous() if topk is not None else None
    sc = 1.0 / math.sqrt(d) if scale is None else scale
    L.call("sd_prefill_attention", q.data_ptr(), dtype_code(k), b, t, hq, hkv, d, q.stride(0), q.stride(1),
           q.stride(2), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k.stride(2), lists.data_ptr(),
           counts.data_ptr(), lists.shape[-1], tk.data_ptr() if tk is not None else None,
           tk.shape[-1] if tk is not None else 0, block_size, int(bool(causal)), sc, out.data_ptr(), out.stride(0),
           out.stride(1), out.stride(2), _stream(q))
    return out


def prefill_attention_backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, dout: torch.Tensor,
                               lists: torch.Tensor, counts: torch.Tensor, block_size: int,
                               topk: Optional[torch.Tensor] = None, causal: bool = True,
                               scale: Optional[float] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients of prefill_attention for the output gradient dout [B,T,Hq,D]
    (the backward of the reference's masked / chunked SDPA, sparse.py:185-364):
    same q, k, v, lists and topk as the forward.  Returns fp32 (dq [B,T,Hq,D],
    dk [B,Hkv,T,D], dv [B,Hkv,T,D])."""
    _check_prefill_shapes(q, k, v, lists, counts, topk, block_size, dout)
    _cuda(q, k, v, dout, lists, counts, topk)
    b, t, hq, d = q.shape
    hkv = k.shape[1]
    q, k, v, dout = _inner1(q), _inner1(k), _inner1(v), _inner1(dout)
    if k.stride() != v.stride():
        k, v = k.contiguous(), v.contiguous()
    if q.dtype != k.dtype:
        q = q.to(k.dtype)
    if dout.dtype != k.dtype:
        dout = dout.to(k.dtype)
    dq = torch.empty(b, t, hq, d, dtype=torch.float32, device=q.device)
    dk = torch.empty(b, hkv, t, d, dtype=torch.float32, device=q.device)
    dv = torch.empty_like(dk)
    tk = topk.to(torch.int64).contiguous() if topk is not None else None
    sc = 1.0 / math.sqrt(d) if scale is None else scale
    L.call("sd_prefill_attention_backward", q.data_ptr(), k.data_ptr(), v.data_ptr(), dout.data_ptr(),
           dtype_code(k), b, t, hq, hkv, d, q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1),
           k.stride(2), dout.stride(0), dout.stride(1), dout.stride(2), lists.data_ptr(), counts.data_ptr(),
           lists.shape[-1], tk.data_ptr() if tk is not None else None, tk.shape[-1] if tk is not None else 0,
           block_size, int(bool(causal)), sc, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), _stream(q))
    return dq, dk, dv


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm (model/norm.py:15-21) over the last dim of a 2-D [rows, C] tensor."""
    _cuda(x, weight)
    x = _inner1(x)
    w = weight.to(x.dtype).contiguous()
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    L.call("sd_rmsnorm", x.data_ptr(), dtype_code(x), x.shape[0], x.shape[1], x.stride(0), w.data_ptr(), eps,
           out.data_ptr(), out.stride(0), _stream(x))
    return out


def silu_mul(gu: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up for gu = [gate | up] rows [rows, 2F] -> [rows, F]."""
    _cuda(gu)
    gu = _inner1(gu)
    f = gu.shape[1] // 2
    out = torch.empty(gu.shape[0], f, dtype=gu.dtype, device=gu.device)
    L.call("sd_silu_mul", gu.data_ptr(), dtype_code(gu), gu.shape[0], f, gu.stride(0), out.data_ptr(),
           out.stride(0), _stream(gu))
    return out


def argmax_rows(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """torch.argmax(x, dim=-1) for 2-D x (rows with unit column stride): the
    first index of each row's maximum, NaN above every number.  Writes int64
    indices into ``out`` (any shape with one element per row) or a new [rows]
    tensor."""
    _cuda(x)
    x = _inner1(x)
    rows, n = x.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.int64, device=x.device)
    if out.dtype != torch.int64 or out.numel() != rows:
        raise ValueError("out must hold one int64 per row")
    o_stride = out.stride(0) if out.dim() >= 1 else 1
    L.call("sd_argmax_rows", x.data_ptr(), dtype_code(x), rows, n, x.stride(0), out.data_ptr(), o_stride, _stream(x))
    return out


def advance_len(lens: torch.Tensor, delta: int = 1) -> None:
    _cuda(lens)
    L.call("sd_advance_len", lens.data_ptr(), lens.numel(), delta, _stream(lens))


def set_programmatic_launch(enable: bool) -> bool:
    """Programmatic dependent launch for the decode-step kernels of this
    library (sd_set_programmatic_launch): each may start while the kernel ahead
    of it is finishing and waits for it before reading its output.  Meant for
    the decode step, where every such kernel follows a library GEMM.  Returns
    the previous setting."""
    return bool(L.load().sd_set_programmatic_launch(int(bool(enable))))


def rope_qk(xq: torch.Tensor, xk: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
            offset: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """apply_rotary_emb (model/rope.py:34-65) on q [B,T,Hq,D] and k [B,T,Hkv,D]
    in one kernel with the reference's rounding sequence; returns contiguous
    rotated copies.  cos/sin: the fp32 tables [max_pos, D/2]."""
    _cuda(xq, xk, cos, sin)
    b, t, hq, d = xq.shape
    hkv = xk.shape[2]
    _rope_tables(cos, sin, d, offset + t)
    if xk.dtype != xq.dtype:
        raise TypeError("q and k must share a dtype")
    xq, xk = _inner1(xq), _inner1(xk)
    qo = torch.empty(b, t, hq, d, dtype=xq.dtype, device=xq.device)
    ko = torch.empty(b, t, hkv, d, dtype=xk.dtype, device=xk.device)
    L.call("sd_rope_qk", xq.data_ptr(), xk.data_ptr(), dtype_code(xq), b, t, hq, hkv, d, xq.stride(0), xq.stride(1),
           xq.stride(2), xk.stride(0), xk.stride(1), xk.stride(2), cos.data_ptr(), sin.data_ptr(), cos.shape[0],
           offset, qo.data_ptr(), ko.data_ptr(), _stream(xq))
    return qo, ko


LINEAR_EPILOGUES = {"store": 0, "residual": 1, "swiglu": 2}


def linear(x: torch.Tensor, w: torch.Tensor, norm_w: Optional[torch.Tensor] = None, eps: float = 1e-6,
           epilogue: str = "store", res: Optional[torch.Tensor] = None,
           out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """A decode-step projection on the tensor cores (sd_linear): out = X W^T
    for x [M, K], w [N, K] (16-bit), with RMSNorm of x in front when norm_w is
    given (model/norm.py:15-21) and one of the epilogues: "store", "residual"
    (res + the projection, model/transformer.py:118-129; out may be res) or
    "swiglu" (w = swiglu_weight(w_gate, w_up); silu(gate) * up, N/2 columns,
    transformer.py:18-31)."""
    _cuda(x, w, norm_w, res)
    if x.dtype != w.dtype or (norm_w is not None and norm_w.dtype != x.dtype):
        raise TypeError("x, w and the norm gain must share a 16-bit dtype")
    x = _inner1(x)
    w = w.contiguous()
    m, k = x.shape
    n = w.shape[0]
    ncols = n // 2 if epilogue == "swiglu" else n
    if out is None:
        out = torch.empty(m, ncols, dtype=x.dtype, device=x.device)
    if epilogue == "residual" and (res is None or res.shape != (m, n) or res.stride(-1) != 1):
        raise ValueError(f"the residual must be [{m}, {n}] with unit column stride")
    nw = norm_w.contiguous() if norm_w is not None else None
    L.call("sd_linear", x.data_ptr(), dtype_code(x), m, k, x.stride(0), w.data_ptr(), n,
           nw.data_ptr() if nw is not None else None, eps, LINEAR_EPILOGUES[epilogue],
           res.data_ptr() if res is not None else None, res.stride(0) if res is not None else 0, out.data_ptr(),
           out.stride(0), error_buffer(x.device).data_ptr(), _stream(x))
    return out


def swiglu_weight(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """[w_gate; w_up] interleaved in groups of 64 rows (64 gate rows, then the
    64 up rows of the same output columns), the layout linear(...,
    epilogue="swiglu") reads."""
    f, k = w_gate.shape
    if f % 64:
        raise ValueError("the FFN width must be a multiple of 64")
    return torch.stack((w_gate.view(f // 64, 64, k), w_up.view(f // 64, 64, k)), dim=1).reshape(2 * f, k).contiguous()
