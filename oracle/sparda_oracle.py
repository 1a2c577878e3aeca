"""CPU oracle for SparDA's forecast-guided block-sparse attention path.

TEST INFRASTRUCTURE ONLY.  This module is the checker: it is imported by the
tests under ``tests/``, by ``__graft_entry__.smoke()`` and by the ``cpu_baseline``
/ ``--impl reference`` legs of ``bench.py``.  The product package never imports
it, and nothing here is a fallback for the CUDA path.

It restates, in numpy (float64 by default), the algorithm of the reference
(tyborra/local-research-Small-Language-Model, "SparDA") for this path.  Each
function cites the reference file:line it follows.  Where the reference's result
is implementation-defined (``torch.topk`` tie order), the oracle fixes one
deterministic rule, and the CUDA kernels implement the same rule:

* top-k ordering: value descending; equal values (``-inf`` included) in
  ascending block index.  This settles which blocks fill the ``-inf`` slots of
  a top-k row that has fewer than k finite scores
  (model/forecast.py:120-129).
* selected-set compaction (``torch.topk(mask.float(), k=MS)``,
  model/attention/sparse.py:154 and :333): the selected blocks are listed in
  ascending order followed by invalid slots.  In the chunked prefill path a
  union larger than MS is truncated by keeping the sink block and the current
  block, then the remaining blocks ranked by how many of the q-block's rows
  voted for them (descending), ties by ascending index.  The reference keeps an
  unspecified MS-subset of the union; this rule picks one such subset.
* decode-time causal rule ("reference" vs "absolute"): the reference's decode
  call passes a single forecast row, so its causal mask uses row index 0 and
  leaves only block 0 finite (model/forecast.py:120-126 called from
  model/attention/sparse.py:139).  ``rule="reference"`` reproduces that;
  ``rule="absolute"`` masks by the query's absolute position instead.

Parity of this restatement is pinned by the golden vectors that
``tests/golden/make_golden.py`` produced by running the reference itself.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np

NEG_INF = -np.inf


def num_blocks(seq_len: int, block_size: int) -> int:
    return (seq_len + block_size - 1) // block_size


# ---------------------------------------------------------------------------
# K1 compressor, K2 selector
# ---------------------------------------------------------------------------

def compress_blocks(k: np.ndarray, block_size: int, dtype=np.float64) -> np.ndarray:
    """KVBlockCompressor.forward (model/forecast.py:57-78).

    k: [B, T, H, D] -> block prototypes [B, N_b, H, D].  The last block is
    zero-padded and still divided by ``block_size`` (forecast.py:69-77), so a
    partial block's prototype is sum/block_size, not the mean of its tokens.
    The projection is the identity because head_dim == forecast_dim
    (forecast.py:51-55).
    """
    k = np.asarray(k, dtype=dtype)
    b, t, h, d = k.shape
    nb = num_blocks(t, block_size)
    pad = nb * block_size - t
    if pad:
        k = np.concatenate([k, np.zeros((b, pad, h, d), dtype=dtype)], axis=1)
    return k.reshape(b, nb, block_size, h, d).sum(axis=2) / block_size


def selector_scores(forecast: np.ndarray, reps: np.ndarray, block_size: int,
                    is_causal: bool, q_offset: int = 0, dtype=np.float64) -> np.ndarray:
    """Score part of ForecastBlockSelector.forward (model/forecast.py:103-126).

    forecast [B, Tq, H, D], reps [B, N_b, H, D] -> scores [B, H, Tq, N_b]
    = (f . rep) / sqrt(D), with blocks j > (t + q_offset) // block_size set to
    -inf when causal.  q_offset = 0 is the reference (t = row index).
    """
    f = np.asarray(forecast, dtype=dtype).transpose(0, 2, 1, 3)
    r = np.asarray(reps, dtype=dtype).transpose(0, 2, 1, 3)
    assert f.shape[1] == r.shape[1], "forecast heads must equal kv heads (forecast.py:110)"
    d = f.shape[-1]
    scores = (f @ r.transpose(0, 1, 3, 2)) * (1.0 / math.sqrt(d))
    if is_causal:
        tq, nb = scores.shape[2], scores.shape[3]
        t = np.arange(tq) + q_offset
        future = np.arange(nb)[None, :] > (t[:, None] // block_size)
        scores = np.where(future[None, None], NEG_INF, scores)
    return scores


def topk_desc(scores: np.ndarray, k: int) -> np.ndarray:
    """``torch.topk(scores, k, dim=-1).indices`` (largest, sorted) with the fixed
    tie rule: equal values, -inf included, in ascending index order."""
    neg = -np.asarray(scores)
    return np.argsort(neg, axis=-1, kind="stable")[..., :k]


def select_blocks(forecast, reps, top_k: int, block_size: int, is_causal: bool = True,
                  q_offset: int = 0, dtype=np.float64) -> Tuple[np.ndarray, np.ndarray]:
    """ForecastBlockSelector.forward (model/forecast.py:89-130): (scores, topk indices)."""
    scores = selector_scores(forecast, reps, block_size, is_causal, q_offset, dtype)
    k = min(top_k, scores.shape[-1])
    return scores, topk_desc(scores, k)


# ---------------------------------------------------------------------------
# RoPE (model/rope.py)
# ---------------------------------------------------------------------------

def rope_tables(head_dim: int, max_seq_len: int, theta: float = 10000.0):
    """precompute_rope_freqs (model/rope.py:8-23), in float32 like the reference.

    theta ** (2i / d) is rounded once to float32 (torch's float32 pow returns
    the correctly rounded power), then inverted in float32 as the reference's
    ``1.0 / tensor`` is.  A 1-ulp error in an inverse frequency becomes a phase
    error of position x ulp, about 1e-3 rad at 16K positions, so the table must
    be built exactly this way to match the reference at long contexts."""
    p = (theta ** (np.arange(0, head_dim, 2, dtype=np.float64) / head_dim)).astype(np.float32)
    inv = (np.float32(1.0) / p).astype(np.float32)
    t = np.arange(max_seq_len, dtype=np.float32)
    freqs = np.outer(t, inv).astype(np.float32)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, offset: int = 0) -> np.ndarray:
    """apply_rotary_emb (model/rope.py:34-65) on one tensor x [B, T, H, D]."""
    t, d = x.shape[1], x.shape[-1]
    c = np.concatenate([cos[offset:offset + t], cos[offset:offset + t]], axis=-1)[None, :, None, :]
    s = np.concatenate([sin[offset:offset + t], sin[offset:offset + t]], axis=-1)[None, :, None, :]
    rot = np.concatenate([-x[..., d // 2:], x[..., :d // 2]], axis=-1)
    return x * c + rot * s


# ---------------------------------------------------------------------------
# Decode path (model/attention/sparse.py:99-183)
# ---------------------------------------------------------------------------

def _compact(mask: np.ndarray, ms: int) -> Tuple[np.ndarray, np.ndarray]:
    """Selected-set compaction: True blocks in ascending order, then -1 slots.
    Stands for ``torch.topk(mask.float(), k=ms)`` (sparse.py:154) when at most ms
    blocks are True, which the decode path guarantees."""
    lead = mask.shape[:-1]
    sel = np.full(lead + (ms,), -1, dtype=np.int64)
    cnt = np.zeros(lead, dtype=np.int64)
    flat_m = mask.reshape(-1, mask.shape[-1])
    flat_s = sel.reshape(-1, ms)
    flat_c = cnt.reshape(-1)
    for r in range(flat_m.shape[0]):
        ids = np.nonzero(flat_m[r])[0]
        assert len(ids) <= ms
        flat_s[r, :len(ids)] = ids
        flat_c[r] = len(ids)
    return sel, cnt


def decode_select(forecast: Optional[np.ndarray], reps: Optional[np.ndarray], seq_len_k: int,
                  block_size: int, top_k: int, batch: int, n_kv_head: int,
                  mode: str = "forecast", rule: str = "reference",
                  dtype=np.float64) -> Tuple[np.ndarray, np.ndarray]:
    """Selected-block list of one decode step (sparse.py:108-154).

    forecast [B, 1, H, D] (layer L-1's forecast) or None; reps = compressor
    output over the cache *after* the new token was appended (sparse.py:134-135).
    Returns sel [B, H, MS] (ascending, -1 padded) and cnt [B, H].  When
    N_b <= MS every block is selected: that is the dense fallback
    (sparse.py:113-123), whose keys are exactly all cached tokens.
    """
    nb = num_blocks(seq_len_k, block_size)
    curr = (seq_len_k - 1) // block_size
    ms = min(nb, top_k + 2)
    if nb <= ms:
        sel = np.broadcast_to(np.arange(nb, dtype=np.int64), (batch, n_kv_head, nb)).copy()
        return sel, np.full((batch, n_kv_head), nb, dtype=np.int64)
    mask = np.zeros((batch, n_kv_head, nb), dtype=bool)
    mask[..., 0] = True
    mask[..., curr] = True
    if mode == "forecast" and forecast is not None:
        q_off = 0 if rule == "reference" else seq_len_k - 1
        _, idx = select_blocks(forecast, reps, top_k, block_size, True, q_off, dtype)
        idx = np.clip(idx[:, :, 0, :], 0, nb - 1)
        np.put_along_axis(mask, idx, True, axis=-1)
    else:
        for j in range(max(0, curr - top_k + 1), curr + 1):
            mask[..., j] = True
    mask[..., curr + 1:] = False
    return _compact(mask, ms)


def decode_attention(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, sel: np.ndarray,
                     cnt: np.ndarray, seq_len_k: int, block_size: int,
                     scale: Optional[float] = None, dtype=np.float64) -> np.ndarray:
    """Gathered decode attention (sparse.py:156-181): gather_kv_blocks
    (sparse.py:19-62), token validity ``pos < seq_len_k`` and slot validity
    (sparse.py:160-167), GQA head h -> kv head h // G (repeat_interleave,
    sparse.py:176-179), softmax(q k^T * scale) v.

    q [B, Hq, D]; k_cache, v_cache [B, Hkv, T, D] with T >= seq_len_k;
    sel [B, Hkv, S], cnt [B, Hkv] -> out [B, Hq, D].
    """
    q = np.asarray(q, dtype=dtype)
    b, hq, d = q.shape
    hkv = k_cache.shape[1]
    g = hq // hkv
    s = sel.shape[-1]
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    slot_ok = np.arange(s)[None, None, :] < cnt[..., None]
    blk = np.where(slot_ok, sel, 0)
    pos = blk[..., None] * block_size + np.arange(block_size)
    valid = (slot_ok[..., None] & (pos < seq_len_k)).reshape(b, hkv, s * block_size)
    pos = np.minimum(pos, seq_len_k - 1).reshape(b, hkv, s * block_size)
    kg = np.take_along_axis(np.asarray(k_cache, dtype=dtype), pos[..., None], axis=2)
    vg = np.take_along_axis(np.asarray(v_cache, dtype=dtype), pos[..., None], axis=2)
    qh = q.reshape(b, hkv, g, d)
    sc = np.einsum("bhgd,bhnd->bhgn", qh, kg) * scale
    sc = np.where(valid[:, :, None, :], sc, NEG_INF)
    sc = sc - sc.max(axis=-1, keepdims=True)
    p = np.exp(sc)
    p = p / p.sum(axis=-1, keepdims=True)
    out = np.einsum("bhgn,bhnd->bhgd", p, vg)
    return out.reshape(b, hq, d)


# ---------------------------------------------------------------------------
# Prefill paths (model/attention/sparse.py:185-364)
# ---------------------------------------------------------------------------

def _softmax_attend(q, k, v, allowed, scale, dtype):
    """softmax(q k^T * scale + mask) v with a boolean ``allowed`` [B, Hkv|1, Tq, Tk]."""
    b, hq, tq, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    out = np.empty((b, hq, tq, d), dtype=dtype)
    for h in range(hq):
        kh = h // g
        a = allowed[:, kh if allowed.shape[1] > 1 else 0]
        sc = np.einsum("btd,bsd->bts", q[:, h], k[:, kh]) * scale
        sc = np.where(a, sc, NEG_INF)
        sc = sc - sc.max(axis=-1, keepdims=True)
        p = np.exp(sc)
        p /= p.sum(axis=-1, keepdims=True)
        out[:, h] = np.einsum("bts,bsd->btd", p, v[:, kh])
    return out


def masked_allowed(forecast, k, seq_len: int, block_size: int, top_k: int, layer_idx: int,
                   mode: str = "forecast", is_causal: bool = True, dtype=np.float64):
    """The boolean ``allowed`` mask of _forward_masked_sdpa (sparse.py:198-253).

    Returns (allowed [B, Hkv|1, T, T], topk indices or None, dense flag)."""
    b, hkv = k.shape[0], k.shape[1]
    nb = num_blocks(seq_len, block_size)
    t = np.arange(seq_len)
    causal = t[None, :] <= t[:, None]
    if nb <= 2 or (mode == "forecast" and (forecast is None or layer_idx == 0)):
        allowed = causal if is_causal else np.ones_like(causal)
        return allowed[None, None], None, True
    bq = (t // block_size)[:, None]
    bk = (t // block_size)[None, :]
    sink = bk == 0
    topk = None
    if mode == "forecast" and forecast is not None:
        reps = compress_blocks(np.asarray(k, dtype=dtype).transpose(0, 2, 1, 3), block_size, dtype)
        _, topk = select_blocks(forecast, reps, top_k, block_size, is_causal, 0, dtype)
        sel = np.zeros((b, hkv, seq_len, nb), dtype=bool)
        np.put_along_axis(sel, np.clip(topk, 0, nb - 1), True, axis=-1)
        topk_sel = sel[..., (t // block_size)]  # [B, H, T, T] via key block
        allowed = (bk == bq)[None, None] | sink[None, None] | topk_sel
    else:
        window = (bk <= bq) & (bq - bk < top_k + 1)
        allowed = (window | sink)[None, None]
    if is_causal:
        allowed = allowed & causal[None, None]
    return allowed, topk, False


def masked_prefill(q, k, v, forecast, block_size: int, top_k: int, layer_idx: int,
                   mode: str = "forecast", is_causal: bool = True, scale: Optional[float] = None,
                   dtype=np.float64) -> np.ndarray:
    """_forward_masked_sdpa (sparse.py:185-282) without the output projection.

    q [B, Hq, T, D]; k, v [B, Hkv, T, D]; forecast [B, T, Hkv, Df] or None.
    Returns [B, Hq, T, D]."""
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    seq_len = q.shape[2]
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    allowed, _, _ = masked_allowed(forecast, k, seq_len, block_size, top_k, layer_idx, mode,
                                   is_causal, dtype)
    return _softmax_attend(q, k, v, allowed, scale, dtype)


def chunked_select(forecast, reps, seq_len: int, block_size: int, top_k: int,
                   batch: int, n_kv_head: int, mode: str = "forecast",
                   dtype=np.float64) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Per-q-block selected lists of _forward_chunked_gather (sparse.py:303-333).

    Returns sel [B, H, N_b, MS] (ascending, -1 padded), cnt [B, H, N_b] and the
    untruncated union mask [B, H, N_b, N_b].  A union larger than MS is cut by
    the documented rule (sink, current, then votes desc / index asc)."""
    nb = num_blocks(seq_len, block_size)
    ms = min(nb, top_k + 2)
    sel = np.full((batch, n_kv_head, nb, ms), -1, dtype=np.int64)
    cnt = np.zeros((batch, n_kv_head, nb), dtype=np.int64)
    union = np.zeros((batch, n_kv_head, nb, nb), dtype=bool)
    use_fc = mode == "forecast" and forecast is not None
    if use_fc:
        _, topk = select_blocks(forecast, reps, top_k, block_size, False, 0, dtype)  # [B,H,T,k]
        topk = np.clip(topk, 0, nb - 1)
    for bq in range(nb):
        votes = np.zeros((batch, n_kv_head, nb), dtype=np.int64)
        mask = np.zeros((batch, n_kv_head, nb), dtype=bool)
        mask[..., 0] = True
        mask[..., bq] = True
        if use_fc and bq > 0:
            rows = topk[:, :, bq * block_size:min(seq_len, (bq + 1) * block_size), :]
            rows = rows.reshape(batch, n_kv_head, -1)
            for bb in range(batch):
                for hh in range(n_kv_head):
                    np.add.at(votes[bb, hh], rows[bb, hh], 1)
            mask |= votes > 0
        else:
            for j in range(max(0, bq - top_k + 1), bq + 1):
                mask[..., j] = True
        mask[..., bq + 1:] = False
        union[:, :, bq] = mask
        for bb in range(batch):
            for hh in range(n_kv_head):
                ids = np.nonzero(mask[bb, hh])[0]
                if len(ids) > ms:
                    keep = [0, bq] if bq != 0 else [0]
                    rest = [j for j in ids if j not in keep]
                    rest.sort(key=lambda j: (-votes[bb, hh, j], j))
                    ids = np.array(sorted(keep + rest[:ms - len(keep)]), dtype=np.int64)
                sel[bb, hh, bq, :len(ids)] = ids
                cnt[bb, hh, bq] = len(ids)
    return sel, cnt, union


def chunked_attention(q, k, v, sel, cnt, block_size: int, scale: Optional[float] = None,
                      dtype=np.float64) -> np.ndarray:
    """Per-q-block gathered attention of _forward_chunked_gather
    (sparse.py:334-360): keys of the listed blocks with ``pos < T`` and
    ``pos <= q_pos``; GQA by repeat_interleave.  q [B, Hq, T, D] -> [B, Hq, T, D]."""
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    b, hq, t, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    out = np.zeros_like(q)
    nb = num_blocks(t, block_size)
    for bb in range(b):
        for h in range(hkv):
            for bq in range(nb):
                ids = sel[bb, h, bq, :cnt[bb, h, bq]]
                pos = (ids[:, None] * block_size + np.arange(block_size)).reshape(-1)
                pos = pos[pos < t]
                q0, q1 = bq * block_size, min(t, (bq + 1) * block_size)
                qpos = np.arange(q0, q1)
                ok = pos[None, :] <= qpos[:, None]
                kk, vv = k[bb, h, pos], v[bb, h, pos]
                for gg in range(g):
                    hh = h * g + gg
                    sc = (q[bb, hh, q0:q1] @ kk.T) * scale
                    sc = np.where(ok, sc, NEG_INF)
                    sc = sc - sc.max(axis=-1, keepdims=True)
                    p = np.exp(sc)
                    p /= p.sum(axis=-1, keepdims=True)
                    out[bb, hh, q0:q1] = p @ vv
    return out


def chunked_prefill(q, k, v, forecast, block_size: int, top_k: int, mode: str = "forecast",
                    scale: Optional[float] = None, dtype=np.float64):
    """_forward_chunked_gather (sparse.py:284-364) without the output projection.
    Returns (out [B, Hq, T, D], sel, cnt)."""
    b, hkv, t, _ = np.shape(k)
    reps = compress_blocks(np.asarray(k, dtype=dtype).transpose(0, 2, 1, 3), block_size, dtype)
    sel, cnt, _ = chunked_select(forecast, reps, t, block_size, top_k, b, hkv, mode, dtype)
    return chunked_attention(q, k, v, sel, cnt, block_size, scale, dtype), sel, cnt


def masked_allowed_from_topk(topk: Optional[np.ndarray], seq_len: int, block_size: int,
                             is_causal: bool = True) -> np.ndarray:
    """The ``allowed`` mask of _forward_masked_sdpa (sparse.py:226-253) for
    given per-row top-k block indices [B, H, T, k] (clamped to [0, N_b - 1]
    like the reference's scatter): same block, the sink block or a top-k block
    of the query row, and causal.  ``topk=None``: the dense causal mask
    (sparse.py:201-224).  Returns [B, H|1, T, T] bool."""
    t = np.arange(seq_len)
    causal = t[None, :] <= t[:, None]
    if topk is None:
        allowed = causal if is_causal else np.ones_like(causal)
        return allowed[None, None]
    nb = num_blocks(seq_len, block_size)
    b, h = topk.shape[0], topk.shape[1]
    sel = np.zeros((b, h, seq_len, nb), dtype=bool)
    np.put_along_axis(sel, np.clip(topk, 0, nb - 1), True, axis=-1)
    bq = (t // block_size)[:, None]
    bk = (t // block_size)[None, :]
    allowed = sel[..., t // block_size] | ((bk == bq) | (bk == 0))[None, None]
    if is_causal:
        allowed = allowed & causal[None, None]
    return allowed


def chunked_allowed(sel: np.ndarray, cnt: np.ndarray, seq_len: int, block_size: int) -> np.ndarray:
    """The key set of _forward_chunked_gather (sparse.py:334-360) as a mask:
    query t sees key s when s's block is listed for t's q-block and s <= t.
    sel [B, H, N_b, MS], cnt [B, H, N_b].  Returns [B, H, T, T] bool."""
    b, h, nb, _ = sel.shape
    t = np.arange(seq_len)
    listed = np.zeros((b, h, nb, nb), dtype=bool)
    for bb in range(b):
        for hh in range(h):
            for q in range(nb):
                ids = sel[bb, hh, q, :cnt[bb, hh, q]]
                listed[bb, hh, q, ids[(ids >= 0) & (ids < nb)]] = True
    allowed = listed[:, :, (t // block_size)[:, None], (t // block_size)[None, :]]
    return allowed & (t[None, :] <= t[:, None])[None, None]


def attention_backward(q, k, v, dout, allowed, scale: Optional[float] = None, dtype=np.float64):
    """Gradients of out = softmax(scale * q k^T over ``allowed``) v, the
    backward autograd takes through the reference's SDPA calls
    (sparse.py:255-282, :334-360) with GQA by repeat_interleave: a kv head's
    dk / dv sum over its query heads.  q, dout [B, Hq, T, D]; k, v
    [B, Hkv, T, D]; allowed [B, Hkv|1, T, T].  A row with no allowed key has a
    zero output and zero gradients.  Returns (dq, dk, dv)."""
    q, k, v, dout = (np.asarray(a, dtype=dtype) for a in (q, k, v, dout))
    b, hq, t, d = q.shape
    hkv = k.shape[1]
    g = hq // hkv
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
    for h in range(hq):
        kh = h // g
        a = allowed[:, kh if allowed.shape[1] > 1 else 0]
        sc = np.where(a, np.einsum("btd,bsd->bts", q[:, h], k[:, kh]) * scale, NEG_INF)
        mx = sc.max(axis=-1, keepdims=True)
        e = np.where(a, np.exp(sc - np.where(np.isfinite(mx), mx, 0.0)), 0.0)
        den = e.sum(axis=-1, keepdims=True)
        p = e / np.where(den > 0, den, 1.0)
        dv[:, kh] += np.einsum("bts,btd->bsd", p, dout[:, h])
        dp = np.einsum("btd,bsd->bts", dout[:, h], v[:, kh])
        ds = p * (dp - (p * dp).sum(axis=-1, keepdims=True))
        dq[:, h] = np.einsum("bts,bsd->btd", ds, k[:, kh]) * scale
        dk[:, kh] += np.einsum("bts,btd->bsd", ds, q[:, h]) * scale
    return dq, dk, dv


def attention_forward(q, k, v, allowed, scale: Optional[float] = None, dtype=np.float64):
    """softmax(scale * q k^T over ``allowed``) v, with zero rows where nothing
    is allowed (the function attention_backward differentiates)."""
    q, k, v = (np.asarray(a, dtype=dtype) for a in (q, k, v))
    b, hq, t, d = q.shape
    g = hq // k.shape[1]
    scale = 1.0 / math.sqrt(d) if scale is None else scale
    out = np.zeros_like(q)
    for h in range(hq):
        kh = h // g
        a = allowed[:, kh if allowed.shape[1] > 1 else 0]
        sc = np.where(a, np.einsum("btd,bsd->bts", q[:, h], k[:, kh]) * scale, NEG_INF)
        mx = sc.max(axis=-1, keepdims=True)
        e = np.where(a, np.exp(sc - np.where(np.isfinite(mx), mx, 0.0)), 0.0)
        den = e.sum(axis=-1, keepdims=True)
        out[:, h] = np.einsum("bts,bsd->btd", e / np.where(den > 0, den, 1.0), v[:, kh])
    return out


def gather_kv_blocks(k, v, block_indices, block_size: int):
    """gather_kv_blocks (sparse.py:19-62): k, v [B, H, T, D], indices [B, H, S]
    -> [B, H, S*block_size, D], zero beyond T."""
    k = np.asarray(k)
    v = np.asarray(v)
    b, h, t, d = k.shape
    nb = num_blocks(t, block_size)
    pad = nb * block_size - t
    if pad:
        k = np.concatenate([k, np.zeros((b, h, pad, d), k.dtype)], axis=2)
        v = np.concatenate([v, np.zeros((b, h, pad, d), v.dtype)], axis=2)
    kb = k.reshape(b, h, nb, block_size, d)
    vb = v.reshape(b, h, nb, block_size, d)
    idx = np.asarray(block_indices)[..., None, None]
    kg = np.take_along_axis(kb, idx, axis=2)
    vg = np.take_along_axis(vb, idx, axis=2)
    s = idx.shape[2]
    return kg.reshape(b, h, s * block_size, d), vg.reshape(b, h, s * block_size, d)


# ---------------------------------------------------------------------------
# Async prefetch selection (model/attention/async_offload.py:190-260)
# ---------------------------------------------------------------------------

def prefetch_select(forecast, k_prefix: np.ndarray, cur_len: int, block_size: int, top_k: int,
                    layer_idx: int, rule: str = "reference", dtype=np.float64):
    """Blocks AsyncForecastOffloadAttention.prefetch stages for the next decode
    step of this layer (async_offload.py:190-260).  Selection runs before the
    new token is appended: prototypes cover ``cur_len`` tokens, the current block
    is ``cur_len // block_size`` and the block count covers ``cur_len + 1``.

    k_prefix [B, cur_len, H, D].  Returns (small_context, sel, cnt); when
    small_context is True the whole prefix up to cur_len + 1 is staged
    (async_offload.py:202-239) and sel/cnt list every block.
    """
    b, _, h, _ = k_prefix.shape
    target = cur_len + 1
    nb = num_blocks(target, block_size)
    curr = cur_len // block_size
    ms = min(nb, top_k + 2)
    if nb <= ms or forecast is None or layer_idx == 0:
        sel = np.broadcast_to(np.arange(nb, dtype=np.int64), (b, h, nb)).copy()
        return True, sel, np.full((b, h), nb, dtype=np.int64)
    reps = compress_blocks(k_prefix, block_size, dtype)
    nbr = reps.shape[1]
    q_off = 0 if rule == "reference" else cur_len
    _, idx = select_blocks(forecast, reps, top_k, block_size, True, q_off, dtype)
    mask = np.zeros((b, h, nb), dtype=bool)
    mask[..., 0] = True
    mask[..., curr] = True
    np.put_along_axis(mask, np.clip(idx[:, :, 0, :], 0, nb - 1), True, axis=-1)
    mask[..., curr + 1:] = False
    del nbr
    sel, cnt = _compact(mask, ms)
    return False, sel, cnt


# ---------------------------------------------------------------------------
# Full model decode step (model/model.py:79-157, model/transformer.py:76-131)
# ---------------------------------------------------------------------------

def rmsnorm(x, w, eps=1e-6):
    """RMSNorm (model/norm.py:15-21)."""
    x = np.asarray(x)
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * w


class OracleModel:
    """Decode step of SparDAResearchModel with the sparse backend, on CPU.

    ``state`` maps the reference's state-dict keys (model/model.py,
    model/transformer.py, model/attention/base.py:49-52) to numpy arrays.
    Caches are per layer: k, v [B, H, Tmax, D].
    """

    def __init__(self, state: dict, n_layer=12, n_head=12, n_kv_head=4, head_dim=64,
                 block_size=64, top_k=8, rope_theta=10000.0, max_seq_len=4096,
                 norm_eps=1e-6, rule="reference", dtype=np.float32):
        self.s = {k: np.asarray(v, dtype=dtype) for k, v in state.items()}
        self.n_layer, self.n_head, self.n_kv_head, self.head_dim = n_layer, n_head, n_kv_head, head_dim
        self.block_size, self.top_k, self.eps, self.rule, self.dtype = block_size, top_k, norm_eps, rule, dtype
        self.cos, self.sin = rope_tables(head_dim, max_seq_len, rope_theta)
        self.last_sel = [None] * n_layer  # (sel, cnt) of every layer in the last decode step

    def decode_step(self, ids: np.ndarray, k_caches, v_caches, cur_len: int) -> np.ndarray:
        """One decode step: writes position ``cur_len`` of every cache and
        returns logits [B, V] (model.py:79-157 with T = 1)."""
        s, dt = self.s, self.dtype
        b = ids.shape[0]
        hq, hkv, d = self.n_head, self.n_kv_head, self.head_dim
        x = s["embeddings.weight"][ids]  # [B, C]
        prev_f = None
        for li in range(self.n_layer):
            p = f"layers.{li}."
            h = rmsnorm(x, s[p + "attn_norm.weight"], self.eps).astype(dt)
            fc = (h @ s[p + "forecast.wf.weight"].T).reshape(b, 1, hkv, d)
            q = (h @ s[p + "attention.wq.weight"].T).reshape(b, 1, hq, d)
            k = (h @ s[p + "attention.wk.weight"].T).reshape(b, 1, hkv, d)
            v = (h @ s[p + "attention.wv.weight"].T).reshape(b, 1, hkv, d)
            q = apply_rope(q, self.cos, self.sin, cur_len).astype(dt)
            k = apply_rope(k, self.cos, self.sin, cur_len).astype(dt)
            kc, vc = k_caches[li], v_caches[li]
            kc[:, :, cur_len] = k[:, 0]
            vc[:, :, cur_len] = v[:, 0]
            L = cur_len + 1
            reps = None
            if prev_f is not None:
                reps = compress_blocks(kc[:, :, :L].transpose(0, 2, 1, 3), self.block_size, dt)
            sel, cnt = decode_select(prev_f, reps, L, self.block_size, self.top_k, b, hkv,
                                     "forecast", self.rule, dt)
            self.last_sel[li] = (sel, cnt)
            a = decode_attention(q[:, 0], kc, vc, sel, cnt, L, self.block_size, dtype=dt)
            x = x + a.reshape(b, hq * d).astype(dt) @ s[p + "attention.wo.weight"].T
            hn = rmsnorm(x, s[p + "ffn_norm.weight"], self.eps).astype(dt)
            gt = hn @ s[p + "ffn.w_gate.weight"].T
            up = hn @ s[p + "ffn.w_up.weight"].T
            x = x + ((gt / (1.0 + np.exp(-gt))) * up) @ s[p + "ffn.w_down.weight"].T
            prev_f = fc
        x = rmsnorm(x, s["final_norm.weight"], self.eps)
        return x @ s["embeddings.weight"].T

    def prefill(self, ids: np.ndarray, k_caches, v_caches) -> np.ndarray:
        """Prompt forward into empty caches (model.py:79-157 with T > 1 and
        T <= 8192): every layer runs the masked path (sparse.py:185-282) with
        the previous layer's forecast and writes positions 0..T-1 of its cache.
        ids [B, T]; returns the last position's logits [B, V]."""
        s, dt = self.s, self.dtype
        b, t = ids.shape
        hq, hkv, d = self.n_head, self.n_kv_head, self.head_dim
        x = s["embeddings.weight"][ids]  # [B, T, C]
        prev_f = None
        for li in range(self.n_layer):
            p = f"layers.{li}."
            h = rmsnorm(x, s[p + "attn_norm.weight"], self.eps).astype(dt)
            fc = (h @ s[p + "forecast.wf.weight"].T).reshape(b, t, hkv, d)
            q = apply_rope((h @ s[p + "attention.wq.weight"].T).reshape(b, t, hq, d), self.cos, self.sin, 0)
            k = apply_rope((h @ s[p + "attention.wk.weight"].T).reshape(b, t, hkv, d), self.cos, self.sin, 0)
            v = (h @ s[p + "attention.wv.weight"].T).reshape(b, t, hkv, d)
            q, k = q.astype(dt).transpose(0, 2, 1, 3), k.astype(dt).transpose(0, 2, 1, 3)
            v = v.transpose(0, 2, 1, 3)
            k_caches[li][:, :, :t] = k
            v_caches[li][:, :, :t] = v
            a = masked_prefill(q, k, v, prev_f, self.block_size, self.top_k, li, dtype=dt)
            x = x + a.transpose(0, 2, 1, 3).reshape(b, t, hq * d).astype(dt) @ s[p + "attention.wo.weight"].T
            hn = rmsnorm(x, s[p + "ffn_norm.weight"], self.eps).astype(dt)
            gt = hn @ s[p + "ffn.w_gate.weight"].T
            up = hn @ s[p + "ffn.w_up.weight"].T
            x = x + ((gt / (1.0 + np.exp(-gt))) * up) @ s[p + "ffn.w_down.weight"].T
            prev_f = fc
        x = rmsnorm(x[:, -1], s["final_norm.weight"], self.eps)
        return x @ s["embeddings.weight"].T
