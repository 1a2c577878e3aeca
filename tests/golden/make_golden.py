"""Generate the golden vectors in tests/golden/ by running the reference itself.

Run in a container where the reference checkout exists (it does not exist on
the GPU box; the committed .npz files travel instead):

    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

Every fixture is produced by the reference's own PyTorch code on CPU (fp32).
Inputs come from seeded generators (torch.manual_seed for BASELINE config 1,
numpy PCG64 elsewhere) so the tests regenerate them instead of storing them.
Where the reference's choice is implementation-defined (torch.topk tie order),
the indices it actually used are captured by wrapping ``gather_kv_blocks`` and
``scaled_dot_product_attention`` during the call, so attention parity can be
checked on identical index tensors.
"""

from __future__ import annotations

import argparse
import contextlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle.synthetic import SmallModelConfig, model_state, normal  # noqa: E402


def _setup(ref_path):
    sys.path.insert(0, ref_path)
    import torch  # noqa: F401
    torch_mod = __import__("torch")
    torch_mod.set_num_threads(max(1, os.cpu_count() or 1))
    return torch_mod


@contextlib.contextmanager
def capture(sp_mod, torch):
    """Record the (indices) passed to gather_kv_blocks and the attn_mask passed to
    SDPA while the reference runs."""
    rec = {"idx": [], "mask": []}
    orig_gather = sp_mod.gather_kv_blocks
    orig_sdpa = torch.nn.functional.scaled_dot_product_attention

    def gather(k, v, block_indices, block_size):
        rec["idx"].append(block_indices.clone())
        return orig_gather(k, v, block_indices, block_size)

    def sdpa(*a, **kw):
        rec["mask"].append(None if kw.get("attn_mask") is None else kw["attn_mask"].clone())
        return orig_sdpa(*a, **kw)

    sp_mod.gather_kv_blocks = gather
    torch.nn.functional.scaled_dot_product_attention = sdpa
    try:
        yield rec
    finally:
        sp_mod.gather_kv_blocks = orig_gather
        torch.nn.functional.scaled_dot_product_attention = orig_sdpa


def _attn(torch, block_size=64, top_k=8, layer_idx=1, mode=None, backend="sparse"):
    from model.config import ModelConfig
    from model.attention.sparse import SparseAttention
    cfg = ModelConfig(block_size=block_size, top_k_blocks=top_k, attention_backend=backend)
    a = SparseAttention(cfg, layer_idx=layer_idx, mode=mode)
    with torch.no_grad():
        a.wo.weight.copy_(torch.eye(768))
    return a


def config1(torch, out):
    """single-layer op, fp32, seed 0 (masked path, T=1024)."""
    torch.manual_seed(0)
    q = torch.randn(1, 1024, 12, 64)
    k = torch.randn(1, 1024, 4, 64)
    v = torch.randn(1, 1024, 4, 64)
    f = torch.randn(1, 1024, 4, 64)
    a = _attn(torch)
    with torch.no_grad():
        o = a._forward_masked_sdpa(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), 1024,
                                   forecast_vector=f)
        reps = a.compressor(k)
        scores, idx = a.selector(f, reps, 8, True)
    o = o[0].double().numpy()  # [1024, 768]
    np.savez(os.path.join(out, "config1.npz"),
             in_sums=np.array([t.double().sum().item() for t in (q, k, v, f)]),
             reps=reps.numpy(), scores=scores.numpy(), idx=idx.numpy().astype(np.int16),
             out_rows=o[::16].astype(np.float32), out_row_sum=o.sum(-1), out_row_abs=np.abs(o).sum(-1))


def compressor_cases(torch, out):
    from model.forecast import KVBlockCompressor
    c = KVBlockCompressor(block_size=64, head_dim=64, forecast_dim=64)
    res = {}
    for i, t in enumerate([1, 63, 64, 65, 129, 640, 641]):
        k = torch.from_numpy(normal((2, t, 4, 64), seed=100 + i))
        with torch.no_grad():
            res[f"T{t}"] = c(k).numpy()
    # the reference's own test geometry (tests/test_forecast.py:53-68): block 16, D 32
    c16 = KVBlockCompressor(block_size=16, head_dim=32, forecast_dim=32)
    k = torch.from_numpy(normal((2, 50, 4, 32), seed=199))
    with torch.no_grad():
        res["bs16_T50"] = c16(k).numpy()
    np.savez(os.path.join(out, "compressor.npz"), **res)


SELECTOR_CASES = [
    # name, B, Tq, H, D, N_b, block, top_k, causal, seed
    ("reftest", 2, 32, 2, 16, 4, 8, 2, True, 300),
    ("decode257", 1, 1, 4, 64, 257, 64, 8, True, 301),
    ("decode16", 2, 1, 4, 64, 16, 64, 8, True, 302),
    ("chunk40", 2, 64, 4, 64, 40, 64, 8, False, 303),
    ("causal300", 1, 300, 4, 64, 5, 64, 8, True, 304),
    ("topk_gt_nb", 1, 70, 4, 64, 3, 64, 8, True, 305),
]


def selector_cases(torch, out):
    from model.forecast import ForecastBlockSelector
    res = {}
    for name, b, tq, h, d, nb, bs, k, causal, seed in SELECTOR_CASES:
        f = torch.from_numpy(normal((b, tq, h, d), seed=seed))
        r = torch.from_numpy(normal((b, nb, h, d), seed=seed + 1000))
        sel = ForecastBlockSelector(block_size=bs, forecast_dim=d)
        with torch.no_grad():
            s, i = sel(f, r, k, causal)
        res[name + "_scores"] = s.numpy()
        res[name + "_idx"] = i.numpy().astype(np.int32)
    np.savez(os.path.join(out, "selector.npz"), **res)


DECODE_CASES = [
    # name, B, L, forecast?, seed
    ("L600", 2, 600, True, 400),
    ("L641", 2, 641, True, 401),
    ("L1000", 2, 1000, True, 402),
    ("L1024", 2, 1024, True, 403),
    ("L1000_static", 2, 1000, False, 404),
]


def decode_cases(torch, out):
    import model.attention.sparse as sp
    a = _attn(torch)
    res = {}
    for name, b, L, with_f, seed in DECODE_CASES:
        q = torch.from_numpy(normal((b, 12, 1, 64), seed=seed))
        k = torch.from_numpy(normal((b, 4, L, 64), seed=seed + 1))
        v = torch.from_numpy(normal((b, 4, L, 64), seed=seed + 2))
        f = torch.from_numpy(normal((b, 1, 4, 64), seed=seed + 3)) if with_f else None
        with capture(sp, torch) as rec, torch.no_grad():
            o = a._forward_decode_gather(q, k, v, L, forecast_vector=f)
        res[name + "_out"] = o.reshape(b, 12, 64).numpy()
        if rec["idx"]:
            idx = rec["idx"][0].numpy()
            m = rec["mask"][0].numpy()  # [B, 4, 1, MS*64]
            valid = m[:, ::3, 0, ::64] == 0  # mask was repeated x3 over query heads
            res[name + "_sel"] = idx.astype(np.int32)
            res[name + "_valid"] = valid
    np.savez(os.path.join(out, "decode.npz"), **res)


MASKED_CASES = [
    # name, B, T, layer_idx, mode, with_forecast, seed
    ("T700", 2, 700, 1, "forecast", True, 500),
    ("T700_static", 2, 700, 1, "static", False, 501),
    ("T700_layer0", 2, 700, 0, "forecast", True, 502),
    ("T128", 1, 128, 1, "forecast", True, 503),
]


def masked_cases(torch, out):
    res = {}
    for name, b, t, li, mode, with_f, seed in MASKED_CASES:
        a = _attn(torch, layer_idx=li, mode=mode)
        q = torch.from_numpy(normal((b, 12, t, 64), seed=seed))
        k = torch.from_numpy(normal((b, 4, t, 64), seed=seed + 1))
        v = torch.from_numpy(normal((b, 4, t, 64), seed=seed + 2))
        f = torch.from_numpy(normal((b, t, 4, 64), seed=seed + 3)) if with_f else None
        with torch.no_grad():
            o = a._forward_masked_sdpa(q, k, v, t, forecast_vector=f)
        o = o.reshape(b, t, 12, 64).double().numpy()
        res[name + "_rows"] = o[:, ::31].astype(np.float32)
        res[name + "_row_sum"] = o.sum(axis=(2, 3))
    np.savez(os.path.join(out, "masked.npz"), **res)


CHUNKED_CASES = [
    # name, B, T, with_forecast, mode, seed
    ("T1024", 1, 1024, True, "forecast", 600),
    ("T700", 2, 700, True, "forecast", 601),
    ("T900_static", 1, 900, False, "static", 602),
]


def chunked_cases(torch, out):
    import model.attention.sparse as sp
    res = {}
    for name, b, t, with_f, mode, seed in CHUNKED_CASES:
        a = _attn(torch, mode=mode)
        q = torch.from_numpy(normal((b, 12, t, 64), seed=seed))
        k = torch.from_numpy(normal((b, 4, t, 64), seed=seed + 1))
        v = torch.from_numpy(normal((b, 4, t, 64), seed=seed + 2))
        f = torch.from_numpy(normal((b, t, 4, 64), seed=seed + 3)) if with_f else None
        with capture(sp, torch) as rec, torch.no_grad():
            o = a._forward_chunked_gather(q, k, v, t, forecast_vector=f)
        o = o.reshape(b, t, 12, 64).double().numpy()
        sel = np.stack([i.numpy() for i in rec["idx"]], axis=2)  # [B, H, N_b, MS]
        # slot validity: first token of a listed block is unmasked for the block's last query
        valid = np.stack([(m[:, ::3, -1, ::64] == 0).numpy() for m in rec["mask"]], axis=2)
        res[name + "_sel"] = sel.astype(np.int32)
        res[name + "_valid"] = valid
        res[name + "_rows"] = o[:, ::31].astype(np.float32)
        res[name + "_row_sum"] = o.sum(axis=(2, 3))
    np.savez(os.path.join(out, "chunked.npz"), **res)


def prefetch_cases(torch, out):
    """AsyncForecastOffloadAttention.prefetch selection (async_offload.py:190-260),
    captured from the attributes it stores (CPU: no stream, no event)."""
    from model.config import ModelConfig
    from model.attention.async_offload import AsyncForecastOffloadAttention, AsyncOffloadedKVCache
    res = {}
    for name, b, L, li, seed in [("L1000", 2, 1000, 1, 700), ("L500", 1, 500, 1, 701),
                                 ("L1000_layer0", 1, 1000, 0, 702)]:
        cfg = ModelConfig(block_size=64, top_k_blocks=8, attention_backend="async_offload")
        attn = AsyncForecastOffloadAttention(cfg, layer_idx=li)
        cache = AsyncOffloadedKVCache(b, 2048, 4, 64, torch.device("cpu"), torch.float32, pin_memory=False)
        k = torch.from_numpy(normal((b, L, 4, 64), seed=seed))
        v = torch.from_numpy(normal((b, L, 4, 64), seed=seed + 1))
        cache.update(k, v)
        f = torch.from_numpy(normal((b, 1, 4, 64), seed=seed + 2))
        with torch.no_grad():
            attn.prefetch(f, cache)
        res[name + "_small"] = np.array(attn.prefetched_is_small_context)
        if attn.prefetched_sel_indices is not None:
            res[name + "_sel"] = attn.prefetched_sel_indices.numpy().astype(np.int32)
            res[name + "_val"] = attn.prefetched_val.numpy()
    np.savez(os.path.join(out, "prefetch.npz"), **res)


MODEL_STEPS = [0, 1, 63, 64, 65, 300, 639]


def model_cases(torch, out):
    """Full SparDAResearchModel decode, token by token from an empty cache, with
    the seeded numpy weights of oracle/synthetic.py.  Up to 640 cached tokens
    every step takes the dense fallback (sparse.py:113-123), so the logits are
    free of the tie hazards."""
    from model.config import ModelConfig
    from model.model import SparDAResearchModel
    from model.attention.base import KVCache
    sc = SmallModelConfig()
    cfg = ModelConfig(vocab_size=sc.vocab_size, n_layer=sc.n_layer, context_length=sc.context_length,
                      block_size=sc.block_size, top_k_blocks=sc.top_k_blocks, attention_backend="sparse")
    m = SparDAResearchModel(cfg).eval()
    st = model_state(sc, seed=7)
    m.load_state_dict({k: torch.from_numpy(v) for k, v in st.items()}, strict=True)
    b = 2
    ids = np.random.default_rng(8).integers(0, sc.vocab_size, size=(b, max(MODEL_STEPS) + 1))
    caches = [KVCache(b, 1024, 4, 64, torch.device("cpu"), torch.float32) for _ in range(sc.n_layer)]
    logits = {}
    with torch.no_grad():
        for s in range(max(MODEL_STEPS) + 1):
            o = m(torch.from_numpy(ids[:, s:s + 1]), kv_caches=caches)["logits"][:, 0]
            if s in MODEL_STEPS:
                logits[f"step{s}"] = o.numpy()
    np.savez(os.path.join(out, "model_decode.npz"), ids=ids.astype(np.int32), **logits)


@contextlib.contextmanager
def absolute_rule():
    """Decode-time selection by the query's absolute position, produced by the
    reference's own ForecastBlockSelector (model/forecast.py:89-130).  In
    decode the reference passes one forecast row with is_causal=True, so its
    mask (forecast.py:120-126) compares blocks with row index 0.  Placed at its
    absolute row L-1 instead, the same mask hides blocks j > (L-1) // bs, i.e.
    none of the cached blocks; the wrapper therefore calls the original method
    with is_causal=False for single-row calls.  Multi-row calls (prefill) are
    passed through unchanged."""
    from model.forecast import ForecastBlockSelector
    orig = ForecastBlockSelector.forward

    def forward(self, forecast, block_reps, top_k, is_causal=True):
        if forecast.shape[1] == 1:
            is_causal = False
        return orig(self, forecast, block_reps, top_k, is_causal)

    ForecastBlockSelector.forward = forward
    try:
        yield
    finally:
        ForecastBlockSelector.forward = orig


DECODE_BIG_CASES = [
    # name, B, L (tokens after the append), rule, seed
    ("L16385_abs", 2, 16385, "absolute", 800),
    ("L16448_abs", 2, 16448, "absolute", 801),
    ("L16400_ref", 2, 16400, "reference", 802),
    ("L1000_abs", 2, 1000, "absolute", 803),
    ("L641_abs", 2, 641, "absolute", 804),
]


def decode_big_inputs(b, L, seed):
    """Inputs of one decode step at BASELINE config-2 lengths, pre-RoPE: the
    cached prefix K/V [B, L-1, 4, 64] (already rotated, as a cache holds them),
    the new token's q [B, 12, 64], k and v [B, 4, 64], and layer L-1's
    forecast [B, 1, 4, 64]."""
    return (normal((b, L - 1, 4, 64), seed=seed), normal((b, L - 1, 4, 64), seed=seed + 1),
            normal((b, 12, 64), seed=seed + 2), normal((b, 4, 64), seed=seed + 3),
            normal((b, 4, 64), seed=seed + 4), normal((b, 1, 4, 64), seed=seed + 5))


def decode_big_cases(torch, out):
    """One decode step of SparseAttention._forward_decode_gather
    (model/attention/sparse.py:99-183) at up to 16,448 cached tokens, with the
    new token rotated by the reference's RotaryEmbedding (model/rope.py:34-98)
    at its position and appended to the cache first, as SparseAttention.forward
    does (sparse.py:390-399).  Captures the selected lists it gathered."""
    import model.attention.sparse as sp
    from model.rope import RotaryEmbedding
    a = _attn(torch)
    res = {}
    for name, b, L, rule, seed in DECODE_BIG_CASES:
        kp, vp, q, kn, vn, f = (torch.from_numpy(x) for x in decode_big_inputs(b, L, seed))
        rot = RotaryEmbedding(64, L + 64)
        qr, kr = rot(q[:, None], kn[:, None], offset=L - 1)
        k_all = torch.cat([kp, kr], dim=1).transpose(1, 2)  # [B, 4, L, 64]
        v_all = torch.cat([vp, vn[:, None]], dim=1).transpose(1, 2)
        ctx = absolute_rule() if rule == "absolute" else contextlib.nullcontext()
        with ctx, capture(sp, torch) as rec, torch.no_grad():
            o = a._forward_decode_gather(qr.transpose(1, 2), k_all, v_all, L, forecast_vector=f)
        res[name + "_out"] = o.reshape(b, 12, 64).numpy()
        res[name + "_sel"] = rec["idx"][0].numpy().astype(np.int32)
        res[name + "_valid"] = rec["mask"][0].numpy()[:, ::3, 0, ::64] == 0
    np.savez(os.path.join(out, "decode_big.npz"), **res)


MODEL_SPARSE_PREFILL = 700
MODEL_SPARSE_STEPS = 72        # decode positions 700..771: 11 to 13 blocks, past the dense fallback
MODEL_SPARSE_LOGIT_EVERY = 4


def model_sparse_cases(torch, out):
    """Full SparDAResearchModel with the sparse backend and the absolute
    decode rule (absolute_rule above): a 700-token prefill (masked path,
    sparse.py:185-282), then 72 decode steps in the sparse regime, where layer
    L's forecast selects layer L+1's blocks (model/model.py:100-139,
    model/transformer.py:76-131).  Stores the prefill's last logits, the logits
    of every 4th decode step and every layer's selected lists."""
    import model.attention.sparse as sp
    from model.config import ModelConfig
    from model.model import SparDAResearchModel
    from model.attention.base import KVCache
    sc = SmallModelConfig()
    cfg = ModelConfig(vocab_size=sc.vocab_size, n_layer=sc.n_layer, context_length=sc.context_length,
                      block_size=sc.block_size, top_k_blocks=sc.top_k_blocks, attention_backend="sparse")
    m = SparDAResearchModel(cfg).eval()
    m.load_state_dict({k: torch.from_numpy(v) for k, v in model_state(sc, seed=9).items()}, strict=True)
    b, p, n = 2, MODEL_SPARSE_PREFILL, MODEL_SPARSE_STEPS
    ids = np.random.default_rng(10).integers(0, sc.vocab_size, size=(b, p + n))
    caches = [KVCache(b, 1024, 4, 64, torch.device("cpu"), torch.float32) for _ in range(sc.n_layer)]
    res = {"ids": ids.astype(np.int32)}
    sels, valids = [], []
    with absolute_rule(), torch.no_grad():
        o = m(torch.from_numpy(ids[:, :p]), kv_caches=caches)["logits"]
        res["prefill_last"] = o[:, -1].numpy()
        for s in range(n):
            with capture(sp, torch) as rec:
                o = m(torch.from_numpy(ids[:, p + s:p + s + 1]), kv_caches=caches)["logits"][:, 0]
            if s % MODEL_SPARSE_LOGIT_EVERY == 0 or s == n - 1:
                res[f"step{s}"] = o.numpy()
            assert len(rec["idx"]) == sc.n_layer
            sels.append(np.stack([i.numpy() for i in rec["idx"]]))           # [layers, B, 4, MS]
            valids.append(np.stack([(mk.numpy()[:, ::3, 0, ::64] == 0) for mk in rec["mask"]]))
    res["sel"] = np.stack(sels).astype(np.int16)   # [steps, layers, B, 4, MS]
    res["valid"] = np.stack(valids)
    np.savez(os.path.join(out, "model_sparse.npz"), **res)


CHUNKED_BIG = ("T32768", 1, 32768, 610)
CHUNKED_BIG_ROW_EVERY = 257


def chunked_big_cases(torch, out):
    """_forward_chunked_gather (sparse.py:284-364) at BASELINE config 3's
    length (T=32,768, 512 q-blocks), fp32: the per-q-block lists the reference
    gathered (its truncation of the union is implementation-defined, so
    attention parity is checked on these lists), every 257th output row and
    every row's sum."""
    import model.attention.sparse as sp
    name, b, t, seed = CHUNKED_BIG
    a = _attn(torch)
    q = torch.from_numpy(normal((b, 12, t, 64), seed=seed))
    k = torch.from_numpy(normal((b, 4, t, 64), seed=seed + 1))
    v = torch.from_numpy(normal((b, 4, t, 64), seed=seed + 2))
    f = torch.from_numpy(normal((b, t, 4, 64), seed=seed + 3))
    with capture(sp, torch) as rec, torch.no_grad():
        o = a._forward_chunked_gather(q, k, v, t, forecast_vector=f)
    o = o.reshape(b, t, 12, 64).double().numpy()
    sel = np.stack([i.numpy() for i in rec["idx"]], axis=2)
    valid = np.stack([(m[:, ::3, -1, ::64] == 0).numpy() for m in rec["mask"]], axis=2)
    np.savez(os.path.join(out, "chunked_big.npz"), sel=sel.astype(np.int16), valid=valid,
             rows=o[:, ::CHUNKED_BIG_ROW_EVERY].astype(np.float32), row_sum=o.sum(axis=(2, 3)))


def prefetch_abs_cases(torch, out):
    """AsyncForecastOffloadAttention.prefetch (async_offload.py:190-260) with
    the absolute decode rule: the blocks it selects before the new token is
    appended, from prototypes that cover the cached tokens only."""
    from model.config import ModelConfig
    from model.attention.async_offload import AsyncForecastOffloadAttention, AsyncOffloadedKVCache
    res = {}
    with absolute_rule():
        for name, b, L, li, seed in PREFETCH_ABS_CASES:
            cfg = ModelConfig(block_size=64, top_k_blocks=8, attention_backend="async_offload")
            attn = AsyncForecastOffloadAttention(cfg, layer_idx=li)
            cache = AsyncOffloadedKVCache(b, L + 64, 4, 64, torch.device("cpu"), torch.float32, pin_memory=False)
            k = torch.from_numpy(normal((b, L, 4, 64), seed=seed))
            v = torch.from_numpy(normal((b, L, 4, 64), seed=seed + 1))
            cache.update(k, v)
            f = torch.from_numpy(normal((b, 1, 4, 64), seed=seed + 2))
            with torch.no_grad():
                attn.prefetch(f, cache)
            res[name + "_small"] = np.array(attn.prefetched_is_small_context)
            if attn.prefetched_sel_indices is not None:
                res[name + "_sel"] = attn.prefetched_sel_indices.numpy().astype(np.int32)
                res[name + "_val"] = attn.prefetched_val.numpy()
    np.savez(os.path.join(out, "prefetch_abs.npz"), **res)


ASYNC_DECODE_CASES = [
    # name, B, cached tokens before the first step, seed
    ("L1000", 2, 1000, 740),
    ("L1023", 2, 1023, 741),
    ("L3000", 2, 3000, 742),
]
ASYNC_DECODE_STEPS = 3


def async_attn_weights(seed):
    """wq, wk, wv, wo of one attention layer, N(0, 0.02), numpy PCG64."""
    return {"wq": normal((768, 768), seed=seed, scale=0.02), "wk": normal((256, 768), seed=seed + 1, scale=0.02),
            "wv": normal((256, 768), seed=seed + 2, scale=0.02), "wo": normal((768, 768), seed=seed + 3, scale=0.02)}


def async_decode_inputs(b, L, seed, step):
    """Cached K/V [B, L, 4, 64] (before the first step) and step `step`'s
    x [B, 1, 768] and forecast [B, 1, 4, 64]."""
    return (normal((b, L, 4, 64), seed=seed + 10), normal((b, L, 4, 64), seed=seed + 11),
            normal((b, 1, 768), seed=seed + 20 + step), normal((b, 1, 4, 64), seed=seed + 30 + step))


def async_decode_cases(torch, out):
    """AsyncForecastOffloadAttention decode steps (model/attention/async_offload.py:
    170-519) with the absolute rule: prefetch (selection before the append,
    :241-260), then the decode that consumes it (:296-390, validity mask
    :466-490).  On CPU the reference creates no transfer event, which would
    route the decode to its synchronous fallback (:392-460); a placeholder
    event object routes it through the prefetch-consuming branch (the event is
    only used for a stream wait that the CPU path skips, :324-325).
    Three consecutive steps per case; the output, and the prefetched lists."""
    from model.config import ModelConfig
    from model.attention.async_offload import AsyncForecastOffloadAttention, AsyncOffloadedKVCache
    from model.rope import RotaryEmbedding

    class _Placeholder:
        pass

    res = {}
    with absolute_rule():
        for name, b, L, seed in ASYNC_DECODE_CASES:
            cfg = ModelConfig(block_size=64, top_k_blocks=8, attention_backend="async_offload")
            attn = AsyncForecastOffloadAttention(cfg, layer_idx=1)
            w = async_attn_weights(seed)
            with torch.no_grad():
                for nm, val in w.items():
                    getattr(attn, nm).weight.copy_(torch.from_numpy(val))
            cache = AsyncOffloadedKVCache(b, L + 64, 4, 64, torch.device("cpu"), torch.float32, pin_memory=False)
            k, v, _, _ = async_decode_inputs(b, L, seed, 0)
            cache.update(torch.from_numpy(k), torch.from_numpy(v))
            rot = RotaryEmbedding(64, L + 128)
            for s in range(ASYNC_DECODE_STEPS):
                _, _, x, f = async_decode_inputs(b, L, seed, s)
                with torch.no_grad():
                    attn.prefetch(torch.from_numpy(f), cache)
                    assert not attn.prefetched_is_small_context
                    res[f"{name}_s{s}_sel"] = attn.prefetched_sel_indices.numpy().astype(np.int32)
                    res[f"{name}_s{s}_val"] = attn.prefetched_val.numpy()
                    attn.prefetch_event = _Placeholder()
                    o = attn(torch.from_numpy(x), rot, kv_cache=cache, forecast_vector=torch.from_numpy(f))
                res[f"{name}_s{s}_out"] = o.numpy()
    np.savez(os.path.join(out, "async_decode.npz"), **res)


PREFETCH_ABS_CASES = [
    # name, B, cached tokens, layer_idx, seed
    ("L1000", 2, 1000, 1, 720),
    ("L1023", 2, 1023, 1, 721),
    ("L1024", 2, 1024, 1, 722),
    ("L3000", 2, 3000, 1, 723),
]


BACKWARD_CASES = [
    # name, B, T, layer_idx, mode, with_forecast, chunked, seed
    ("T256", 1, 256, 1, "forecast", True, False, 800),
    ("T300_static", 1, 300, 1, "static", False, False, 801),
    ("T200_layer0", 1, 200, 0, "forecast", True, False, 802),
    ("T640_chunked", 1, 640, 1, "forecast", True, True, 803),
]


def backward_cases(torch, out):
    """Gradients autograd takes through the reference's masked and chunked
    attention cores (sparse.py:185-364) for loss = sum(out * w): q, k, v
    gradients, row-subsampled, plus their full per-row sums.  The chunked case
    has N_b = 10 = MS, so its unions are never truncated."""
    res = {}
    for name, b, t, li, mode, with_f, chunked, seed in BACKWARD_CASES:
        a = _attn(torch, layer_idx=li, mode=mode)
        q = torch.from_numpy(normal((b, 12, t, 64), seed=seed)).requires_grad_(True)
        k = torch.from_numpy(normal((b, 4, t, 64), seed=seed + 1)).requires_grad_(True)
        v = torch.from_numpy(normal((b, 4, t, 64), seed=seed + 2)).requires_grad_(True)
        f = torch.from_numpy(normal((b, t, 4, 64), seed=seed + 3)) if with_f else None
        w = torch.from_numpy(normal((b, t, 768), seed=seed + 4))
        if chunked:
            o = a._forward_chunked_gather(q, k, v, t, forecast_vector=f)
        else:
            o = a._forward_masked_sdpa(q, k, v, t, forecast_vector=f)
        (o.reshape(b, t, 768) * w).sum().backward()
        gq, gk, gv = (x.grad.double().numpy() for x in (q, k, v))
        res[name + "_dq_rows"] = gq[:, :, ::29].astype(np.float32)
        res[name + "_dk_rows"] = gk[:, :, ::13].astype(np.float32)
        res[name + "_dv_rows"] = gv[:, :, ::13].astype(np.float32)
        res[name + "_dq_sum"] = gq.sum(-1).astype(np.float32)
        res[name + "_dk_sum"] = gk.sum(-1).astype(np.float32)
        res[name + "_dv_sum"] = gv.sum(-1).astype(np.float32)
    np.savez(os.path.join(out, "backward.npz"), **res)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    torch = _setup(args.reference)
    jobs = [config1, compressor_cases, selector_cases, decode_cases, masked_cases, chunked_cases,
            prefetch_cases, model_cases, decode_big_cases, model_sparse_cases, chunked_big_cases,
            prefetch_abs_cases, async_decode_cases, backward_cases]
    for job in jobs:
        if args.only and job.__name__ not in args.only.split(","):
            continue
        job(torch, args.out)
        print("wrote", job.__name__)


if __name__ == "__main__":
    main()
