"""Parity of the sm_100a kernels (through the C ABI) with the CPU oracle and
with golden vectors the reference produced.  Needs a B200.

Tolerances: fp32 attention max-abs 1e-4, bf16 attention max-abs 2e-2 (the
north-star gates); prototypes and selector scores in fp32 to 1e-5 relative;
block indices bit-exact wherever the selected score is finite and not within
1e-5 (relative) of its neighbour in the order."""

import math

import numpy as np
import pytest
import torch

import local_research_small_language_model_b200 as sd
from local_research_small_language_model_b200 import ops
from local_research_small_language_model_b200.rope import precompute_rope_freqs
from oracle import sparda_oracle as O
from oracle.synthetic import normal

pytestmark = pytest.mark.gpu

ATOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}


def t(x, dev, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev, dtype)


def n(x):
    return x.detach().float().cpu().numpy()


def _no_device_errors(dev):
    torch.cuda.synchronize()
    ops.check_device_errors(dev)


# ------------------------------------------------------------------ compressor
@pytest.mark.parametrize("tt", [1, 63, 64, 65, 129, 640, 641])
def test_compressor_vs_reference_golden(dev, golden, tt):
    i = [1, 63, 64, 65, 129, 640, 641].index(tt)
    k = normal((2, tt, 4, 64), seed=100 + i)
    out = sd.KVBlockCompressor(64, 64, 64)(t(k, dev))
    np.testing.assert_allclose(n(out), golden("compressor")[f"T{tt}"], rtol=1e-5, atol=1e-6)


def test_compressor_strided_bf16_and_small_geometry(dev, golden):
    k = normal((2, 50, 4, 32), seed=199)
    out = sd.KVBlockCompressor(16, 32, 32)(t(k, dev))
    np.testing.assert_allclose(n(out), golden("compressor")["bs16_T50"], rtol=1e-5, atol=1e-6)
    kb = t(normal((3, 1000, 4, 64), seed=5), dev, torch.bfloat16)
    kv = kb.transpose(1, 2).contiguous().transpose(1, 2)  # non-contiguous [B,T,H,D] view
    ref = O.compress_blocks(n(kb), 64)
    np.testing.assert_allclose(n(ops.compress_blocks(kv, 64)), ref, rtol=1e-5, atol=1e-5)


# ------------------------------------------------------------------ selector
def _finite_slots_equal(scores, ref_idx, idx, gap=1e-5):
    """Equality wherever the reference slot is finite and not a near-tie."""
    vals = np.take_along_axis(scores, ref_idx.astype(np.int64), axis=-1)
    ok = np.isfinite(vals)
    nxt = np.concatenate([vals[..., 1:], np.full(vals.shape[:-1] + (1,), -np.inf)], axis=-1)
    prv = np.concatenate([np.full(vals.shape[:-1] + (1,), np.inf), vals[..., :-1]], axis=-1)
    scale = np.maximum(np.abs(vals), 1e-30)
    with np.errstate(invalid="ignore"):  # -inf - -inf at the non-finite slots, which `ok` drops
        clear = ((vals - nxt) > gap * scale) & ((prv - vals) > gap * scale)
    sel = ok & clear
    return np.array_equal(ref_idx[sel], idx[sel]), sel.mean()


def test_topk_bit_exact_on_reference_scores(dev, golden):
    """Top-k fed the reference's own fp32 score tensors: bit-exact on finite slots."""
    g = golden("config1")
    ref_s, ref_i = g["scores"], g["idx"].astype(np.int64)
    _, idx = ops.topk_rows(t(ref_s, dev), 8)
    vals = np.take_along_axis(ref_s, ref_i, axis=-1)
    fin = np.isfinite(vals)
    assert np.array_equal(n(idx).astype(np.int64)[fin], ref_i[fin])
    sel = golden("selector")
    for case in ["reftest", "decode257", "decode16", "chunk40", "causal300", "topk_gt_nb"]:
        s, i = sel[case + "_scores"], sel[case + "_idx"].astype(np.int64)
        _, idx = ops.topk_rows(t(s, dev), i.shape[-1])
        v = np.take_along_axis(s, i, axis=-1)
        fin = np.isfinite(v)
        assert np.array_equal(n(idx).astype(np.int64)[fin], i[fin]), case
        # the -inf slots follow the documented rule: ascending block index
        np.testing.assert_array_equal(n(idx).astype(np.int64), O.topk_desc(s, i.shape[-1]))


def test_selector_config1_end_to_end(dev, golden):
    import torch as th
    th.manual_seed(0)
    q = th.randn(1, 1024, 12, 64)
    k = th.randn(1, 1024, 4, 64)
    th.randn(1, 1024, 4, 64)
    f = th.randn(1, 1024, 4, 64)
    g = golden("config1")
    reps = sd.KVBlockCompressor(64, 64, 64)(k.to(dev))
    np.testing.assert_allclose(n(reps), g["reps"], rtol=1e-5, atol=1e-6)
    scores, idx = sd.ForecastBlockSelector(64, 64)(f.to(dev), reps, 8, True)
    ref = g["scores"]
    assert np.array_equal(np.isfinite(n(scores)), np.isfinite(ref))
    fin = np.isfinite(ref)
    np.testing.assert_allclose(n(scores)[fin], ref[fin], rtol=1e-5, atol=1e-5)
    same, frac = _finite_slots_equal(ref, g["idx"], n(idx).astype(np.int64))
    assert same and frac > 0.5


@pytest.mark.parametrize("case", ["reftest", "decode257", "decode16", "chunk40", "causal300", "topk_gt_nb"])
def test_selector_cases(dev, golden, case):
    from tests.golden.make_golden import SELECTOR_CASES
    name, b, tq, h, d, nb, bs, k, causal, seed = [c for c in SELECTOR_CASES if c[0] == case][0]
    g = golden("selector")
    f = normal((b, tq, h, d), seed=seed)
    r = normal((b, nb, h, d), seed=seed + 1000)
    scores, idx = ops.select_blocks(t(f, dev), t(r, dev), k, bs, causal)
    ref_s, ref_i = g[case + "_scores"], g[case + "_idx"]
    fin = np.isfinite(ref_s)
    assert np.array_equal(np.isfinite(n(scores)), fin)
    np.testing.assert_allclose(n(scores)[fin], ref_s[fin], rtol=1e-5, atol=1e-5)
    same, _ = _finite_slots_equal(ref_s, ref_i, n(idx).astype(np.int64))
    assert same
    # -inf fills follow the ascending-index rule, exactly as the oracle
    np.testing.assert_array_equal(n(idx).astype(np.int64), O.topk_desc(n(scores), idx.shape[-1]))


def test_selector_large_prefill_rows(dev):
    """Prefill-sized selector (T=4096, N_b=64, causal and not) vs the oracle."""
    f = normal((1, 4096, 4, 64), seed=11)
    r = normal((1, 64, 4, 64), seed=12)
    for causal in (True, False):
        scores, idx = ops.select_blocks(t(f, dev), t(r, dev), 8, 64, causal)
        ref_s, ref_i = O.select_blocks(f, r, 8, 64, causal)
        fin = np.isfinite(ref_s)
        np.testing.assert_allclose(n(scores)[fin], ref_s[fin], rtol=1e-5, atol=1e-5)
        same, frac = _finite_slots_equal(ref_s, ref_i, n(idx).astype(np.int64))
        assert same and frac > 0.9


@pytest.mark.parametrize("nb,tq,causal,k", [(300, 1000, False, 8), (300, 1000, True, 8), (129, 200, False, 5)])
def test_selector_many_blocks_tie_order(dev, nb, tq, causal, k):
    """Many-row selector over several 128-block chunks (partial last chunk):
    scores vs the oracle, and indices exactly the top-k of the kernel's own
    scores under the value-desc / index-asc rule (-inf fills included)."""
    f = normal((2, tq, 4, 64), seed=21)
    r = normal((2, nb, 4, 64), seed=22)
    scores, idx = ops.select_blocks(t(f, dev), t(r, dev), k, 64, causal)
    ref_s, _ = O.select_blocks(f, r, k, 64, causal)
    fin = np.isfinite(ref_s)
    assert np.array_equal(np.isfinite(n(scores)), fin)
    np.testing.assert_allclose(n(scores)[fin], ref_s[fin], rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(n(idx).astype(np.int64), O.topk_desc(n(scores), k))
    _, idx2 = ops.select_blocks(t(f, dev), t(r, dev), k, 64, causal, return_scores=False)
    assert torch.equal(idx, idx2)


# ------------------------------------------------------------------ gather
def test_gather_kv_blocks_vs_oracle(dev):
    k = normal((2, 4, 1000, 64), seed=21)
    v = normal((2, 4, 1000, 64), seed=22)
    idx = np.random.default_rng(3).integers(0, 16, size=(2, 4, 10))
    for dt in (torch.float32, torch.bfloat16):
        kg, vg = sd.gather_kv_blocks(t(k, dev, dt), t(v, dev, dt), t(idx, dev, torch.int64), 64)
        rk, rv = O.gather_kv_blocks(n(t(k, dev, dt)), n(t(v, dev, dt)), idx, 64)
        assert np.array_equal(n(kg), rk) and np.array_equal(n(vg), rv)


# ------------------------------------------------------------------ decode
def _ref_lists(sel, valid):
    lead = sel.shape[:-1]
    out = np.full(lead + (sel.shape[-1],), -1, dtype=np.int64)
    cnt = np.zeros(lead, dtype=np.int64)
    for ix in np.ndindex(*lead):
        ids = np.sort(sel[ix][valid[ix]])
        out[ix][:len(ids)] = ids
        cnt[ix] = len(ids)
    return out, cnt


@pytest.mark.parametrize("case", ["L600", "L641", "L1000", "L1024", "L1000_static"])
def test_decode_attention_vs_reference_golden(dev, golden, case):
    """Attention on the reference's own index tensor: fp32 max-abs 1e-4."""
    from tests.golden.make_golden import DECODE_CASES
    name, b, L, with_f, seed = [c for c in DECODE_CASES if c[0] == case][0]
    g = golden("decode")
    q = normal((b, 12, 1, 64), seed=seed)[:, :, 0]
    k = normal((b, 4, L, 64), seed=seed + 1)
    v = normal((b, 4, L, 64), seed=seed + 2)
    if case + "_sel" in g:
        sel, cnt = _ref_lists(g[case + "_sel"], g[case + "_valid"])
    else:
        sel, cnt = O.decode_select(None, None, L, 64, 8, b, 4)
    out = ops.decode_attention(t(q, dev), t(k, dev), t(v, dev), t(sel, dev, torch.int32), t(cnt, dev, torch.int32),
                               L, 64)
    _no_device_errors(dev)
    np.testing.assert_allclose(n(out), g[case + "_out"], rtol=0, atol=1e-4)


@pytest.mark.parametrize("rule", ["reference", "absolute"])
@pytest.mark.parametrize("L", [1, 65, 640, 641, 1000, 1024, 4097])
def test_decode_select_vs_oracle(dev, rule, L):
    b = 3
    k = normal((b, L, 4, 64), seed=L)
    f = normal((b, 1, 4, 64), seed=L + 1)
    reps = O.compress_blocks(k, 64)
    sel, cnt = ops.decode_select(t(f, dev), t(reps, dev), L, b, 4, 64, 64, 8, rule)
    rs, rc = O.decode_select(f, reps, L, 64, 8, b, 4, "forecast", rule)
    assert np.array_equal(n(cnt).astype(np.int64), rc)
    for ix in np.ndindex(b, 4):
        assert list(n(sel)[ix][:rc[ix]].astype(np.int64)) == list(rs[ix][:rc[ix]])
    sel, cnt = ops.decode_select(None, None, L, b, 4, 64, 64, 8, rule, device=dev)
    rs, rc = O.decode_select(None, None, L, 64, 8, b, 4, "forecast", rule)
    assert np.array_equal(n(cnt).astype(np.int64), rc)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("geom", [(12, 4), (8, 2), (4, 4)])
def test_decode_attention_vs_oracle(dev, dt, geom):
    hq, hkv = geom
    b, L = 3, 3000
    q = normal((b, hq, 64), seed=31)
    kc = normal((b, hkv, 3072, 64), seed=32)
    vc = normal((b, hkv, 3072, 64), seed=33)
    f = normal((b, 1, hkv, 64), seed=34)
    qd, kd, vd = t(q, dev, dt), t(kc, dev, dt), t(vc, dev, dt)
    reps = O.compress_blocks(n(kd)[:, :, :L].transpose(0, 2, 1, 3), 64)
    sel, cnt = O.decode_select(f, reps, L, 64, 8, b, hkv, "forecast", "absolute")
    out = ops.decode_attention(qd, kd, vd, t(sel, dev, torch.int32), t(cnt, dev, torch.int32), L, 64)
    _no_device_errors(dev)
    ref = O.decode_attention(n(qd), n(kd), n(vd), sel, cnt, L, 64)
    np.testing.assert_allclose(n(out), ref, rtol=0, atol=ATOL[dt])


def test_decode_attention_reference_cache_layout(dev):
    """Strided [B,T,H,D] cache of the reference's KVCache (per-row bulk copies)."""
    b, L = 2, 1500
    kc = normal((b, 2048, 4, 64), seed=41)
    vc = normal((b, 2048, 4, 64), seed=42)
    q = normal((b, 12, 64), seed=43)
    kd, vd = t(kc, dev), t(vc, dev)
    sel, cnt = O.decode_select(None, None, L, 64, 8, b, 4)
    out = ops.decode_attention(t(q, dev), kd[:, :L].transpose(1, 2), vd[:, :L].transpose(1, 2),
                               t(sel, dev, torch.int32), t(cnt, dev, torch.int32), L, 64)
    ref = O.decode_attention(q, kc.transpose(0, 2, 1, 3), vc.transpose(0, 2, 1, 3), sel, cnt, L, 64)
    np.testing.assert_allclose(n(out), ref, rtol=0, atol=1e-4)


@pytest.mark.parametrize("bs", [32, 128])
def test_decode_attention_other_block_sizes(dev, bs):
    b, L = 2, 2000
    kc, vc = normal((b, 4, 2048, 64), seed=51), normal((b, 4, 2048, 64), seed=52)
    q = normal((b, 12, 64), seed=53)
    sel, cnt = O.decode_select(None, None, L, bs, 8, b, 4)
    out = ops.decode_attention(t(q, dev), t(kc, dev), t(vc, dev), t(sel, dev, torch.int32),
                               t(cnt, dev, torch.int32), L, bs)
    ref = O.decode_attention(q, kc, vc, sel, cnt, L, bs)
    np.testing.assert_allclose(n(out), ref, rtol=0, atol=1e-4)


# ------------------------------------------------------------------ cache + fused layer
def test_kv_append_prototypes(dev):
    b = 2
    cache = sd.B200KVCache(b, 1000, 4, 64, dev, torch.float32)
    k1, v1 = normal((b, 100, 4, 64), seed=61), normal((b, 100, 4, 64), seed=62)
    k2, v2 = normal((b, 37, 4, 64), seed=63), normal((b, 37, 4, 64), seed=64)
    cache.update(t(k1, dev), t(v1, dev))
    ka, va = cache.update(t(k2, dev), t(v2, dev))
    kk = np.concatenate([k1, k2], axis=1)
    assert cache.current_len == 137 and int(cache.len_dev.item()) == 137
    assert np.array_equal(n(ka), kk) and np.array_equal(n(va), np.concatenate([v1, v2], 1))
    np.testing.assert_allclose(n(cache.prototypes()), O.compress_blocks(kk, 64), rtol=1e-5, atol=1e-6)


def _oracle_step(kd_np, vd_np, qkv_np, f_np, pos, cos, sin, rule, hq=12, hkv=4):
    b = qkv_np.shape[0]
    q = qkv_np[:, :hq * 64].reshape(b, 1, hq, 64)
    k = qkv_np[:, hq * 64:(hq + hkv) * 64].reshape(b, 1, hkv, 64)
    qr = O.apply_rope(q.astype(np.float64), cos, sin, pos)[:, 0]
    kr = O.apply_rope(k.astype(np.float64), cos, sin, pos)[:, 0]
    L = pos + 1
    reps = O.compress_blocks(kd_np[:, :, :L].transpose(0, 2, 1, 3), 64)
    sel, cnt = O.decode_select(f_np, reps if f_np is not None else None, L, 64, 8, b, hkv, "forecast", rule)
    return O.decode_attention(qr, kd_np, vd_np, sel, cnt, L, 64), kr


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rule", ["reference", "absolute"])
@pytest.mark.parametrize("start", [0, 62, 700, 1023])
def test_decode_layer_vs_oracle(dev, dt, rule, start):
    """Fused RoPE + append + compressor + selection + attention, 3 steps."""
    b, hq, hkv = 3, 12, 4
    cache = sd.B200KVCache(b, 2048, hkv, 64, dev, dt)
    if start:
        cache.update(t(normal((b, start, hkv, 64), seed=71), dev, dt), t(normal((b, start, hkv, 64), seed=72), dev, dt))
    cos, sin = precompute_rope_freqs(64, 2048)
    cos_d, sin_d = cos.to(dev), sin.to(dev)
    for step in range(3):
        pos = cache.current_len
        qkv = t(normal((b, (hq + 2 * hkv) * 64), seed=80 + step), dev, dt)
        f = t(normal((b, hkv, 64), seed=90 + step), dev, dt) if step != 1 else None
        out = ops.decode_layer(qkv, f, cos_d, sin_d, cache.len_dev, cache.k_store, cache.v_store, cache.proto_sum,
                               hq, hkv, 64, 8, rule)
        cache.advance(1)
        _no_device_errors(dev)
        kd, vd = n(cache.k_store), n(cache.v_store)
        ref, kr = _oracle_step(kd, vd, n(qkv), None if f is None else n(f)[:, None], pos, n(cos_d), n(sin_d), rule)
        np.testing.assert_allclose(kd[:, :, pos], kr, rtol=0, atol=1e-5 if dt == torch.float32 else 2e-2)
        assert np.array_equal(vd[:, :, pos], n(qkv)[:, (hq + hkv) * 64:].reshape(b, hkv, 64))
        np.testing.assert_allclose(n(out).reshape(b, hq, 64), ref, rtol=0, atol=ATOL[dt])
        np.testing.assert_allclose(n(cache.prototypes()), O.compress_blocks(kd[:, :, :pos + 1].transpose(0, 2, 1, 3), 64),
                                   rtol=1e-5, atol=2e-5)


def test_decode_layer_rope_bitexact_bf16(dev):
    """The fused RoPE reproduces the reference's bf16 rounding sequence
    (model/rope.py:58-63) bit for bit."""
    from local_research_small_language_model_b200.rope import apply_rotary_emb
    b, hq, hkv = 2, 12, 4
    cache = sd.B200KVCache(b, 512, hkv, 64, dev, torch.bfloat16)
    cache.update(t(normal((b, 300, hkv, 64), seed=1), dev, torch.bfloat16),
                 t(normal((b, 300, hkv, 64), seed=2), dev, torch.bfloat16))
    cos, sin = precompute_rope_freqs(64, 512)
    qkv = t(normal((b, (hq + 2 * hkv) * 64), seed=3), dev, torch.bfloat16)
    ops.decode_layer(qkv, None, cos.to(dev), sin.to(dev), cache.len_dev, cache.k_store, cache.v_store,
                     cache.proto_sum, hq, hkv, 64, 8)
    xq = qkv[:, :hq * 64].view(b, 1, hq, 64)
    xk = qkv[:, hq * 64:(hq + hkv) * 64].view(b, 1, hkv, 64)
    _, kr = apply_rotary_emb(xq, xk, cos.to(dev), sin.to(dev), offset=300)
    assert torch.equal(cache.k_store[:, :, 300], kr[:, 0])


# ------------------------------------------------------------------ decode-step row kernels
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,c,offset", [(64, 768, 0), (1000, 768, 0), (64, 1000, 0), (64, 768, 3)])
def test_rmsnorm_matches_reference_formula(dev, dt, rows, c, offset):
    """model/norm.py:15-21: fp32 normalisation, cast, gain multiply in dtype.
    Each case reaches a different kernel of sd_rmsnorm: 64 rows of 768 -> the
    one-16-byte-chunk-per-thread kernel (rmsnorm_chunk_kernel); 1000 rows ->
    the warp-per-row kernel (rmsnorm_rows_kernel); C=1000 (not a multiple of
    256 bf16 values) and a row view starting 3 elements in (unaligned) -> the
    generic block-per-row kernel (rmsnorm_kernel)."""
    base = t(normal((rows, c + offset), seed=1), dev, dt)
    x = base[:, offset:]
    w = t(1.0 + 0.1 * normal((c,), seed=2), dev, dt)
    ref = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)).type_as(x) * w
    got = ops.rmsnorm(x, w, 1e-6)
    tol = 1e-6 if dt == torch.float32 else 8e-3  # one bf16 ulp of the normalised value
    torch.testing.assert_close(got.float(), ref.float(), rtol=tol, atol=tol)


@pytest.mark.parametrize("dt,rows,f", [(torch.float32, 64, 2048), (torch.bfloat16, 64, 2048),
                                       (torch.float16, 4096, 2048), (torch.bfloat16, 70000, 64),
                                       (torch.bfloat16, 5, 1001)])
def test_silu_mul_matches_reference_formula(dev, dt, rows, f):
    """model/transformer.py:30-31 on a fused [gate | up] projection: the
    16-byte-chunk kernel (16-bit, F % 8 == 0; also past 65,535 rows) and the
    scalar kernel (fp32, F = 1001)."""
    gu = t(normal((rows, 2 * f), seed=3), dev, dt)
    ref = torch.nn.functional.silu(gu[:, :f]) * gu[:, f:]
    torch.testing.assert_close(ops.silu_mul(gu).float(), ref.float(), rtol=1e-5 if dt == torch.float32 else 8e-3,
                               atol=1e-6 if dt == torch.float32 else 8e-3)


# ------------------------------------------------------------------ fused-kernel selection
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rule", ["reference", "absolute"])
@pytest.mark.parametrize("start", [700, 1023, 1087, 1600])
def test_decode_layer_selection_and_candidates(dev, dt, rule, start):
    """The fused kernel's own selected lists equal the oracle's, and merging
    precomputed candidates (sd_decode_candidates) gives the same lists and the
    same output bits as scoring inside the kernel."""
    b, hq, hkv = 3, 12, 4
    caches = [sd.B200KVCache(b, 2048, hkv, 64, dev, dt) for _ in range(2)]
    k0, v0 = t(normal((b, start, hkv, 64), seed=171), dev, dt), t(normal((b, start, hkv, 64), seed=172), dev, dt)
    for c in caches:
        c.update(k0, v0)
    cos, sin = precompute_rope_freqs(64, 2048)
    cos_d, sin_d = cos.to(dev), sin.to(dev)
    for step in range(3):
        pos = caches[0].current_len
        qkv = t(normal((b, (hq + 2 * hkv) * 64), seed=180 + step), dev, dt)
        f = t(normal((b, hkv, 64), seed=190 + step), dev, dt)
        sels, outs = [], []
        for i, c in enumerate(caches):
            sel = torch.full((b, hkv, 10), -1, dtype=torch.int32, device=dev)
            cnt = torch.zeros(b, hkv, dtype=torch.int32, device=dev)
            cand = ops.decode_candidates(f, c.proto_sum, c.len_dev, hkv, 64, 8, rule) if i == 1 else None
            outs.append(ops.decode_layer(qkv, f, cos_d, sin_d, c.len_dev, c.k_store, c.v_store, c.proto_sum, hq, hkv,
                                         64, 8, rule, sel_out=sel, cnt_out=cnt, cand=cand))
            c.advance(1)
            sels.append((n(sel).astype(np.int64), n(cnt).astype(np.int64)))
        _no_device_errors(dev)
        assert np.array_equal(sels[0][0], sels[1][0]) and np.array_equal(sels[0][1], sels[1][1])
        assert torch.equal(outs[0], outs[1])
        kd = n(caches[0].k_store)
        L = pos + 1
        reps = O.compress_blocks(kd[:, :, :L].transpose(0, 2, 1, 3), 64)
        rs, rc = O.decode_select(n(f)[:, None], reps, L, 64, 8, b, hkv, "forecast", rule)
        assert np.array_equal(sels[0][1], rc)
        for ix in np.ndindex(b, hkv):
            assert list(sels[0][0][ix][:rc[ix]]) == list(rs[ix][:rc[ix]]), (step, ix)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("offset,tt", [(0, 700), (16000, 96)])
def test_rope_qk_bit_exact_vs_reference_formula(dev, dt, offset, tt):
    """sd_rope_qk on strided q/k views of one packed projection equals the
    reference's apply_rotary_emb (model/rope.py:34-65) bit for bit, tables
    cast to the activation dtype as type_as does."""
    from local_research_small_language_model_b200.rope import apply_rotary_emb
    b = 2
    proj = t(normal((b, tt, 1536), seed=21), dev, dt)
    xq = proj[..., :768].unflatten(-1, (12, 64))
    xk = proj[..., 768:1024].unflatten(-1, (4, 64))
    cos, sin = precompute_rope_freqs(64, offset + tt + 64)
    cos, sin = cos.to(dev), sin.to(dev)
    q1, k1 = ops.rope_qk(xq, xk, cos, sin, offset)
    q2, k2 = apply_rotary_emb(xq, xk, cos, sin, offset=offset)
    assert torch.equal(q1, q2) and torch.equal(k1, k2)


@pytest.mark.parametrize("dt,rows,n", [(torch.bfloat16, 64, 32000), (torch.float16, 3, 1000), (torch.float32, 5, 777),
                                       (torch.bfloat16, 7, 1001)])
def test_argmax_rows_matches_torch(dev, dt, rows, n):
    """Greedy next token (model/model.py:185): the first index of each row's
    maximum, NaN above every number, as torch.argmax; ties planted on purpose
    (16-byte path for 16-bit rows with n % 8 == 0, the scalar path otherwise)."""
    g = torch.Generator(device=dev).manual_seed(rows + n)
    x = torch.randn(rows, n, generator=g, device=dev).to(dt)
    x[0, n // 3] = x[0, n - 1] = x[0].max() + 1  # tie: the first wins
    if rows > 2:
        x[2, 5] = float("nan")
        x[2, n - 2] = float("nan")
    got = ops.argmax_rows(x)
    ref = torch.argmax(x, dim=-1)
    assert torch.equal(got, ref)
    out = torch.full((rows, 1), -7, dtype=torch.int64, device=dev)
    ops.argmax_rows(x, out=out)
    assert torch.equal(out[:, 0], ref)
