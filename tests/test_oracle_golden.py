"""Pins the CPU oracle against golden vectors produced by the reference itself
(tests/golden/make_golden.py).  CPU only."""

import numpy as np
import pytest

from oracle import sparda_oracle as O
from oracle.synthetic import SmallModelConfig, model_state, normal


def _torch_inputs_config1():
    import torch
    torch.manual_seed(0)
    q = torch.randn(1, 1024, 12, 64)
    k = torch.randn(1, 1024, 4, 64)
    v = torch.randn(1, 1024, 4, 64)
    f = torch.randn(1, 1024, 4, 64)
    return [t.numpy() for t in (q, k, v, f)]


def _finite_slots_equal(ref_scores, ref_idx, idx):
    """Slot-by-slot equality wherever the reference's selected score is finite."""
    vals = np.take_along_axis(ref_scores, ref_idx.astype(np.int64), axis=-1)
    fin = np.isfinite(vals)
    return np.array_equal(ref_idx[fin], idx[fin])


def test_config1_inputs_regenerate(golden):
    g = golden("config1")
    sums = [x.astype(np.float64).sum() for x in _torch_inputs_config1()]
    np.testing.assert_allclose(sums, g["in_sums"], rtol=0, atol=1e-6)


def test_config1_compressor_selector(golden):
    g = golden("config1")
    q, k, v, f = _torch_inputs_config1()
    reps = O.compress_blocks(k, 64)
    np.testing.assert_allclose(reps, g["reps"], rtol=0, atol=2e-7)
    scores, idx = O.select_blocks(f, reps, 8, 64, True)
    ref = g["scores"]
    assert np.array_equal(np.isfinite(scores), np.isfinite(ref))
    fin = np.isfinite(ref)
    np.testing.assert_allclose(scores[fin], ref[fin], rtol=0, atol=2e-6)
    # top-k of the reference's own fp32 scores: bit-exact on finite slots
    assert _finite_slots_equal(ref, g["idx"], O.topk_desc(ref, 8))
    # end to end: no finite near-ties in config 1, so the oracle's own scores agree too
    assert _finite_slots_equal(ref, g["idx"], idx)


def test_config1_masked_output(golden):
    g = golden("config1")
    q, k, v, f = _torch_inputs_config1()
    out = O.masked_prefill(q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3), f,
                           64, 8, layer_idx=1)
    out = out.transpose(0, 2, 1, 3).reshape(1024, 768)
    np.testing.assert_allclose(out[::16], g["out_rows"], rtol=0, atol=2e-5)
    np.testing.assert_allclose(out.sum(-1), g["out_row_sum"], rtol=0, atol=5e-4)
    np.testing.assert_allclose(np.abs(out).sum(-1), g["out_row_abs"], rtol=1e-5)


@pytest.mark.parametrize("t", [1, 63, 64, 65, 129, 640, 641])
def test_compressor_partial_blocks(golden, t):
    g = golden("compressor")
    i = [1, 63, 64, 65, 129, 640, 641].index(t)
    k = normal((2, t, 4, 64), seed=100 + i)
    np.testing.assert_allclose(O.compress_blocks(k, 64), g[f"T{t}"], rtol=0, atol=2e-7)


def test_compressor_reference_test_geometry(golden):
    k = normal((2, 50, 4, 32), seed=199)
    out = O.compress_blocks(k, 16)
    assert out.shape == (2, 4, 4, 32)
    np.testing.assert_allclose(out, golden("compressor")["bs16_T50"], rtol=0, atol=2e-7)


@pytest.mark.parametrize("case", ["reftest", "decode257", "decode16", "chunk40", "causal300", "topk_gt_nb"])
def test_selector_cases(golden, case):
    from tests.golden.make_golden import SELECTOR_CASES
    name, b, tq, h, d, nb, bs, k, causal, seed = [c for c in SELECTOR_CASES if c[0] == case][0]
    g = golden("selector")
    f = normal((b, tq, h, d), seed=seed)
    r = normal((b, nb, h, d), seed=seed + 1000)
    scores, idx = O.select_blocks(f, r, k, bs, causal)
    ref_s, ref_i = g[case + "_scores"], g[case + "_idx"]
    assert np.array_equal(np.isfinite(scores), np.isfinite(ref_s))
    fin = np.isfinite(ref_s)
    np.testing.assert_allclose(scores[fin], ref_s[fin], rtol=1e-6, atol=1e-6)
    assert idx.shape == ref_i.shape
    assert _finite_slots_equal(ref_s, ref_i, O.topk_desc(ref_s, idx.shape[-1]))
    assert _finite_slots_equal(ref_s, ref_i, idx)


def _ref_lists(sel, valid):
    """Reference (sel, valid) capture -> compact ascending lists + counts."""
    lead = sel.shape[:-1]
    ms = sel.shape[-1]
    out = np.full(lead + (ms,), -1, dtype=np.int64)
    cnt = np.zeros(lead, dtype=np.int64)
    for ix in np.ndindex(*lead):
        ids = np.sort(sel[ix][valid[ix]])
        out[ix][:len(ids)] = ids
        cnt[ix] = len(ids)
    return out, cnt


@pytest.mark.parametrize("case", ["L600", "L641", "L1000", "L1024", "L1000_static"])
def test_decode_cases(golden, case):
    from tests.golden.make_golden import DECODE_CASES
    name, b, L, with_f, seed = [c for c in DECODE_CASES if c[0] == case][0]
    g = golden("decode")
    q = normal((b, 12, 1, 64), seed=seed)[:, :, 0]
    k = normal((b, 4, L, 64), seed=seed + 1)
    v = normal((b, 4, L, 64), seed=seed + 2)
    f = normal((b, 1, 4, 64), seed=seed + 3) if with_f else None
    reps = O.compress_blocks(k.transpose(0, 2, 1, 3), 64)
    sel, cnt = O.decode_select(f, reps, L, 64, 8, b, 4, "forecast", "reference")
    if case + "_sel" not in g:  # dense fallback: fully defined
        out = O.decode_attention(q, k, v, sel, cnt, L, 64)
        np.testing.assert_allclose(out, g[case + "_out"], rtol=0, atol=2e-6)
        return
    rsel, rcnt = _ref_lists(g[case + "_sel"], g[case + "_valid"])
    # attention conditioned on the reference's own index tensor
    out = O.decode_attention(q, k, v, rsel, rcnt, L, 64)
    np.testing.assert_allclose(out, g[case + "_out"], rtol=0, atol=2e-6)
    # selection: the well-defined part (sink, current, finite top-k) is in the reference set
    curr = (L - 1) // 64
    for ix in np.ndindex(b, 4):
        ref_set = set(rsel[ix][:rcnt[ix]].tolist())
        mine = set(sel[ix][:cnt[ix]].tolist())
        assert {0, curr} <= ref_set and rcnt[ix] <= 10
        if not with_f:
            assert mine == ref_set  # static window is fully defined
        else:
            assert {0, curr} <= mine and len(mine) <= 10


@pytest.mark.parametrize("case", ["T700", "T700_static", "T700_layer0", "T128"])
def test_masked_cases(golden, case):
    from tests.golden.make_golden import MASKED_CASES
    name, b, t, li, mode, with_f, seed = [c for c in MASKED_CASES if c[0] == case][0]
    g = golden("masked")
    q = normal((b, 12, t, 64), seed=seed)
    k = normal((b, 4, t, 64), seed=seed + 1)
    v = normal((b, 4, t, 64), seed=seed + 2)
    f = normal((b, t, 4, 64), seed=seed + 3) if with_f else None
    out = O.masked_prefill(q, k, v, f, 64, 8, layer_idx=li, mode=mode).transpose(0, 2, 1, 3)
    np.testing.assert_allclose(out[:, ::31], g[case + "_rows"], rtol=0, atol=2e-5)
    np.testing.assert_allclose(out.sum(axis=(2, 3)), g[case + "_row_sum"], rtol=0, atol=5e-4)


@pytest.mark.parametrize("case", ["T1024", "T700", "T900_static"])
def test_chunked_cases(golden, case):
    from tests.golden.make_golden import CHUNKED_CASES
    name, b, t, with_f, mode, seed = [c for c in CHUNKED_CASES if c[0] == case][0]
    g = golden("chunked")
    q = normal((b, 12, t, 64), seed=seed)
    k = normal((b, 4, t, 64), seed=seed + 1)
    v = normal((b, 4, t, 64), seed=seed + 2)
    f = normal((b, t, 4, 64), seed=seed + 3) if with_f else None
    rsel, rcnt = _ref_lists(g[case + "_sel"], g[case + "_valid"])
    out = O.chunked_attention(q, k, v, rsel, rcnt, 64).transpose(0, 2, 1, 3)
    np.testing.assert_allclose(out[:, ::31], g[case + "_rows"], rtol=0, atol=2e-5)
    np.testing.assert_allclose(out.sum(axis=(2, 3)), g[case + "_row_sum"], rtol=0, atol=5e-4)
    # selection: reference subset of the oracle's union, of size min(MS, |union|);
    # the oracle's own truncated list is such a subset too
    reps = O.compress_blocks(k.transpose(0, 2, 1, 3), 64)
    sel, cnt, union = O.chunked_select(f, reps, t, 64, 8, b, 4, mode)
    nb = O.num_blocks(t, 64)
    ms = min(nb, 10)
    n_trunc = 0
    for ix in np.ndindex(b, 4, nb):
        u = set(np.nonzero(union[ix])[0].tolist())
        ref_set = set(rsel[ix][:rcnt[ix]].tolist())
        mine = set(sel[ix][:cnt[ix]].tolist())
        assert ref_set <= u and len(ref_set) == min(ms, len(u))
        assert mine <= u and len(mine) == min(ms, len(u))
        assert {0, ix[2]} <= mine
        if len(u) <= ms:
            assert mine == ref_set
        else:
            n_trunc += 1
    if case == "T1024":
        assert n_trunc > 0  # the truncation hazard is exercised


@pytest.mark.parametrize("case", ["L1000", "L500", "L1000_layer0"])
def test_prefetch_selection(golden, case):
    b, L, li, seed = {"L1000": (2, 1000, 1, 700), "L500": (1, 500, 1, 701),
                      "L1000_layer0": (1, 1000, 0, 702)}[case]
    g = golden("prefetch")
    k = normal((b, L, 4, 64), seed=seed)
    f = normal((b, 1, 4, 64), seed=seed + 2)
    small, sel, cnt = O.prefetch_select(f, k, L, 64, 8, li)
    assert bool(small) == bool(g[case + "_small"])
    if not small:
        rsel, rcnt = _ref_lists(g[case + "_sel"], g[case + "_val"] > 0.5)
        curr = L // 64
        for ix in np.ndindex(b, 4):
            ref_set = set(rsel[ix][:rcnt[ix]].tolist())
            assert {0, curr} <= ref_set and {0, curr} <= set(sel[ix][:cnt[ix]].tolist())


def test_model_decode_logits(golden):
    """Oracle model decode vs the reference model, token by token from an empty
    cache (dense-fallback region, no tie hazards)."""
    from tests.golden.make_golden import MODEL_STEPS
    g = golden("model_decode")
    sc = SmallModelConfig()
    m = O.OracleModel(model_state(sc, seed=7), n_layer=sc.n_layer, max_seq_len=1024, dtype=np.float64)
    ids = g["ids"]
    b = ids.shape[0]
    kc = [np.zeros((b, 4, 1024, 64)) for _ in range(sc.n_layer)]
    vc = [np.zeros((b, 4, 1024, 64)) for _ in range(sc.n_layer)]
    for s in range(max(MODEL_STEPS) + 1):
        lg = m.decode_step(ids[:, s], kc, vc, s)
        if s in MODEL_STEPS:
            np.testing.assert_allclose(lg, g[f"step{s}"], rtol=0, atol=2e-4)


# ---------------------------------------------------------------- BASELINE-sized and sparse-regime goldens
def _decode_big_oracle(b, L, rule, seed):
    """The oracle fed the same step the golden generator ran: the prefix cache,
    the new token rotated at position L-1 and appended, then selection +
    attention.  Returns (q_rot [B,12,64], k_all, v_all [B,4,L,64], sel, cnt)."""
    from tests.golden.make_golden import decode_big_inputs
    kp, vp, q, kn, vn, f = decode_big_inputs(b, L, seed)
    cos, sin = O.rope_tables(64, L + 64)
    qr = O.apply_rope(q[:, None].astype(np.float64), cos, sin, L - 1)[:, 0]
    kr = O.apply_rope(kn[:, None].astype(np.float64), cos, sin, L - 1)[:, 0]
    k_all = np.concatenate([kp, kr[:, None].astype(np.float32)], axis=1).transpose(0, 2, 1, 3)
    v_all = np.concatenate([vp, vn[:, None]], axis=1).transpose(0, 2, 1, 3)
    reps = O.compress_blocks(k_all.transpose(0, 2, 1, 3), 64)
    sel, cnt = O.decode_select(f, reps, L, 64, 8, b, 4, "forecast", rule)
    return qr, k_all, v_all, sel, cnt


@pytest.mark.parametrize("case", ["L16385_abs", "L16448_abs", "L16400_ref", "L1000_abs", "L641_abs"])
def test_decode_big_cases(golden, case):
    """Decode steps at BASELINE config-2 lengths (16,385-16,448 cached tokens).
    Absolute rule: every score is finite, so the oracle's selected set equals
    the reference's and its output matches unconditioned.  Reference rule:
    attention on the reference's captured lists (its -inf tie order is
    implementation-defined) and the sink/current blocks in both sets."""
    from tests.golden.make_golden import DECODE_BIG_CASES
    name, b, L, rule, seed = [c for c in DECODE_BIG_CASES if c[0] == case][0]
    g = golden("decode_big")
    qr, k_all, v_all, sel, cnt = _decode_big_oracle(b, L, rule, seed)
    rsel, rcnt = _ref_lists(g[case + "_sel"], g[case + "_valid"])
    curr = (L - 1) // 64
    out_ref_lists = O.decode_attention(qr, k_all, v_all, rsel, rcnt, L, 64)
    np.testing.assert_allclose(out_ref_lists, g[case + "_out"], rtol=0, atol=2e-6)
    for ix in np.ndindex(b, 4):
        ref_set = set(rsel[ix][:rcnt[ix]].tolist())
        mine = set(sel[ix][:cnt[ix]].tolist())
        assert {0, curr} <= ref_set and {0, curr} <= mine
        if rule == "absolute":
            assert mine == ref_set, ix
    if rule == "absolute":
        out = O.decode_attention(qr, k_all, v_all, sel, cnt, L, 64)
        np.testing.assert_allclose(out, g[case + "_out"], rtol=0, atol=2e-6)


def test_model_sparse_regime_logits(golden):
    """Oracle model (prefill, then decode with the absolute rule) vs the
    reference model past the dense fallback: layer L's forecast selects layer
    L+1's blocks in every decode step.  Logits and every layer's selected set."""
    from tests.golden.make_golden import MODEL_SPARSE_PREFILL, MODEL_SPARSE_STEPS
    g = golden("model_sparse")
    sc = SmallModelConfig()
    m = O.OracleModel(model_state(sc, seed=9), n_layer=sc.n_layer, max_seq_len=1024, rule="absolute",
                      dtype=np.float64)
    ids = g["ids"].astype(np.int64)
    b = ids.shape[0]
    p = MODEL_SPARSE_PREFILL
    kc = [np.zeros((b, 4, 1024, 64)) for _ in range(sc.n_layer)]
    vc = [np.zeros((b, 4, 1024, 64)) for _ in range(sc.n_layer)]
    np.testing.assert_allclose(m.prefill(ids[:, :p], kc, vc), g["prefill_last"], rtol=0, atol=2e-4)
    sel_ref = g["sel"].astype(np.int64)
    for s in range(MODEL_SPARSE_STEPS):
        lg = m.decode_step(ids[:, p + s], kc, vc, p + s)
        if f"step{s}" in g:
            np.testing.assert_allclose(lg, g[f"step{s}"], rtol=0, atol=2e-4, err_msg=f"step {s}")
        curr = (p + s) // 64
        for li in range(sc.n_layer):
            rsel, rcnt = _ref_lists(sel_ref[s, li], g["valid"][s, li])
            sel, cnt = m.last_sel[li]
            for ix in np.ndindex(b, 4):
                st = set(rsel[ix][:rcnt[ix]].tolist())
                assert {0, curr} <= st and len(st) <= 10
                assert set(sel[ix][:cnt[ix]].tolist()) == st, (s, li, ix)


def test_chunked_prefill_32k(golden):
    """Config-3 length (T=32,768): oracle attention on the reference's own
    per-q-block lists vs its output rows, and the oracle's lists equal the
    reference's wherever the union needs no truncation."""
    from tests.golden.make_golden import CHUNKED_BIG, CHUNKED_BIG_ROW_EVERY
    name, b, t, seed = CHUNKED_BIG
    g = golden("chunked_big")
    q = normal((b, 12, t, 64), seed=seed)
    k = normal((b, 4, t, 64), seed=seed + 1)
    v = normal((b, 4, t, 64), seed=seed + 2)
    f = normal((b, t, 4, 64), seed=seed + 3)
    rsel, rcnt = _ref_lists(g["sel"].astype(np.int64), g["valid"])
    out = O.chunked_attention(q, k, v, rsel, rcnt, 64).transpose(0, 2, 1, 3)
    np.testing.assert_allclose(out[:, ::CHUNKED_BIG_ROW_EVERY], g["rows"], rtol=0, atol=2e-5)
    np.testing.assert_allclose(out.sum(axis=(2, 3)), g["row_sum"], rtol=0, atol=5e-4)
    reps = O.compress_blocks(k.transpose(0, 2, 1, 3), 64)
    sel, cnt, union = O.chunked_select(f, reps, t, 64, 8, b, 4, "forecast")
    nb = O.num_blocks(t, 64)
    n_same = n_trunc = 0
    for ix in np.ndindex(b, 4, nb):
        u = set(np.nonzero(union[ix])[0].tolist())
        ref_set = set(rsel[ix][:rcnt[ix]].tolist())
        mine = set(sel[ix][:cnt[ix]].tolist())
        assert ref_set <= u and len(ref_set) == min(10, len(u))
        if len(u) <= 10:
            assert mine == ref_set
            n_same += 1
        else:
            n_trunc += 1
    assert n_same > 0 and n_trunc > 0


@pytest.mark.parametrize("case", ["L1000", "L1023", "L1024", "L3000"])
def test_prefetch_selection_absolute(golden, case):
    """The reference's prefetch selection (before the append, async_offload.py:
    241-260) under the absolute rule: every score is finite, so the oracle's
    selected set equals the reference's."""
    from tests.golden.make_golden import PREFETCH_ABS_CASES
    name, b, L, li, seed = [c for c in PREFETCH_ABS_CASES if c[0] == case][0]
    g = golden("prefetch_abs")
    k = normal((b, L, 4, 64), seed=seed)
    f = normal((b, 1, 4, 64), seed=seed + 2)
    small, sel, cnt = O.prefetch_select(f, k, L, 64, 8, li, rule="absolute")
    assert bool(small) == bool(g[case + "_small"])
    assert not small
    rsel, rcnt = _ref_lists(g[case + "_sel"], g[case + "_val"] > 0.5)
    for ix in np.ndindex(b, 4):
        assert set(sel[ix][:cnt[ix]].tolist()) == set(rsel[ix][:rcnt[ix]].tolist()), ix


def _async_decode_oracle(case):
    """Oracle restatement of the reference's async decode steps: the prefetch
    selection before the append (prefetch_select), then attention over those
    blocks with the new token in place (async_offload.py:296-390, :466-490),
    wq/wk/wv/wo and RoPE (model/rope.py:34-65) around it."""
    from tests.golden.make_golden import ASYNC_DECODE_CASES, ASYNC_DECODE_STEPS, async_attn_weights, \
        async_decode_inputs
    name, b, L, seed = [c for c in ASYNC_DECODE_CASES if c[0] == case][0]
    w = async_attn_weights(seed)
    k0, v0, _, _ = async_decode_inputs(b, L, seed, 0)
    kc = np.zeros((b, 4, L + 64, 64))
    vc = np.zeros((b, 4, L + 64, 64))
    kc[:, :, :L] = k0.transpose(0, 2, 1, 3)
    vc[:, :, :L] = v0.transpose(0, 2, 1, 3)
    cos, sin = O.rope_tables(64, L + 128)
    outs, sels = [], []
    for s in range(ASYNC_DECODE_STEPS):
        cur = L + s
        _, _, x, f = async_decode_inputs(b, L, seed, s)
        small, sel, cnt = O.prefetch_select(f, kc[:, :, :cur].transpose(0, 2, 1, 3), cur, 64, 8, 1, rule="absolute")
        assert not small
        x32 = x.astype(np.float32)
        q = (x32 @ w["wq"].T).reshape(b, 1, 12, 64)
        k = (x32 @ w["wk"].T).reshape(b, 1, 4, 64)
        v = (x32 @ w["wv"].T).reshape(b, 1, 4, 64)
        q = O.apply_rope(q.astype(np.float64), cos, sin, cur)
        k = O.apply_rope(k.astype(np.float64), cos, sin, cur)
        kc[:, :, cur] = k[:, 0]
        vc[:, :, cur] = v[:, 0]
        a = O.decode_attention(q[:, 0], kc, vc, sel, cnt, cur + 1, 64)
        outs.append(a.reshape(b, 1, 768) @ w["wo"].T.astype(np.float64))
        sels.append((sel, cnt))
    return outs, sels


@pytest.mark.parametrize("case", ["L1000", "L1023", "L3000"])
def test_async_decode_vs_reference(golden, case):
    """AsyncForecastOffloadAttention's prefetch-consuming decode, three steps:
    the oracle's selection (before the append, absolute rule) equals the
    reference's prefetched lists and its output matches."""
    from tests.golden.make_golden import ASYNC_DECODE_STEPS
    g = golden("async_decode")
    outs, sels = _async_decode_oracle(case)
    for s in range(ASYNC_DECODE_STEPS):
        rsel, rcnt = _ref_lists(g[f"{case}_s{s}_sel"], g[f"{case}_s{s}_val"] > 0.5)
        sel, cnt = sels[s]
        for ix in np.ndindex(*cnt.shape):
            assert set(sel[ix][:cnt[ix]].tolist()) == set(rsel[ix][:rcnt[ix]].tolist()), (s, ix)
        np.testing.assert_allclose(outs[s], g[f"{case}_s{s}_out"], rtol=0, atol=2e-6)


def backward_inputs(b, t, with_f, seed):
    """Regenerates a backward case's inputs (make_golden.backward_cases):
    q [B,12,T,64], k, v [B,4,T,64], forecast [B,T,4,64] or None, and the
    output gradient [B,12,T,64] of loss = sum(out * w)."""
    q = normal((b, 12, t, 64), seed=seed)
    k = normal((b, 4, t, 64), seed=seed + 1)
    v = normal((b, 4, t, 64), seed=seed + 2)
    f = normal((b, t, 4, 64), seed=seed + 3) if with_f else None
    dout = normal((b, t, 768), seed=seed + 4).reshape(b, t, 12, 64).transpose(0, 2, 1, 3)
    return q, k, v, f, dout


def oracle_backward_allowed(k, f, t, layer_idx, mode, chunked):
    """The oracle's allowed mask of a backward case (masked or chunked path)."""
    if chunked:
        reps = O.compress_blocks(k.transpose(0, 2, 1, 3), 64)
        sel, cnt, union = O.chunked_select(f, reps, t, 64, 8, k.shape[0], k.shape[1], mode)
        assert union.sum(-1).max() <= 10  # N_b = MS: no truncation, the reference's lists
        return O.chunked_allowed(sel, cnt, t, 64)
    allowed, _, _ = O.masked_allowed(f, k, t, 64, 8, layer_idx, mode, True)
    return allowed


def _bwd_ids():
    from tests.golden.make_golden import BACKWARD_CASES
    return BACKWARD_CASES


@pytest.mark.parametrize("case", _bwd_ids(), ids=[c[0] for c in _bwd_ids()])
def test_attention_backward_vs_reference(golden, case):
    """The oracle's gradients of the masked / chunked attention cores equal the
    ones autograd took through the reference (fp32) for loss = sum(out * w)."""
    name, b, t, li, mode, with_f, chunked, seed = case
    g = golden("backward")
    q, k, v, f, dout = backward_inputs(b, t, with_f, seed)
    allowed = oracle_backward_allowed(k, f, t, li, mode, chunked)
    dq, dk, dv = O.attention_backward(q, k, v, dout, allowed)
    for got, key, every in ((dq, "dq", 29), (dk, "dk", 13), (dv, "dv", 13)):
        np.testing.assert_allclose(got[:, :, ::every], g[f"{name}_{key}_rows"], rtol=1e-4, atol=2e-5)
        np.testing.assert_allclose(got.sum(-1), g[f"{name}_{key}_sum"], rtol=1e-4, atol=2e-4)


def test_attention_backward_finite_differences():
    """attention_backward is the gradient of attention_forward: central
    differences in float64 on a small GQA case with a row that sees nothing."""
    rng = np.random.default_rng(7)
    b, hq, hkv, t, d = 1, 4, 2, 9, 8
    q, dout = rng.standard_normal((b, hq, t, d)), rng.standard_normal((b, hq, t, d))
    k, v = rng.standard_normal((b, hkv, t, d)), rng.standard_normal((b, hkv, t, d))
    allowed = rng.random((b, hkv, t, t)) < 0.6
    allowed[:, 1, 3] = False  # an empty row: zero output, zero gradients
    dq, dk, dv = O.attention_backward(q, k, v, dout, allowed)

    def loss(qq, kk, vv):
        return float((O.attention_forward(qq, kk, vv, allowed) * dout).sum())

    eps = 1e-6
    for x, gx, which in ((q, dq, 0), (k, dk, 1), (v, dv, 2)):
        for ix in [tuple(rng.integers(0, n) for n in x.shape) for _ in range(12)]:
            args = [q.copy(), k.copy(), v.copy()]
            args[which][ix] += eps
            up = loss(*args)
            args[which][ix] -= 2 * eps
            fd = (up - loss(*args)) / (2 * eps)
            assert abs(fd - gx[ix]) <= 1e-6 * max(1.0, abs(fd)), (which, ix, fd, gx[ix])
    assert np.all(dq[:, 2:4, 3] == 0)  # query heads 2, 3 use kv head 1's empty row


def test_mask_helpers_match_the_oracle_paths():
    """masked_allowed_from_topk equals masked_allowed's mask for the same top-k,
    and attention over chunked_allowed equals chunked_attention on the same
    lists: the two helpers the GPU backward tests build their masks with."""
    b, t = 2, 300
    q, k, v = normal((b, 12, t, 64), seed=901), normal((b, 4, t, 64), seed=902), normal((b, 4, t, 64), seed=903)
    f = normal((b, t, 4, 64), seed=904)
    reps = O.compress_blocks(k.transpose(0, 2, 1, 3), 64)
    _, topk = O.select_blocks(f, reps, 3, 64, True)
    for causal in (True, False):
        want, _, _ = O.masked_allowed(f, k, t, 64, 3, 1, "forecast", causal)
        _, topk_c = O.select_blocks(f, reps, 3, 64, causal)
        assert np.array_equal(O.masked_allowed_from_topk(topk_c, t, 64, causal), want)
    dense, _, _ = O.masked_allowed(None, k, t, 64, 3, 0, "forecast", True)
    assert np.array_equal(O.masked_allowed_from_topk(None, t, 64, True), dense)
    sel, cnt, _ = O.chunked_select(f, reps, t, 64, 3, b, 4, "forecast")
    np.testing.assert_allclose(O.attention_forward(q, k, v, O.chunked_allowed(sel, cnt, t, 64)),
                               O.chunked_attention(q, k, v, sel, cnt, 64), rtol=0, atol=1e-12)
