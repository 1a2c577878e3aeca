"""Prefill parity: block lists and block-sparse prefill attention against the
reference's golden outputs (fp32, max-abs 1e-4 on the attention output) and
against the oracle (bf16, max-abs 2e-2).  Needs a B200."""

import numpy as np
import pytest
import torch

import local_research_small_language_model_b200 as sd
from local_research_small_language_model_b200 import ops
from oracle import sparda_oracle as O
from oracle.synthetic import normal

pytestmark = pytest.mark.gpu


def t(x, dev, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to(dev, dtype)


def n(x):
    return x.detach().float().cpu().numpy()


def _masked(dev, q, k, v, f, layer_idx=1, mode="forecast", is_causal=True, dtype=torch.float32):
    """The masked prefill path through the ops, q [B,Hq,T,D], k/v [B,Hkv,T,D]."""
    b, hq, tt, d = q.shape
    hkv = k.shape[1]
    qd = t(q, dev, dtype).transpose(1, 2)
    kd, vd = t(k, dev, dtype), t(v, dev, dtype)
    nb = O.num_blocks(tt, 64)
    topk = None
    if nb <= 2 or (mode == "forecast" and (f is None or layer_idx == 0)):
        lm = "dense"
    elif mode == "forecast":
        reps = ops.compress_blocks(kd.transpose(1, 2), 64)
        _, topk = ops.select_blocks(t(f, dev), reps, 8, 64, is_causal)
        lm = "masked_forecast"
    else:
        lm = "masked_static"
    lists, counts = ops.prefill_lists(lm, b, hkv, tt, 64, 8, topk, is_causal, device=dev)
    out = ops.prefill_attention(qd, kd, vd, lists, counts, 64, topk, is_causal)
    return out, lists, counts, topk


def test_config1_masked_prefill_fp32(dev, golden):
    """BASELINE config 1 end to end on the GPU: compressor + selector + lists +
    attention vs the reference's own output (fp32, 1e-4)."""
    torch.manual_seed(0)
    q = torch.randn(1, 1024, 12, 64).numpy()
    k = torch.randn(1, 1024, 4, 64).numpy()
    v = torch.randn(1, 1024, 4, 64).numpy()
    f = torch.randn(1, 1024, 4, 64).numpy()
    g = golden("config1")
    out, _, _, topk = _masked(dev, q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3), f)
    o = n(out).reshape(1024, 768)
    np.testing.assert_allclose(o[::16], g["out_rows"], rtol=0, atol=1e-4)
    np.testing.assert_allclose(o.sum(-1), g["out_row_sum"], rtol=0, atol=2e-3)
    fin = np.isfinite(np.take_along_axis(g["scores"], g["idx"].astype(np.int64), -1))
    assert np.array_equal(n(topk).astype(np.int64)[fin], g["idx"].astype(np.int64)[fin])


@pytest.mark.parametrize("case", ["T700", "T700_static", "T700_layer0", "T128"])
def test_masked_prefill_vs_reference_golden(dev, golden, case):
    from tests.golden.make_golden import MASKED_CASES
    name, b, tt, li, mode, with_f, seed = [c for c in MASKED_CASES if c[0] == case][0]
    g = golden("masked")
    q = normal((b, 12, tt, 64), seed=seed)
    k = normal((b, 4, tt, 64), seed=seed + 1)
    v = normal((b, 4, tt, 64), seed=seed + 2)
    f = normal((b, tt, 4, 64), seed=seed + 3) if with_f else None
    out, *_ = _masked(dev, q, k, v, f, layer_idx=li, mode=mode)
    o = n(out)
    np.testing.assert_allclose(o[:, ::31], g[case + "_rows"], rtol=0, atol=1e-4)
    np.testing.assert_allclose(o.sum(axis=(2, 3)), g[case + "_row_sum"], rtol=0, atol=2e-3)


def test_masked_prefill_non_causal_vs_oracle(dev):
    b, tt = 1, 320
    q, k, v = normal((b, 12, tt, 64), seed=1), normal((b, 4, tt, 64), seed=2), normal((b, 4, tt, 64), seed=3)
    f = normal((b, tt, 4, 64), seed=4)
    out, *_ = _masked(dev, q, k, v, f, is_causal=False)
    ref = O.masked_prefill(q, k, v, f, 64, 8, layer_idx=1, is_causal=False).transpose(0, 2, 1, 3)
    np.testing.assert_allclose(n(out), ref, rtol=0, atol=1e-4)


def _ref_lists(sel, valid, cap):
    lead = sel.shape[:-1]
    out = np.full(lead + (cap,), -1, dtype=np.int32)
    cnt = np.zeros(lead, dtype=np.int32)
    for ix in np.ndindex(*lead):
        ids = np.sort(sel[ix][valid[ix]])
        out[ix][:len(ids)] = ids
        cnt[ix] = len(ids)
    return out, cnt


@pytest.mark.parametrize("case", ["T1024", "T700", "T900_static"])
def test_chunked_prefill_vs_reference_golden(dev, golden, case):
    """Chunked path: attention on the reference's own per-q-block lists (1e-4),
    and the kernel's own lists equal the oracle's (the truncation rule)."""
    from tests.golden.make_golden import CHUNKED_CASES
    name, b, tt, with_f, mode, seed = [c for c in CHUNKED_CASES if c[0] == case][0]
    g = golden("chunked")
    q = normal((b, 12, tt, 64), seed=seed)
    k = normal((b, 4, tt, 64), seed=seed + 1)
    v = normal((b, 4, tt, 64), seed=seed + 2)
    f = normal((b, tt, 4, 64), seed=seed + 3) if with_f else None
    nb = O.num_blocks(tt, 64)
    cap = min(nb, 10)
    rl, rc = _ref_lists(g[case + "_sel"], g[case + "_valid"], cap)
    qd, kd, vd = t(q, dev).transpose(1, 2), t(k, dev), t(v, dev)
    out = ops.prefill_attention(qd, kd, vd, t(rl, dev, torch.int32), t(rc, dev, torch.int32), 64, None, True)
    o = n(out)
    np.testing.assert_allclose(o[:, ::31], g[case + "_rows"], rtol=0, atol=1e-4)
    np.testing.assert_allclose(o.sum(axis=(2, 3)), g[case + "_row_sum"], rtol=0, atol=2e-3)
    # the kernel's lists vs the oracle's (same documented truncation rule)
    topk = None
    if with_f:
        reps = ops.compress_blocks(kd.transpose(1, 2), 64)
        _, topk = ops.select_blocks(t(f, dev), reps, 8, 64, False)
    lists, counts = ops.prefill_lists("chunked_forecast" if with_f else "chunked_static", b, 4, tt, 64, 8, topk,
                                      True, device=dev)
    reps_np = O.compress_blocks(k.transpose(0, 2, 1, 3), 64)
    osel, ocnt, _ = O.chunked_select(f, reps_np, tt, 64, 8, b, 4, mode)
    assert np.array_equal(n(counts).astype(np.int64), ocnt)
    for ix in np.ndindex(b, 4, nb):
        assert list(n(lists)[ix][:ocnt[ix]].astype(np.int64)) == list(osel[ix][:ocnt[ix]])


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_attention_module_prefill_paths_vs_oracle(dev, dt):
    """B200SparseAttention.forward prefill (masked and forced chunked) against
    the oracle fed the module's own projections."""
    torch.manual_seed(3)
    cfg = sd.ModelConfig(block_size=64, top_k_blocks=8)
    attn = sd.B200SparseAttention(cfg, layer_idx=1).to(dev, dt)
    with torch.no_grad():
        attn.wo.weight.copy_(torch.eye(768))
    rot = sd.RotaryEmbedding(64, 2048).to(dev)
    b, tt = 2, 700
    x = torch.randn(b, tt, 768, device=dev).to(dt)
    f = torch.randn(b, tt, 4, 64, device=dev).to(dt)
    with torch.no_grad():
        xq = attn.wq(x).view(b, tt, 12, 64)
        xk = attn.wk(x).view(b, tt, 4, 64)
        xv = attn.wv(x).view(b, tt, 4, 64)
        xq, xk = rot(xq, xk, 0)
        q_, k_, v_ = (n(z).transpose(0, 2, 1, 3) for z in (xq, xk, xv))
        for chunked in (False, True):
            out = attn(x, rot, forecast_vector=f, use_chunked_gather=chunked)
            if chunked:
                ref, _, _ = O.chunked_prefill(q_, k_, v_, n(f), 64, 8)
            else:
                ref = O.masked_prefill(q_, k_, v_, n(f), 64, 8, layer_idx=1)
            ref = ref.transpose(0, 2, 1, 3).reshape(b, tt, 768)
            tol = 1e-4 if dt == torch.float32 else 2e-2
            np.testing.assert_allclose(n(out), ref, rtol=0, atol=tol)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("mode,tt,causal", [("masked_forecast", 700, True), ("masked_forecast", 640, False),
                                            ("masked_static", 900, True), ("chunked_forecast", 1000, True),
                                            ("dense", 128, True), ("dense", 100, False)])
def test_tensor_core_prefill_matches_fp32_path(dev, dt, mode, tt, causal):
    """The tcgen05 kernel (16-bit inputs) against the CUDA-core kernel run in
    fp32 on the same rounded inputs and the same lists: max-abs 2e-2 (P is
    rounded to 16 bits before the PV product)."""
    b, hq, hkv = 2, 12, 4
    q = normal((b, tt, hq, 64), seed=41)
    k = normal((b, hkv, tt, 64), seed=42)
    v = normal((b, hkv, tt, 64), seed=43)
    f = normal((b, tt, hkv, 64), seed=44)
    qd, kd, vd = t(q, dev, dt), t(k, dev, dt), t(v, dev, dt)
    topk = None
    if mode in ("masked_forecast", "chunked_forecast"):
        reps = ops.compress_blocks(kd.float().transpose(1, 2), 64)
        _, topk = ops.select_blocks(t(f, dev), reps, 8, 64, mode == "masked_forecast" and causal)
    lists, counts = ops.prefill_lists(mode, b, hkv, tt, 64, 8, topk, causal, device=dev)
    row_topk = topk if mode == "masked_forecast" else None
    got = ops.prefill_attention(qd, kd, vd, lists, counts, 64, row_topk, causal)
    ref = ops.prefill_attention(qd.float(), kd.float(), vd.float(), lists, counts, 64, row_topk, causal)
    assert torch.isfinite(got.float()).all()
    np.testing.assert_allclose(n(got), n(ref), rtol=0, atol=2e-2)
    if mode == "masked_forecast" and causal:
        oref = O.masked_prefill(n(qd).transpose(0, 2, 1, 3), n(kd), n(vd), f, 64, 8, layer_idx=1)
        np.testing.assert_allclose(n(got), oref.transpose(0, 2, 1, 3), rtol=0, atol=2e-2)
