"""Backward of the block-sparse prefill attention (sd_prefill_attention_backward)
and training through B200SparseAttention / SparDAB200Model.

Checked against (1) the gradients autograd took through the reference itself
(tests/golden/backward.npz, fp32, loss = sum(out * w)), (2) the float64 oracle
(oracle.attention_backward) on the allowed mask of the kernel's own block
lists, in fp32 and bf16, and (3) a plain PyTorch fp32 autograd restatement of
the module (projections, RoPE, masked softmax attention, wo).  The kernel
computes in fp32 from the inputs' values, so every comparison uses fp32-level
tolerances: 1e-4 relative plus 1e-4 absolute (gradients are O(1) to O(10)).
Needs a B200."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import local_research_small_language_model_b200 as sd
from local_research_small_language_model_b200 import ops
from local_research_small_language_model_b200.model import SparDAB200Model
from local_research_small_language_model_b200.rope import apply_rotary_emb
from oracle import sparda_oracle as O
from tests.golden.make_golden import BACKWARD_CASES
from tests.test_oracle_golden import backward_inputs, oracle_backward_allowed

pytestmark = pytest.mark.gpu

TOL = dict(rtol=1e-4, atol=1e-4)


def n(x):
    return x.detach().float().cpu().numpy().astype(np.float64)


def _allowed_of_lists(attn, lists, counts, row_topk, causal, k, f, t, chunked):
    """The allowed mask [B,H,T,T] that the kernel's lists describe, built by the
    oracle's restatements of the reference's masks."""
    if chunked:
        return O.chunked_allowed(lists.cpu().numpy(), counts.cpu().numpy(), t, 64)
    if row_topk is not None:
        return O.masked_allowed_from_topk(row_topk.cpu().numpy(), t, 64, causal)
    # dense or static window: no selection involved
    allowed, _, _ = O.masked_allowed(None, k, t, 64, 8, attn.layer_idx, attn.mode, causal)
    return allowed


def _backward_case(dev, dtype, case):
    name, b, t, li, mode, with_f, chunked, seed = case
    q, k, v, f, dout = backward_inputs(b, t, with_f, seed)

    def cuda(x):
        return torch.from_numpy(np.ascontiguousarray(x)).to(dev, dtype)

    qd, kd, vd, gd = cuda(q.transpose(0, 2, 1, 3)), cuda(k), cuda(v), cuda(dout.transpose(0, 2, 1, 3))
    fd = cuda(f) if f is not None else None
    attn = sd.B200SparseAttention(sd.ModelConfig(block_size=64, top_k_blocks=8), li, mode=mode).to(dev)
    lists, counts, row_topk, causal = attn.block_lists(kd.transpose(1, 2).contiguous(), fd, True, chunked)
    dq, dk, dv = ops.prefill_attention_backward(qd, kd, vd, gd, lists, counts, 64, row_topk, causal)
    ops.check_device_errors(dev)
    # the oracle on the values the kernel saw, with the kernel's own mask
    qn, kn, vn, gn = n(qd).transpose(0, 2, 1, 3), n(kd), n(vd), n(gd).transpose(0, 2, 1, 3)
    allowed = _allowed_of_lists(attn, lists, counts, row_topk, causal, kn, n(fd) if fd is not None else None, t,
                                chunked)
    rq, rk, rv = O.attention_backward(qn, kn, vn, gn, allowed)
    return (n(dq).transpose(0, 2, 1, 3), n(dk), n(dv)), (rq, rk, rv), allowed


@pytest.mark.parametrize("case", BACKWARD_CASES, ids=[c[0] for c in BACKWARD_CASES])
def test_backward_vs_reference_gradients(dev, golden, case):
    """fp32: the kernel's gradients equal the reference's autograd gradients
    (masked forecast, static window, dense layer 0, chunked), and its lists
    describe the same allowed pairs as the oracle's own selection."""
    name, b, t, li, mode, with_f, chunked, seed = case
    (dq, dk, dv), _, allowed = _backward_case(dev, torch.float32, case)
    _, k, _, f, _ = backward_inputs(b, t, with_f, seed)
    assert np.array_equal(np.broadcast_to(allowed, (b, 4, t, t)),
                          np.broadcast_to(oracle_backward_allowed(k, f, t, li, mode, chunked), (b, 4, t, t)))
    g = golden("backward")
    for got, key, every in ((dq, "dq", 29), (dk, "dk", 13), (dv, "dv", 13)):
        np.testing.assert_allclose(got[:, :, ::every], g[f"{name}_{key}_rows"], **TOL)
        np.testing.assert_allclose(got.sum(-1), g[f"{name}_{key}_sum"], rtol=1e-4, atol=5e-4)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("case", BACKWARD_CASES, ids=[c[0] for c in BACKWARD_CASES])
def test_backward_vs_oracle(dev, case, dtype):
    """The kernel's gradients equal the float64 oracle's on the same inputs and
    allowed mask (bf16 inputs: the oracle sees the same bf16 values)."""
    got, ref, _ = _backward_case(dev, dtype, case)
    for a, r in zip(got, ref):
        np.testing.assert_allclose(a, r, **TOL)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16], ids=["f32", "bf16", "f16"])
@torch.no_grad()
def test_backward_ragged_batch_and_gqa_groups(dev, dtype):
    """B = 3 sequences of T = 130 (a 2-row last q-block), G = 1, 2 and 4
    query heads per kv head, chunked and masked lists: against the oracle.
    16-bit inputs run S and dP on the tensor cores, fp32 inputs on CUDA cores."""
    g = torch.Generator(device=dev).manual_seed(5)
    for hq, hkv in ((4, 4), (8, 4), (8, 2)):
        b, t = 3, 130
        q = torch.randn(b, t, hq, 64, generator=g, device=dev).to(dtype)
        k = torch.randn(b, hkv, t, 64, generator=g, device=dev).to(dtype)
        v = torch.randn(b, hkv, t, 64, generator=g, device=dev).to(dtype)
        go = torch.randn(b, t, hq, 64, generator=g, device=dev).to(dtype)
        f = torch.randn(b, t, hkv, 64, generator=g, device=dev).to(dtype)
        for chunked in (False, True):
            reps = ops.compress_blocks(k.transpose(1, 2).contiguous(), 64)
            _, topk = ops.select_blocks(f, reps, 2, 64, not chunked, return_scores=False)
            mode = "chunked_forecast" if chunked else "masked_forecast"
            lists, counts = ops.prefill_lists(mode, b, hkv, t, 64, 2, topk, True)
            row_topk = None if chunked else topk
            dq, dk, dv = ops.prefill_attention_backward(q, k, v, go, lists, counts, 64, row_topk, True)
            ops.check_device_errors(dev)
            if chunked:
                allowed = O.chunked_allowed(lists.cpu().numpy(), counts.cpu().numpy(), t, 64)
            else:
                allowed = O.masked_allowed_from_topk(topk.cpu().numpy(), t, 64, True)
            rq, rk, rv = O.attention_backward(n(q).transpose(0, 2, 1, 3), n(k), n(v), n(go).transpose(0, 2, 1, 3),
                                              allowed)
            np.testing.assert_allclose(n(dq).transpose(0, 2, 1, 3), rq, **TOL)
            np.testing.assert_allclose(n(dk), rk, **TOL)
            np.testing.assert_allclose(n(dv), rv, **TOL)


def _torch_module_reference(attn, x, rot, f, w, t):
    """PyTorch fp32 autograd restatement of the module's prefill (projections,
    RoPE, masked GQA softmax attention over the module's own allowed mask, wo),
    with its own copies of the weights.  Returns (x grad, {name: weight grad})."""
    xr = x.detach().clone().requires_grad_(True)
    ws = {nm: getattr(attn, nm).weight.detach().clone().requires_grad_(True) for nm in ("wq", "wk", "wv", "wo")}
    b = x.shape[0]
    q = F.linear(xr, ws["wq"]).view(b, t, 12, 64)
    k = F.linear(xr, ws["wk"]).view(b, t, 4, 64)
    v = F.linear(xr, ws["wv"]).view(b, t, 4, 64)
    q, k = apply_rotary_emb(q, k, rot.cos, rot.sin)
    with torch.no_grad():
        lists, counts, row_topk, causal = attn.block_lists(k.detach().contiguous(), f, True, False)
        allowed = _allowed_of_lists(attn, lists, counts, row_topk, causal, n(k).transpose(0, 2, 1, 3), None, t,
                                    False)
    mask = torch.from_numpy(np.broadcast_to(allowed, (b, 4, t, t)).copy()).to(x.device)
    mask = mask.repeat_interleave(3, dim=1)
    kk = k.transpose(1, 2).repeat_interleave(3, dim=1)
    vv = v.transpose(1, 2).repeat_interleave(3, dim=1)
    s = torch.einsum("bhtd,bhsd->bhts", q.transpose(1, 2), kk) / 8.0
    p = torch.softmax(s.masked_fill(~mask, float("-inf")), dim=-1)
    o = torch.einsum("bhts,bhsd->bhtd", p, vv).transpose(1, 2).reshape(b, t, 768)
    (F.linear(o, ws["wo"]) * w).sum().backward()
    return xr.grad, {nm: ws[nm].grad for nm in ws}


@pytest.mark.parametrize("t,layer_idx,mode", [(64, 1, "forecast"), (256, 1, "forecast"), (300, 1, "static"),
                                              (192, 0, "forecast")])
def test_module_gradients_match_torch_autograd(dev, t, layer_idx, mode):
    """tests/test_sparse_attention.py:63-77 on this backend: x.grad exists and
    is finite after out.sum()-style backward, and x's and the projections'
    gradients equal a PyTorch fp32 autograd restatement of the module."""
    torch.manual_seed(11)
    attn = sd.B200SparseAttention(sd.ModelConfig(block_size=64, top_k_blocks=8), layer_idx, mode=mode).to(dev)
    rot = sd.RotaryEmbedding(64, t).to(dev)
    b = 2
    x = torch.randn(b, t, 768, device=dev, requires_grad=True)
    f = torch.randn(b, t, 4, 64, device=dev)
    out = attn(x, rotary_emb=rot, forecast_vector=f)
    assert out.shape == (b, t, 768)
    w = torch.randn_like(out)
    (out * w).sum().backward()
    ops.check_device_errors(dev)
    assert x.grad is not None and bool(torch.isfinite(x.grad).all())
    gx, gws = _torch_module_reference(attn, x, rot, f, w, t)
    np.testing.assert_allclose(n(x.grad), n(gx), rtol=1e-3, atol=1e-3)
    for nm, gw in gws.items():
        got = getattr(attn, nm).weight.grad
        assert got is not None
        np.testing.assert_allclose(n(got), n(gw), rtol=1e-3, atol=1e-3)


def test_model_forward_backward(dev):
    """Whole-model training step (the reference's model forward/backward test):
    cross-entropy loss over a 2-layer model with sparse attention past the
    dense regime; every attention and FFN weight receives a finite, nonzero
    gradient, and the kernels' paths were the ones taken (no graph break)."""
    torch.manual_seed(2)
    cfg = sd.ModelConfig(n_layer=2, block_size=64, top_k_blocks=2)
    model = SparDAB200Model(cfg).to(dev)
    ids = torch.randint(0, cfg.vocab_size, (2, 320), device=dev)
    out = model(ids, targets=ids)
    out["loss"].backward()
    ops.check_device_errors(dev)
    assert bool(torch.isfinite(out["loss"]))
    for layer in model.layers:
        for w in (layer.attention.wq.weight, layer.attention.wk.weight, layer.attention.wv.weight,
                  layer.attention.wo.weight, layer.ffn.w_down.weight, layer.attn_norm.weight):
            assert w.grad is not None and bool(torch.isfinite(w.grad).all()) and float(w.grad.abs().sum()) > 0


def test_gradients_through_a_cache_are_refused(dev):
    attn = sd.B200SparseAttention(sd.ModelConfig(block_size=64, top_k_blocks=8), 1).to(dev)
    rot = sd.RotaryEmbedding(64, 128).to(dev)
    cache = sd.B200KVCache(1, 128, 4, 64, device=dev, dtype=torch.float32)
    x = torch.randn(1, 128, 768, device=dev, requires_grad=True)
    with pytest.raises(NotImplementedError):
        attn(x, rotary_emb=rot, kv_cache=cache)
