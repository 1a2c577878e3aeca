"""The tensor-core projections of the decode step (sd_linear) against a
plain PyTorch fp32 reference on the same 16-bit inputs: RMSNorm prologue
(model/norm.py:15-21), store / residual (transformer.py:118-129) / SwiGLU
(transformer.py:18-31) epilogues.  Tolerance: one 16-bit rounding of the
output (the fp32 accumulation order differs).  Needs a B200."""

import pytest
import torch
import torch.nn.functional as F

from local_research_small_language_model_b200 import ops

pytestmark = pytest.mark.gpu


def _rms(x, w, eps=1e-6):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).type_as(x) * w


def _close(got, ref):
    tol = 8e-3 if got.dtype == torch.bfloat16 else 1e-3
    torch.testing.assert_close(got.float(), ref.float(), rtol=tol, atol=tol * ref.float().abs().max().item() * 0.05 + 1e-5)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,k,n,norm", [(64, 768, 1536, True), (64, 768, 768, False), (1, 768, 1536, True),
                                        (100, 768, 4096, True), (130, 2048, 768, False), (64, 768, 32000, True)])
@torch.no_grad()
def test_linear_store(dev, dt, m, k, n, norm):
    g = torch.Generator(device=dev).manual_seed(m + k + n)
    x = torch.randn(m, k, generator=g, device=dev).to(dt)
    w = (0.02 * torch.randn(n, k, generator=g, device=dev)).to(dt)
    nw = (1 + 0.1 * torch.randn(k, generator=g, device=dev)).to(dt) if norm else None
    got = ops.linear(x, w, nw)
    xn = _rms(x, nw) if norm else x
    ref = (xn.float() @ w.float().t()).to(dt)
    _close(got, ref)
    ops.check_device_errors(dev)


@pytest.mark.parametrize("m,k", [(64, 768), (64, 2048), (200, 768)])
@torch.no_grad()
def test_linear_residual_in_place(dev, m, k):
    dt = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(7 + k)
    h = torch.randn(m, k, generator=g, device=dev).to(dt)
    w = (0.02 * torch.randn(768, k, generator=g, device=dev)).to(dt)
    x = torch.randn(m, 768, generator=g, device=dev).to(dt)
    acc = h.float() @ w.float().t()
    ref = x + acc.to(dt)  # the reference's x + Linear(h) in the activation dtype
    x2 = x.clone()
    got = ops.linear(h, w, epilogue="residual", res=x2, out=x2)
    assert got.data_ptr() == x2.data_ptr()
    # the projection may round one ulp apart (accumulation order), and an ulp
    # of the projection can exceed one of the sum
    ulp = 2.0 ** -7 * acc.abs().max().item()
    torch.testing.assert_close(got.float(), ref.float(), rtol=8e-3, atol=ulp)


@pytest.mark.parametrize("m", [1, 64, 77])
@torch.no_grad()
def test_linear_swiglu_with_norm(dev, m):
    dt = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(11 + m)
    x = torch.randn(m, 768, generator=g, device=dev).to(dt)
    wg = (0.02 * torch.randn(2048, 768, generator=g, device=dev)).to(dt)
    wu = (0.02 * torch.randn(2048, 768, generator=g, device=dev)).to(dt)
    nw = (1 + 0.1 * torch.randn(768, generator=g, device=dev)).to(dt)
    got = ops.linear(x, ops.swiglu_weight(wg, wu), nw, epilogue="swiglu")
    xn = _rms(x, nw)
    gate = (xn.float() @ wg.float().t()).to(dt)
    up = (xn.float() @ wu.float().t()).to(dt)
    ref = F.silu(gate) * up
    assert got.shape == (m, 2048)
    # gate and up may each round one ulp apart (accumulation order): allow
    # the product to move by about two ulps
    torch.testing.assert_close(got.float(), ref.float(), rtol=2e-2, atol=2.0 ** -8)


@torch.no_grad()
def test_linear_norm_prologue_matches_rmsnorm_kernel(dev):
    """The fused prologue normalises as sd_rmsnorm does (the sum of squares may
    round differently in its last bit): with an identity weight the
    projection returns the normalised rows."""
    dt = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(64, 768, generator=g, device=dev).to(dt)
    nw = (1 + 0.1 * torch.randn(768, generator=g, device=dev)).to(dt)
    eye = torch.eye(768, device=dev, dtype=dt)
    torch.testing.assert_close(ops.linear(x, eye, nw).float(), ops.rmsnorm(x, nw, 1e-6).float(), rtol=8e-3, atol=1e-2)


@torch.no_grad()
def test_linear_rejects_unsupported_shapes(dev):
    x = torch.randn(8, 96, device=dev, dtype=torch.bfloat16)  # K not a multiple of 64
    with pytest.raises(Exception):
        ops.linear(x, torch.randn(128, 96, device=dev, dtype=torch.bfloat16))
    x = torch.randn(8, 2048, device=dev, dtype=torch.bfloat16)  # RMSNorm prologue limited to K <= 1024
    with pytest.raises(Exception):
        ops.linear(x, torch.randn(128, 2048, device=dev, dtype=torch.bfloat16),
                   torch.ones(2048, device=dev, dtype=torch.bfloat16))


@pytest.mark.parametrize("m", [3, 64])
@torch.no_grad()
def test_decode_step_with_fused_projections(dev, m):
    """The model's decode step with every projection on sd_linear (RMSNorm
    prologue, residual and SwiGLU epilogues, LM head) against the default
    cuBLAS path: the same greedy tokens and logits within bf16 rounding, in
    eager mode and replayed as a CUDA graph."""
    import local_research_small_language_model_b200 as sd
    from local_research_small_language_model_b200.model import DecodeEngine, SparDAB200Model
    cfg = sd.ModelConfig(vocab_size=1024, n_layer=3, block_size=64, top_k_blocks=8, selector_rule="absolute")
    torch.manual_seed(5)
    m1 = SparDAB200Model(cfg).to(dev, torch.bfloat16).eval()
    m2 = SparDAB200Model(cfg).to(dev, torch.bfloat16).eval()
    m2.load_state_dict(m1.state_dict())
    for layer in m2.layers:
        layer.use_tc_linear = True
    c1, c2 = m1.allocate_caches(m, 1024), m2.allocate_caches(m, 1024)
    gen = torch.Generator(device="cpu").manual_seed(2)
    for a, b in zip(c1, c2):
        k = torch.randn(m, 700, 4, 64, generator=gen).to(dev, torch.bfloat16)
        v = torch.randn(m, 700, 4, 64, generator=gen).to(dev, torch.bfloat16)
        a.update(k, v)
        b.update(k, v)
    ids = torch.randint(0, cfg.vocab_size, (m, 1), generator=gen).to(dev)
    for step in range(3):
        l1 = m1(ids, kv_caches=c1)["logits"][:, -1].float()
        l2 = m2(ids, kv_caches=c2)["logits"][:, -1].float()
        torch.testing.assert_close(l2, l1, rtol=0.05, atol=0.05 * l1.abs().max().item())
        ids = l1.argmax(-1, keepdim=True)
    ops.check_device_errors(dev)
    # graph replay of the fused path against its own eager step (same kernels)
    m3 = SparDAB200Model(cfg).to(dev, torch.bfloat16).eval()
    m3.load_state_dict(m1.state_dict())
    for layer in m3.layers:
        layer.use_tc_linear = True
    c3 = m3.allocate_caches(m, 1024)
    for a, b in zip(c2, c3):
        b.update(a.k[:, :a.current_len], a.v[:, :a.current_len])
    m3._lens.copy_(m2._lens)
    eng = DecodeEngine(m2, c2, m)
    eng.ids.copy_(ids)
    eng.capture()
    got = eng.step().clone()
    ref = m3(ids, kv_caches=c3)["logits"][:, -1:].argmax(-1)
    assert torch.equal(got, ref)
    ops.check_device_errors(dev)
