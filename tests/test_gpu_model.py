"""End-to-end parity of the B200 model driver: logits against the reference
model's own golden logits, the generic (reference-cache) decode path against
the fused one, and the CUDA-graph engine against eager decode.  Needs a B200."""

import numpy as np
import pytest
import torch

import local_research_small_language_model_b200 as sd
from local_research_small_language_model_b200.model import DecodeEngine, SparDAB200Model
from oracle.synthetic import SmallModelConfig, model_state

pytestmark = pytest.mark.gpu


def _model(dev, dtype=torch.float32, seed=7, rule="reference"):
    sc = SmallModelConfig()
    cfg = sd.ModelConfig(vocab_size=sc.vocab_size, n_layer=sc.n_layer, context_length=sc.context_length,
                         block_size=sc.block_size, top_k_blocks=sc.top_k_blocks, selector_rule=rule)
    m = SparDAB200Model(cfg)
    m.load_state_dict({k: torch.from_numpy(v) for k, v in model_state(sc, seed=seed).items()})
    return m.to(dev, dtype).eval(), sc


@torch.no_grad()
def test_model_decode_logits_match_reference(dev, golden):
    """Token-by-token decode from an empty cache: logits vs the reference model
    (CPU fp32) at the golden steps (dense-fallback region, tie-free)."""
    from tests.golden.make_golden import MODEL_STEPS
    g = golden("model_decode")
    m, sc = _model(dev)
    ids = torch.from_numpy(g["ids"].astype(np.int64)).to(dev)
    caches = m.allocate_caches(ids.shape[0], 1024)
    for s in range(max(MODEL_STEPS) + 1):
        lg = m(ids[:, s:s + 1], kv_caches=caches)["logits"][:, 0]
        if s in MODEL_STEPS:
            np.testing.assert_allclose(lg.cpu().numpy(), g[f"step{s}"], rtol=0, atol=2e-4, err_msg=f"step {s}")
    sd.ops.check_device_errors(dev)
    assert all(c.current_len == max(MODEL_STEPS) + 1 for c in caches)
    assert torch.equal(m._lens.cpu(), torch.full((sc.n_layer,), max(MODEL_STEPS) + 1, dtype=torch.int32))


class RefStyleKVCache:
    """The reference's KVCache layout and API (model/attention/base.py:11-32)."""

    def __init__(self, b, tmax, h, d, device, dtype):
        self.k = torch.zeros(b, tmax, h, d, device=device, dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.current_len = 0

    def update(self, xk, xv):
        s, e = self.current_len, self.current_len + xk.shape[1]
        self.k[:, s:e] = xk
        self.v[:, s:e] = xv
        self.current_len = e
        return self.k[:, :e], self.v[:, :e]


@pytest.mark.parametrize("rule", ["reference", "absolute"])
@torch.no_grad()
def test_generic_decode_path_matches_fused(dev, rule):
    """B200SparseAttention on the reference's own cache object (unfused
    kernels) vs the fused kernel on a B200KVCache: same outputs."""
    torch.manual_seed(0)
    cfg = sd.ModelConfig(block_size=64, top_k_blocks=8, selector_rule=rule)
    attn = sd.B200SparseAttention(cfg, layer_idx=1).to(dev)
    rot = sd.RotaryEmbedding(64, 4096).to(dev)
    b, pre = 2, 1100
    c1 = RefStyleKVCache(b, 4096, 4, 64, dev, torch.float32)
    c2 = sd.B200KVCache(b, 4096, 4, 64, dev, torch.float32)
    k0, v0 = torch.randn(b, pre, 4, 64, device=dev), torch.randn(b, pre, 4, 64, device=dev)
    c1.update(k0, v0)
    c2.update(k0, v0)
    for step in range(4):
        x = torch.randn(b, 1, 768, device=dev)
        f = torch.randn(b, 1, 4, 64, device=dev)
        o1 = attn(x, rot, kv_cache=c1, forecast_vector=f)
        o2 = attn(x, rot, kv_cache=c2, forecast_vector=f)
        torch.testing.assert_close(o1, o2, rtol=0, atol=1e-4)
    assert c1.current_len == c2.current_len == pre + 4


@torch.no_grad()
def test_decode_engine_graph_matches_eager(dev):
    m1, sc = _model(dev, torch.bfloat16, rule="absolute")
    m2, _ = _model(dev, torch.bfloat16, rule="absolute")
    b, pre = 4, 900
    c1, c2 = m1.allocate_caches(b, 2048), m2.allocate_caches(b, 2048)
    gen = torch.Generator(device="cpu").manual_seed(1)
    for c_a, c_b in zip(c1, c2):
        k = torch.randn(b, pre, 4, 64, generator=gen).to(dev, torch.bfloat16)
        v = torch.randn(b, pre, 4, 64, generator=gen).to(dev, torch.bfloat16)
        c_a.update(k, v)
        c_b.update(k, v)
    ids = torch.randint(0, sc.vocab_size, (b, 1), generator=gen).to(dev)
    eng = DecodeEngine(m2, c2, b)
    eng.ids.copy_(ids)
    eng.capture()
    assert all(c.current_len == pre for c in c2)
    cur = ids
    for step in range(6):
        nxt = m1(cur, kv_caches=c1)["logits"][:, -1:].argmax(-1)
        got = eng.step().clone()
        assert torch.equal(nxt, got), f"step {step}"
        cur = nxt
    assert all(c.current_len == pre + 6 for c in c2)
    assert torch.equal(m1._lens, m2._lens)


@pytest.mark.parametrize("mode", ["side-stream", "chain"])
@pytest.mark.parametrize("rule", ["reference", "absolute"])
@torch.no_grad()
def test_overlapped_selection_matches_in_kernel_selection(dev, rule, mode):
    """Decode with layer L+1's candidates computed ahead of time (on the side
    stream during layer L, or at the end of layer L's fused kernel) gives
    bit-identical logits to decode with selection in the kernel."""
    m1, sc = _model(dev, torch.bfloat16, rule=rule)
    m2, _ = _model(dev, torch.bfloat16, rule=rule)
    b, pre = 3, 1500
    c1 = m1.allocate_caches(b, 2048, selection="kernel")
    c2 = m2.allocate_caches(b, 2048, selection=mode)
    gen = torch.Generator(device="cpu").manual_seed(2)
    for ca, cb in zip(c1, c2):
        k = torch.randn(b, pre, 4, 64, generator=gen).to(dev, torch.bfloat16)
        v = torch.randn(b, pre, 4, 64, generator=gen).to(dev, torch.bfloat16)
        ca.update(k, v)
        cb.update(k, v)
    ids = torch.randint(0, sc.vocab_size, (b, 1), generator=gen).to(dev)
    for step in range(5):
        l1 = m1(ids, kv_caches=c1)["logits"]
        l2 = m2(ids, kv_caches=c2)["logits"]
        assert torch.equal(l1, l2), f"step {step}"
        ids = l1[:, -1:].argmax(-1)
    sd.ops.check_device_errors(dev)
