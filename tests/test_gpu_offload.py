"""Offloaded KV caches (model/attention/offload.py, async_offload.py) on the B200
path: K/V rows in pinned host memory, forecast-guided prefetch into device
slots on a side stream, fused decode reading the slots.  Decoding with
offloaded caches must give the same logits, bit for bit, as decoding with
device-resident caches (same selection, same kernels, same data), and the host
store must hold every row the device cache holds.  Needs a B200."""

import numpy as np
import pytest
import torch

import local_research_small_language_model_b200 as sd
from local_research_small_language_model_b200.model import DecodeEngine, SparDAB200Model
from local_research_small_language_model_b200.offload import B200OffloadKVCache
from oracle.synthetic import SmallModelConfig, model_state

pytestmark = pytest.mark.gpu


def _model(dev, rule, seed=7):
    sc = SmallModelConfig()
    cfg = sd.ModelConfig(vocab_size=sc.vocab_size, n_layer=sc.n_layer, context_length=sc.context_length,
                         block_size=64, top_k_blocks=8, selector_rule=rule)
    m = SparDAB200Model(cfg)
    m.load_state_dict({k: torch.from_numpy(v) for k, v in model_state(sc, seed=seed).items()})
    return m.to(dev, torch.bfloat16).eval(), sc


def _prefill(caches, b, pre, dev, seed):
    gen = torch.Generator(device="cpu").manual_seed(seed)
    kv = []
    for _ in caches[0]:
        kv.append((torch.randn(b, pre, 4, 64, generator=gen).to(dev, torch.bfloat16),
                   torch.randn(b, pre, 4, 64, generator=gen).to(dev, torch.bfloat16)))
    for cs in caches:
        for c, (k, v) in zip(cs, kv):
            c.update(k, v)


@pytest.mark.parametrize("rule", ["reference", "absolute"])
@torch.no_grad()
def test_offload_decode_matches_device_cache(dev, rule):
    """70 steps from 900 cached tokens (crossing the block boundary at 960):
    identical logits, identical host store and block sums."""
    m1, sc = _model(dev, rule)
    m2, _ = _model(dev, rule)
    b, pre = 3, 900
    c1 = m1.allocate_caches(b, 2048)
    c2 = m2.allocate_caches(b, 2048, offload=True)
    assert all(isinstance(c, B200OffloadKVCache) for c in c2)
    _prefill([c1, c2], b, pre, dev, seed=5)
    ids = torch.randint(0, sc.vocab_size, (b, 1), generator=torch.Generator(device="cpu").manual_seed(3)).to(dev)
    for step in range(70):
        l1 = m1(ids, kv_caches=c1)["logits"]
        l2 = m2(ids, kv_caches=c2)["logits"]
        assert torch.equal(l1, l2), f"step {step}"
        ids = l1[:, -1:].argmax(-1)
    sd.ops.check_device_errors(dev)
    torch.cuda.synchronize()
    L = pre + 70
    for a, o in zip(c1, c2):
        assert o.current_len == a.current_len == L
        assert torch.equal(o.host_k[:, :, :L], a.k_store[:, :, :L].cpu())
        assert torch.equal(o.host_v[:, :, :L], a.v_store[:, :, :L].cpu())
        assert torch.equal(o.proto_sum, a.proto_sum)
    st = c2[1].stats.cpu().tolist()
    assert 0 <= st[1] <= st[0] and st[2] % (2 * 64 * 64 * 2) == 0 and st[2] > 0
    assert 0.0 <= c2[1].hit_rate() <= 1.0


@torch.no_grad()
def test_offload_graph_engine_matches_eager(dev):
    """The CUDA-graph decode step (prefetch on the side stream inside the
    graph) gives the same tokens as eager decode on offloaded caches."""
    m1, sc = _model(dev, "absolute")
    m2, _ = _model(dev, "absolute")
    b, pre = 4, 1000
    c1 = m1.allocate_caches(b, 2048, offload=True)
    c2 = m2.allocate_caches(b, 2048, offload=True)
    _prefill([c1, c2], b, pre, dev, seed=9)
    ids = torch.randint(0, sc.vocab_size, (b, 1), generator=torch.Generator(device="cpu").manual_seed(4)).to(dev)
    eng = DecodeEngine(m2, c2, b)
    eng.ids.copy_(ids)
    eng.capture()
    cur = ids
    for step in range(8):
        nxt = m1(cur, kv_caches=c1)["logits"][:, -1:].argmax(-1)
        got = eng.step().clone()
        assert torch.equal(nxt, got), f"step {step}"
        cur = nxt
    sd.ops.check_device_errors(dev)


@torch.no_grad()
def test_transfer_selected_blocks_reads_host_store(dev):
    """OffloadedKVCache.transfer_selected_blocks (offload.py:83-123): the
    gathered blocks equal the host rows, read by the GPU in place."""
    b, L = 2, 700
    c = B200OffloadKVCache(b, 1024, 4, 64, dev, torch.bfloat16)
    gen = torch.Generator(device="cpu").manual_seed(11)
    k = torch.randn(b, L, 4, 64, generator=gen).to(dev, torch.bfloat16)
    v = torch.randn(b, L, 4, 64, generator=gen).to(dev, torch.bfloat16)
    c.update(k, v)
    idx = torch.tensor([[[0, 3, 10, -1]] * 4] * b, dtype=torch.int64, device=dev)
    gk, gv, nbytes = c.transfer_selected_blocks(idx, 64)
    torch.cuda.synchronize()
    assert nbytes == 2 * b * 4 * 4 * 64 * 64 * 2
    kh = k.transpose(1, 2).cpu()
    for s, j in enumerate([0, 3, 10]):
        n = min(64, L - j * 64)
        assert torch.equal(gk[:, :, s * 64:s * 64 + n].cpu(), kh[:, :, j * 64:j * 64 + n])
    assert torch.count_nonzero(gk[:, :, 3 * 64:].float()) == 0  # the invalid slot is zero-filled
