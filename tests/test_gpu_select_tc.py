"""The tensor-core many-row selector (sd_select_blocks without a score tensor,
bf16 forecast, D = 64, top-k <= 8: the prefill path) against the oracle's
float64 scores (model/forecast.py:89-130).  Tolerance: the chosen indices
equal the oracle's top-k wherever the slot is not a near-tie (relative score
gap <= 1e-5 to a neighbour: the split-bf16 tensor-core sums round differently
from float64), including the -inf slots, which follow the ascending-index
rule exactly.  Also agreement with the CUDA-core kernel (the score-tensor
path).  Needs a B200."""

import numpy as np
import pytest
import torch

from local_research_small_language_model_b200 import ops
from oracle import sparda_oracle as O
from oracle.synthetic import normal

pytestmark = pytest.mark.gpu


def _check_vs_oracle(f, r, k, causal, q_offset, idx):
    ref_s, ref_i = O.select_blocks(f.float().cpu().numpy(), r.cpu().numpy(), k, 64, causal, q_offset)
    got = idx.cpu().numpy().astype(np.int64)
    vals = np.take_along_axis(ref_s, ref_i, axis=-1)
    nxt = np.concatenate([vals[..., 1:], np.full(vals.shape[:-1] + (1,), -np.inf)], axis=-1)
    prv = np.concatenate([np.full(vals.shape[:-1] + (1,), np.inf), vals[..., :-1]], axis=-1)
    scale = np.maximum(np.abs(vals), 1e-30)
    with np.errstate(invalid="ignore"):
        near = np.isfinite(vals) & (((vals - nxt) <= 1e-5 * scale) | ((prv - vals) <= 1e-5 * scale))
    clear = ~near
    assert np.array_equal(got[clear], ref_i[clear])
    # the chosen blocks' oracle scores equal the oracle's best scores
    got_vals = np.take_along_axis(ref_s, np.where(got < 0, 0, got), axis=-1)
    fin = np.isfinite(vals)
    np.testing.assert_allclose(got_vals[fin], vals[fin], rtol=1e-5, atol=1e-6)
    return clear.mean()


@pytest.mark.parametrize("tq,nb,k,causal,q_offset", [
    (256, 2, 8, True, 0),        # fewer visible blocks than k: -inf fills
    (300, 5, 5, True, 0),        # ragged last tile
    (4096, 64, 8, True, 0),
    (4096, 64, 8, False, 0),
    (1000, 80, 3, True, 4096),   # chunked prefill: rows start past the cache
    (2048, 200, 8, False, 0),    # several 128-block chunks
    (260, 300, 1, True, 16000),
])
@torch.no_grad()
def test_tensor_core_selector_vs_oracle(dev, tq, nb, k, causal, q_offset):
    b, h = 2, 4
    f = torch.from_numpy(normal((b, tq, h, 64), seed=tq + nb)).to(dev, torch.bfloat16)
    r = torch.from_numpy(normal((b, nb, h, 64), seed=tq + nb + 1) * 0.3).to(dev, torch.float32)
    _, idx = ops.select_blocks(f, r, k, 64, causal, q_offset, return_scores=False)
    ops.check_device_errors(dev)
    frac = _check_vs_oracle(f, r, k, causal, q_offset, idx)
    assert frac > 0.9


@torch.no_grad()
def test_tensor_core_selector_agrees_with_cuda_core_kernel(dev):
    """Config-3-shaped layer (32,768 rows x 512 blocks x 4 heads): the two
    kernels choose the same blocks in >= 99.9 % of the slots, and every
    disagreement is a near-tie of the CUDA-core kernel's fp32 scores."""
    g = torch.Generator(device=dev).manual_seed(3)
    f = torch.randn(1, 32768, 4, 64, generator=g, device=dev).to(torch.bfloat16)
    r = 0.3 * torch.randn(1, 512, 4, 64, generator=g, device=dev)
    _, idx_tc = ops.select_blocks(f, r, 8, 64, True, return_scores=False)
    s_cc, idx_cc = ops.select_blocks(f, r, 8, 64, True, return_scores=True)
    ops.check_device_errors(dev)
    same = (idx_tc == idx_cc)
    rate = same.float().mean().item()
    assert rate >= 0.999, rate
    if not bool(same.all()):
        bad = ~same
        a = torch.gather(s_cc, -1, idx_tc.clamp_min(0))[bad]
        c = torch.gather(s_cc, -1, idx_cc.clamp_min(0))[bad]
        rel = ((a - c).abs() / c.abs().clamp_min(1e-30))
        assert bool((rel <= 1e-5).all()), rel.max().item()
