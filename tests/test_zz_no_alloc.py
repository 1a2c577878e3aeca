"""sd_decode_sparse_noalloc (the unfused decode with its selected-block lists
in the library's fixed device scratch) called through the C ABI, against the
two caller-buffer entry points it chains (sd_decode_select +
sd_decode_attention, through ops).  Both run the same kernels on the same
inputs, so the tolerance is zero: outputs must be bit-identical.  Two calls in
a row with different inputs check that nothing of the first call's lists
leaks into the second.  The file sorts last so it also runs after every other
GPU test in the same process; it passes alone as well.  Needs a B200."""

import ctypes

import numpy as np
import pytest
import torch

import local_research_small_language_model_b200 as sd
from local_research_small_language_model_b200 import _lib, ops
from oracle import sparda_oracle as O
from oracle.synthetic import normal

pytestmark = pytest.mark.gpu

SD_ERR_UNSUPPORTED = -2  # include/spardab200.h


def _call_noalloc(q, f, reps, kc, vc, L, top_k, rule, out, err):
    lib = sd.load_library()
    b, hq, d = q.shape
    hkv, tcap = kc.shape[1], kc.shape[2]
    fp = f.data_ptr() if f is not None else None
    rp = reps.data_ptr() if reps is not None else None
    return lib.sd_decode_sparse_noalloc(
        q.data_ptr(), ops.dtype_code(q), q.stride(0), q.stride(1),
        fp, ops.dtype_code(f) if f is not None else _lib.SD_DTYPE_F32, f.stride(0) if f is not None else 0,
        f.stride(1) if f is not None else 0,
        rp, reps.stride(0) if reps is not None else 0, reps.stride(1) if reps is not None else 0,
        reps.stride(2) if reps is not None else 0,
        kc.data_ptr(), vc.data_ptr(), kc.stride(0), kc.stride(1), kc.stride(2), tcap,
        b, hq, hkv, d, L, 64, top_k, ops.RULES[rule], ctypes.c_float(1.0 / 8.0), out.data_ptr(), out.stride(0),
        out.stride(1), err.data_ptr(), torch.cuda.current_stream(q.device).cuda_stream)


def _inputs(dev, b, hkv, L, seed):
    q = torch.from_numpy(normal((b, 3 * hkv, 64), seed=seed)).to(dev, torch.bfloat16)
    kc = torch.from_numpy(normal((b, hkv, 4096, 64), seed=seed + 1)).to(dev, torch.bfloat16)
    vc = torch.from_numpy(normal((b, hkv, 4096, 64), seed=seed + 2)).to(dev, torch.bfloat16)
    f = torch.from_numpy(normal((b, hkv, 64), seed=seed + 3)).to(dev, torch.bfloat16)
    reps = torch.from_numpy(O.compress_blocks(kc[:, :, :L].float().cpu().numpy().transpose(0, 2, 1, 3), 64))
    return q, kc, vc, f, reps.to(dev, torch.float32).contiguous()  # the oracle computes in float64


@pytest.mark.parametrize("rule", ["reference", "absolute"])
@torch.no_grad()
def test_noalloc_decode_matches_caller_buffer_entry_points(dev, rule):
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for call, (b, L, seed) in enumerate([(4, 3000, 11), (6, 1500, 23)]):
        q, kc, vc, f, reps = _inputs(dev, b, 4, L, seed)
        sel, cnt = ops.decode_select(f, reps, L, b, 4, 64, 64, 8, rule)
        ref = ops.decode_attention(q, kc, vc, sel, cnt, L, 64, scale=1.0 / 8.0)
        out = torch.full_like(ref, float("nan"))
        assert _call_noalloc(q, f, reps, kc, vc, L, 8, rule, out, err) == 0, f"call {call}"
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        torch.testing.assert_close(out, ref, rtol=0, atol=0)
    # static window (no forecast): the same lists as the caller-buffer path
    q, kc, vc, _, _ = _inputs(dev, 2, 4, 2000, 5)
    sel, cnt = ops.decode_select(None, None, 2000, 2, 4, 64, 64, 8, rule, device=dev)
    ref = ops.decode_attention(q, kc, vc, sel, cnt, 2000, 64, scale=1.0 / 8.0)
    out = torch.full_like(ref, float("nan"))
    assert _call_noalloc(q, None, None, kc, vc, 2000, 8, rule, out, err) == 0
    torch.cuda.synchronize()
    torch.testing.assert_close(out, ref, rtol=0, atol=0)


@torch.no_grad()
def test_noalloc_rejects_sizes_beyond_its_scratch(dev):
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    q, kc, vc, f, reps = _inputs(dev, 2, 4, 3000, 3)
    out = torch.empty_like(q)
    lib = sd.load_library()

    def raw(b, L, tcap, top_k):
        # both limits are checked before any pointer is read or kernel launched
        return lib.sd_decode_sparse_noalloc(q.data_ptr(), ops.dtype_code(q), 0, 0, f.data_ptr(), ops.dtype_code(f),
                                            0, 0, reps.data_ptr(), 0, 0, 0, kc.data_ptr(), vc.data_ptr(), 0, 0, 0,
                                            tcap, b, 12, 4, 64, L, 64, top_k, 1, ctypes.c_float(0.125),
                                            out.data_ptr(), 0, 0, err.data_ptr(), None)

    assert raw(2, 5000, 8192, 63) == SD_ERR_UNSUPPORTED   # 65 list entries per (sequence, kv head) > 64
    assert raw(1025, 3000, 4096, 8) == SD_ERR_UNSUPPORTED  # 4100 (sequence, kv head) pairs > 4096
    np.testing.assert_equal(int(err.item()), 0)
